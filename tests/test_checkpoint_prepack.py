"""Load-time conversion of per-expert checkpoint tensors (HF gate_proj /
up_proj / down_proj) into the op's K-major weight storage, against the
reference's own loader recipe (kernel_bench.py:212-235: cat(gate, up, dim=0),
stack over experts, transpose(1, 2)). Layout work is exact, so the bar is
bit-exact equality."""
import pytest
import torch

import mail_b200 as mb


def checkpoint(E, I, H, dtype=torch.bfloat16, seed=0):
    g = torch.Generator().manual_seed(seed)
    gate = [(torch.randn(I, H, generator=g) * 0.02).to(dtype) for _ in range(E)]
    up = [(torch.randn(I, H, generator=g) * 0.02).to(dtype) for _ in range(E)]
    down = [(torch.randn(H, I, generator=g) * 0.02).to(dtype) for _ in range(E)]
    return gate, up, down


def reference_recipe(gate, up, down):
    """kernel_bench.py:219-235, restated."""
    w13 = torch.stack([torch.cat([g, u], dim=0) for g, u in zip(gate, up)], dim=0).transpose(1, 2)
    w2 = torch.stack(list(down), dim=0).transpose(1, 2)
    return w13, w2


@pytest.mark.parametrize("E,I,H", [(4, 48, 64), (3, 16, 40), (1, 8, 8)])
def test_matches_reference_loader_bit_exact(E, I, H):
    gate, up, down = checkpoint(E, I, H)
    w13, w2 = mb.weights_from_checkpoint(gate, up, down)
    r13, r2 = reference_recipe(gate, up, down)
    assert w13.shape == (E, H, 2 * I) and w2.shape == (E, I, H)
    assert torch.equal(w13, r13) and torch.equal(w2, r2)
    # storage is K-major: the transposed views are contiguous [E, 2I, H] / [E, H, I]
    assert w13.transpose(1, 2).is_contiguous() and w2.transpose(1, 2).is_contiguous()
    # gate is the first I logical columns
    assert torch.equal(w13[0, :, :I], gate[0].t())


def test_stacked_inputs_and_dtype_cast():
    gate, up, down = checkpoint(2, 32, 24, dtype=torch.float32)
    w13, w2 = mb.weights_from_checkpoint(torch.stack(gate), torch.stack(up), torch.stack(down),
                                         dtype=torch.bfloat16)
    r13, r2 = reference_recipe(gate, up, down)
    assert w13.dtype == torch.bfloat16
    assert torch.equal(w13, r13.to(torch.bfloat16)) and torch.equal(w2, r2.to(torch.bfloat16))


def test_rejects_mismatched_shapes():
    gate, up, down = checkpoint(2, 16, 32)
    with pytest.raises(ValueError):
        mb.weights_from_checkpoint(gate, up[:1], down)
    with pytest.raises(ValueError):
        mb.weights_from_checkpoint(gate, up, [d.t() for d in down])


@pytest.mark.gpu
def test_quantized_checkpoint_matches_quantize_weights_int8():
    gate, up, down = checkpoint(4, 64, 128)
    q13, q2, (s13, s2) = mb.weights_from_checkpoint(gate, up, down, device="cuda", quantize=True)
    r13, r2 = reference_recipe(gate, up, down)
    e13, e2, (t13, t2) = mb.quantize_weights_int8(r13.cuda(), r2.cuda())
    assert q13.dtype == torch.int8 and torch.equal(q13, e13) and torch.equal(q2, e2)
    assert torch.equal(s13, t13) and torch.equal(s2, t2)
    # the op runs on them (w8a8) and agrees with the bf16 weights within the w8a8 tolerance
    x = torch.randn(64, 128, device="cuda").to(torch.bfloat16)
    ids = torch.randint(0, 4, (64, 2), device="cuda", dtype=torch.int32)
    ids[:, 1] = (ids[:, 0] + 1) % 4
    wts = torch.full((64, 2), 0.5, device="cuda")
    y8 = mb.fused_moe_mlp(x, q13, q2, wts, ids, scales=(s13, s2)).float()
    yb = mb.fused_moe_mlp(x, r13.cuda(), r2.cuda(), wts, ids).float()
    assert float((y8 - yb).abs().max() / yb.abs().max()) < 3e-2
