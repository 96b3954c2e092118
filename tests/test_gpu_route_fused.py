"""moe_fused_experts_from_logits: routing and the layer in one call. A
decode-sized batch (at most 16 tokens, E <= 256, bf16/fp16) routes inside
the one-launch decode kernel's first phase, so the whole layer is one launch;
other batches launch the router (moe_route_topk) first.

The routing it returns must be bit-identical to the stand-alone router's on
the same logits (ids and fp32 weights; integer and index work is held to
bit-exact), and the output must match the oracle on that routing and the
two-call path route_topk + fused_moe_mlp within max-abs-rel 1e-2, the bar of
every bf16/fp16 output here."""
import numpy as np
import pytest
import torch

import mail_b200 as mb
from mail_b200 import _lib
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2


def dev():
    return torch.device("cuda", 0)


def max_abs_rel(y, ref):
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


CASES = [
    # T, H, I, E, k, scoring, renormalize, logits dtype, x dtype, ties, one launch
    (1, 2048, 768, 128, 8, "softmax", True, torch.float32, torch.bfloat16, False, True),  # Qwen3 shape, one token
    (16, 2048, 768, 128, 8, "softmax", True, torch.bfloat16, torch.bfloat16, False, True),  # 128 slots
    (5, 1024, 256, 256, 8, "sigmoid", True, torch.float32, torch.bfloat16, False, True),  # E = 256: 8 logits a lane
    (3, 512, 136, 20, 2, "softmax", False, torch.float16, torch.float16, False, True),  # softmax over all E
    (7, 1024, 256, 64, 6, "sigmoid", False, torch.bfloat16, torch.bfloat16, False, True),
    (9, 1024, 256, 64, 8, "softmax", True, torch.float32, torch.bfloat16, True, True),  # tied logits
    (40, 1024, 256, 64, 6, "softmax", True, torch.float32, torch.bfloat16, False, False),  # > 16 tokens
    (4, 1024, 256, 300, 4, "softmax", True, torch.float32, torch.bfloat16, False, False),  # E > 256
]


@pytest.mark.parametrize("T,H,I,E,k,scoring,renorm,ldt,dt,ties,one", CASES)
def test_from_logits_matches_router_then_layer(T, H, I, E, k, scoring, renorm, ldt, dt, ties, one):
    rng = np.random.default_rng(T * 1000 + E)
    x = torch.from_numpy(rng.standard_normal((T, H), dtype=np.float32)).to(dev(), dt)
    w13 = (torch.from_numpy(rng.standard_normal((E, 2 * I, H), dtype=np.float32) * 0.02).to(dev(), dt)
           .transpose(1, 2))
    w2 = torch.from_numpy(rng.standard_normal((E, H, I), dtype=np.float32) * 0.02).to(dev(), dt).transpose(1, 2)
    lg = rng.standard_normal((T, E), dtype=np.float32)
    if ties:
        lg = np.round(lg * 2) / 2  # few distinct values: the lower expert id must win every tie
    logits = torch.from_numpy(lg).to(dev(), ldt)

    lib = _lib.load()
    before = lib.moe_launch_count()
    y, wts, ids = mb.fused_moe_mlp_from_logits(x, w13, w2, logits, k, scoring=scoring, renormalize=renorm)
    launches = lib.moe_launch_count() - before
    assert launches == 1 if one else launches > 1

    ref_ids, ref_wts = mb.route_topk(logits, k, scoring=scoring, renormalize=renorm)
    assert torch.equal(ids, ref_ids)
    assert torch.equal(wts, ref_wts)

    y2 = mb.fused_moe_mlp(x, w13, w2, ref_wts, ref_ids)
    assert max_abs_rel(y.float().cpu().numpy(), y2.float().cpu().numpy()) < TOL
    rnd = O.round_bf16 if dt == torch.bfloat16 else O.round_fp16
    ref = O.moe_mlp_topk(x.float().cpu().numpy(), w13.float().cpu().numpy(), w2.float().cpu().numpy(),
                         ref_wts.cpu().numpy(), ref_ids.cpu().numpy(), round_hidden=rnd)
    assert max_abs_rel(y.float().cpu().numpy(), ref) < TOL
    assert mb.device_error(dev()) == 0


def test_from_logits_back_to_back_and_graph_capture():
    """Consecutive one-launch calls with different logits (each launch routes
    afresh) and a CUDA-graph replay of the call, on the Qwen3 decode shape."""
    T, H, I, E, k = 4, 2048, 768, 128, 8
    w13 = (torch.randn(E, 2 * I, H, device=dev()) * 0.02).to(torch.bfloat16).transpose(1, 2)
    w2 = (torch.randn(E, H, I, device=dev()) * 0.02).to(torch.bfloat16).transpose(1, 2)
    x = torch.randn(T, H, device=dev()).to(torch.bfloat16)
    logits = torch.randn(T, E, device=dev())
    for _ in range(3):
        logits.normal_()
        y, wts, ids = mb.fused_moe_mlp_from_logits(x, w13, w2, logits, k)
        ref_ids, ref_wts = mb.route_topk(logits, k)
        assert torch.equal(ids, ref_ids) and torch.equal(wts, ref_wts)
        ref = mb.fused_moe_mlp(x, w13, w2, ref_wts, ref_ids)
        assert max_abs_rel(y.float().cpu().numpy(), ref.float().cpu().numpy()) < TOL
    mb.fused_moe_mlp_from_logits(x, w13, w2, logits, k)  # warm-up on the capture stream's allocator
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        mb.fused_moe_mlp_from_logits(x, w13, w2, logits, k)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        yg, wg, ig = mb.fused_moe_mlp_from_logits(x, w13, w2, logits, k)
    for _ in range(2):
        logits.normal_()
        g.replay()
        torch.cuda.synchronize()
        ref_ids, ref_wts = mb.route_topk(logits, k)
        assert torch.equal(ig, ref_ids) and torch.equal(wg, ref_wts)
        ref = mb.fused_moe_mlp(x, w13, w2, ref_wts, ref_ids)
        assert max_abs_rel(yg.float().cpu().numpy(), ref.float().cpu().numpy()) < TOL
    del g
    assert mb.device_error(dev()) == 0
