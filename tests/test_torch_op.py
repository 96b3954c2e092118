"""The two forms of fused_moe_mlp registered as PyTorch operators
(torch.ops.mail_b200.fused_moe_mlp / fused_experts): schemas, fake (meta)
kernels that trace without running the library, one node per call in a
traced graph, and (GPU) torch.compile(fullgraph=True) with no graph break."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode
from torch.fx.experimental.proxy_tensor import make_fx

import mail_b200 as mb  # noqa: F401  (registers the operators)


def fake_inputs(T=64, H=128, I=64, E=4, k=2, dtype=torch.bfloat16, quant=False):
    wd = torch.int8 if quant else dtype
    x = torch.empty(T, H, device="cuda", dtype=dtype)
    w13 = torch.empty(E, 2 * I, H, device="cuda", dtype=wd).transpose(1, 2)
    w2 = torch.empty(E, H, I, device="cuda", dtype=wd).transpose(1, 2)
    ids = torch.empty(T, k, device="cuda", dtype=torch.int32)
    w = torch.empty(T, k, device="cuda", dtype=torch.float32)
    s13 = torch.empty(E, 2 * I, device="cuda") if quant else None
    s2 = torch.empty(E, H, device="cuda") if quant else None
    return x, w13, w2, w, ids, s13, s2


def test_schemas():
    assert str(torch.ops.mail_b200.fused_moe_mlp.default._schema) == (
        "mail_b200::fused_moe_mlp(Tensor x, Tensor w13, Tensor w2, Tensor group_sizes) -> Tensor")
    assert str(torch.ops.mail_b200.fused_experts.default._schema) == (
        "mail_b200::fused_experts(Tensor x, Tensor w13, Tensor w2, Tensor topk_weights, Tensor topk_ids, "
        "Tensor? w13_scale, Tensor? w2_scale) -> Tensor")


def test_from_logits_schema_and_fake_kernel():
    """The logits-in call: routing outputs beside y, shapes from the fake
    kernel; a bad top_k or scoring fails while tracing."""
    assert str(torch.ops.mail_b200.fused_experts_from_logits.default._schema) == (
        "mail_b200::fused_experts_from_logits(Tensor x, Tensor w13, Tensor w2, Tensor router_logits, SymInt top_k, "
        "str scoring, bool renormalize, Tensor? w13_scale, Tensor? w2_scale) -> (Tensor, Tensor, Tensor)")
    with FakeTensorMode():
        x, w13, w2, _, _, _, _ = fake_inputs(T=5, E=16)
        lg = torch.empty(5, 16, device="cuda")
        y, w, ids = torch.ops.mail_b200.fused_experts_from_logits(x, w13, w2, lg, 8, "sigmoid", True, None, None)
        assert y.shape == (5, 128) and y.dtype == torch.bfloat16
        assert w.shape == (5, 8) and w.dtype == torch.float32
        assert ids.shape == (5, 8) and ids.dtype == torch.int32
        with pytest.raises(ValueError):
            torch.ops.mail_b200.fused_experts_from_logits(x, w13, w2, lg, 17, "softmax", True, None, None)
        with pytest.raises(ValueError):
            torch.ops.mail_b200.fused_experts_from_logits(x, w13, w2, lg, 2, "relu", True, None, None)
        with pytest.raises(ValueError):
            torch.ops.mail_b200.fused_experts_from_logits(x, w13, w2, lg[:, :8], 2, "softmax", True, None, None)


@pytest.mark.parametrize("quant", [False, True])
def test_fake_kernels_give_output_shape_and_dtype(quant):
    with FakeTensorMode():
        x, w13, w2, w, ids, s13, s2 = fake_inputs(quant=quant)
        y = torch.ops.mail_b200.fused_experts(x, w13, w2, w, ids, s13, s2)
        assert y.shape == (64, 128) and y.dtype == torch.bfloat16 and y.device.type == "cuda"
        gs = torch.empty(4, device="cuda", dtype=torch.int64)
        y2 = torch.ops.mail_b200.fused_moe_mlp(x, w13, w2, gs)
        assert y2.shape == x.shape and y2.dtype == x.dtype


def test_fake_kernels_reject_bad_shapes():
    with FakeTensorMode():
        x, w13, w2, w, ids, _, _ = fake_inputs()
        with pytest.raises(ValueError):
            torch.ops.mail_b200.fused_experts(x, w13, w2, w[:, :1], ids, None, None)
        with pytest.raises(ValueError):
            torch.ops.mail_b200.fused_moe_mlp(x, w13, w2[:, :, :64], torch.empty(4, device="cuda"))


def test_traced_graph_holds_one_op_node():
    def layer(x, w13, w2, w, ids):
        return torch.ops.mail_b200.fused_experts(x, w13, w2, w, ids, None, None) * 2.0

    with FakeTensorMode() as mode:
        args = fake_inputs()[:5]
    gm = make_fx(layer, tracing_mode="fake")(*args)
    targets = [n.target for n in gm.graph.nodes if n.op == "call_function"]
    assert targets.count(torch.ops.mail_b200.fused_experts.default) == 1
    del mode


@pytest.mark.gpu
@pytest.mark.parametrize("quant", [False, True])
def test_torch_compile_fullgraph_matches_eager(quant):
    torch.manual_seed(0)
    T, H, I, E, k = 96, 256, 128, 8, 2
    x = torch.randn(T, H, device="cuda").to(torch.bfloat16)
    w13 = (torch.randn(E, 2 * I, H, device="cuda") * 0.02).to(torch.bfloat16).transpose(1, 2)
    w2 = (torch.randn(E, H, I, device="cuda") * 0.02).to(torch.bfloat16).transpose(1, 2)
    scales = None
    if quant:
        w13, w2, scales = mb.quantize_weights_int8(w13, w2)
    ids = torch.stack([torch.randperm(E, device="cuda")[:k] for _ in range(T)]).to(torch.int32)
    wts = torch.softmax(torch.randn(T, k, device="cuda"), dim=1)

    def layer(x, wts, ids):
        return mb.fused_moe_mlp(x, w13, w2, wts, ids, scales=scales) + x

    ref = layer(x, wts, ids).float()
    torch._dynamo.reset()
    got = torch.compile(layer, fullgraph=True)(x, wts, ids).float()
    assert float((got - ref).abs().max() / ref.abs().max()) < 1e-2
    args = (x, w13, w2, wts, ids, *(scales if scales else (None, None)))
    torch.library.opcheck(torch.ops.mail_b200.fused_experts.default, args,
                          test_utils=("test_schema", "test_faketensor"))
    assert mb.device_error() == 0


@pytest.mark.gpu
def test_torch_compile_prerouted_form():
    torch.manual_seed(1)
    E, H, I = 4, 128, 64
    gs = torch.tensor([37, 0, 50, 21], device="cuda")
    x = torch.randn(int(gs.sum()), H, device="cuda").to(torch.bfloat16)
    w13 = (torch.randn(E, 2 * I, H, device="cuda") * 0.05).to(torch.bfloat16).transpose(1, 2)
    w2 = (torch.randn(E, H, I, device="cuda") * 0.05).to(torch.bfloat16).transpose(1, 2)
    ref = mb.fused_moe_mlp(x, w13, w2, gs)
    torch._dynamo.reset()
    got = torch.compile(lambda a: mb.fused_moe_mlp(a, w13, w2, gs), fullgraph=True)(x)
    assert torch.equal(got, ref)  # the pre-routed form has no atomics: bit-identical


@pytest.mark.gpu
def test_torch_compile_from_logits():
    """The logits-in call under torch.compile(fullgraph=True): one operator,
    the same routing and output as the eager call (decode-sized: the routing
    runs inside the one-launch kernel)."""
    torch.manual_seed(2)
    T, H, I, E, k = 4, 256, 128, 16, 4
    x = torch.randn(T, H, device="cuda").to(torch.bfloat16)
    w13 = (torch.randn(E, 2 * I, H, device="cuda") * 0.02).to(torch.bfloat16).transpose(1, 2)
    w2 = (torch.randn(E, H, I, device="cuda") * 0.02).to(torch.bfloat16).transpose(1, 2)
    lg = torch.randn(T, E, device="cuda")

    def layer(x, lg):
        y, _, ids = mb.fused_moe_mlp_from_logits(x, w13, w2, lg, k)
        return y + x, ids

    ref_y, ref_ids = layer(x, lg)
    torch._dynamo.reset()
    got_y, got_ids = torch.compile(layer, fullgraph=True)(x, lg)
    assert torch.equal(got_ids, ref_ids)
    ref = ref_y.float()
    assert float((got_y.float() - ref).abs().max() / ref.abs().max()) < 1e-2
    assert mb.device_error() == 0
