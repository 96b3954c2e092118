"""GPU parity of the swapped-operand grouped GEMMs (few token rows per
expert: the weights are the MMA's 128-row operand, the expert's tokens its N
operand; MOE_OPT_GEMM_SWAP_AB), including the K-split launches decode takes
when an op has fewer work items than SMs. Same bars as the other parity
tests: max-abs-rel error 1e-2 against the fp32 oracle."""
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


@pytest.fixture(autouse=True)
def multi_launch_path():
    """These tests cover the multi-launch path's swapped GEMMs: the one-launch
    decode kernel (tested in test_gpu_decode.py) is switched off."""
    lib = _lib.load()
    old = lib.moe_get_option(_lib.OPT_DECODE_FUSED)
    lib.moe_set_option(_lib.OPT_DECODE_FUSED, 0)
    yield
    lib.moe_set_option(_lib.OPT_DECODE_FUSED, old)


@pytest.fixture(params=[2, 1], ids=["swap_auto", "swap_forced"])
def swap(request):
    lib = _lib.load()
    old = lib.moe_get_option(_lib.OPT_GEMM_SWAP_AB)
    assert lib.moe_set_option(_lib.OPT_GEMM_SWAP_AB, request.param) == 0
    yield request.param
    lib.moe_set_option(_lib.OPT_GEMM_SWAP_AB, old)


CASES = [
    # T, H, I, E, k, routing, dtype, quant
    (1, 2048, 768, 128, 8, "zipf1.2", torch.bfloat16, False),     # decode: 8 slots, K split 3 ways
    (4, 2048, 768, 128, 8, "zipf1.2", torch.bfloat16, False),     # 32 slots: 32-row token items
    (32, 2048, 768, 128, 8, "zipf1.2", torch.bfloat16, False),
    (256, 2048, 768, 128, 8, "zipf1.2", torch.bfloat16, False),   # up to 128 token rows per item
    (1, 2048, 768, 128, 8, "zipf1.2", torch.bfloat16, True),      # w8a8 decode (int32 split partials)
    (64, 2048, 768, 128, 8, "zipf1.2", torch.bfloat16, True),
    (64, 1024, 512, 8, 2, "uniform-softmax", torch.float32, False),  # tiny fp32 layer (tf32)
    (5, 512, 136, 16, 4, "sigmoid", torch.float16, False),        # ragged I: a partial feature tile
    (300, 256, 384, 64, 6, "hot25-zipf1.0", torch.bfloat16, False),  # a hot expert with several token tiles
    (512, 1024, 256, 128, 8, "zipf1.2", torch.bfloat16, False),   # 4096 slots: the largest one-launch prep
    (513, 1024, 256, 128, 8, "zipf1.2", torch.bfloat16, False),   # 4104 slots: align + gather launches
]


@pytest.mark.parametrize("T,H,I,E,k,routing,dtype,quant", CASES)
def test_swapped_gemms_match_oracle(T, H, I, E, k, routing, dtype, quant, swap):
    rng = np.random.default_rng(T + H + I)
    x = torch.from_numpy(rng.standard_normal((T, H), dtype=np.float32)).to(dev(), dtype)
    w13 = torch.from_numpy(rng.standard_normal((E, 2 * I, H), dtype=np.float32) * 0.02).to(dev(), dtype)
    w2 = torch.from_numpy(rng.standard_normal((E, H, I), dtype=np.float32) * 0.02).to(dev(), dtype)
    w13, w2 = w13.transpose(1, 2), w2.transpose(1, 2)
    ids, wts = O.synthetic_routing(routing, T, E, k, 5)
    scales = None
    if quant:
        w13, w2, scales = mb.quantize_weights_int8(w13, w2)
    y = mb.fused_moe_mlp(x, w13, w2, torch.from_numpy(wts).to(dev()), torch.from_numpy(ids).to(dev()),
                         scales=scales)
    xf = x.float().cpu().numpy()
    rnd = None if dtype == torch.float32 else (O.round_bf16 if dtype == torch.bfloat16 else O.round_fp16)
    if quant:
        ref = O.moe_mlp_w8a8(xf, w13.transpose(1, 2).cpu().numpy(), scales[0].cpu().numpy(),
                             w2.transpose(1, 2).cpu().numpy(), scales[1].cpu().numpy(), wts, ids,
                             round_hidden=O.round_bf16)
    else:
        ref = O.moe_mlp_topk(xf, w13.float().cpu().numpy(), w2.float().cpu().numpy(), wts, ids, round_hidden=rnd)
    err = max_abs_rel(y.float().cpu().numpy(), ref)
    assert err < TOL, err
    assert mb.device_error(dev()) == 0


def test_swapped_split_matches_unsplit_gate_up():
    """The decode launch with its K split (auto) and the same op with the
    swap forced on the stand-alone-style plan differ only in how K is summed:
    outputs agree to fp32 rounding of the partial sums."""
    T, H, I, E, k = 1, 2048, 768, 128, 8
    rng = np.random.default_rng(3)
    x = torch.from_numpy(rng.standard_normal((T, H), dtype=np.float32)).to(dev(), torch.bfloat16)
    w13 = (torch.randn(E, 2 * I, H, device=dev()) * 0.02).to(torch.bfloat16).transpose(1, 2)
    w2 = (torch.randn(E, H, I, device=dev()) * 0.02).to(torch.bfloat16).transpose(1, 2)
    ids, wts = O.synthetic_routing("zipf1.2", T, E, k, 9)
    args = (x, w13, w2, torch.from_numpy(wts).to(dev()), torch.from_numpy(ids).to(dev()))
    lib = _lib.load()
    old = lib.moe_get_option(_lib.OPT_GEMM_SWAP_AB)
    try:
        lib.moe_set_option(_lib.OPT_GEMM_SWAP_AB, 2)
        y_split = mb.fused_moe_mlp(*args).float()
        y_split2 = mb.fused_moe_mlp(*args).float()
        lib.moe_set_option(_lib.OPT_GEMM_SWAP_AB, 0)
        y_rows = mb.fused_moe_mlp(*args).float()
    finally:
        lib.moe_set_option(_lib.OPT_GEMM_SWAP_AB, old)
    assert max_abs_rel(y_split.cpu().numpy(), y_rows.cpu().numpy()) < 2e-2
    # one token: every output element is a sum over k slots only, added by
    # atomics in any order; the gate_up partial sums are added in a fixed order
    assert max_abs_rel(y_split.cpu().numpy(), y_split2.cpu().numpy()) < 1e-2
    assert mb.device_error(dev()) == 0


def test_swapped_graph_replay_matches_eager():
    """The decode op (align, gather, K-split counters cleared, swapped GEMMs)
    captured in a CUDA graph replays to the eager result."""
    T, H, I, E, k = 8, 2048, 768, 128, 8
    w13 = (torch.randn(E, 2 * I, H, device=dev()) * 0.02).to(torch.bfloat16).transpose(1, 2)
    w2 = (torch.randn(E, H, I, device=dev()) * 0.02).to(torch.bfloat16).transpose(1, 2)
    cap = mb.CapturedMoeMLP(w13, w2, T, k, dtype=torch.bfloat16)
    for seed in range(3):
        x = torch.randn(T, H, device=dev()).to(torch.bfloat16)
        ids, wts = O.synthetic_routing("zipf1.2", T, E, k, seed)
        ids_t, wts_t = torch.from_numpy(ids).to(dev()), torch.from_numpy(wts).to(dev())
        ref = mb.fused_moe_mlp(x, w13, w2, wts_t, ids_t).float()
        got = cap(x, wts_t, ids_t).float()
        assert max_abs_rel(got.cpu().numpy(), ref.cpu().numpy()) < 1e-2
    assert mb.device_error(dev()) == 0


@pytest.mark.parametrize("quant", [False, True])
def test_fused_conversion_with_dropped_tokens(quant):
    """Decode-sized batch where some tokens have every slot dropped (ids
    outside [0, E)) and others some: the down GEMM converts each output group
    once all of its token's routed slots have been added, and the tokens with
    none get zero rows."""
    T, H, I, E, k = 24, 1024, 512, 64, 6
    rng = np.random.default_rng(17)
    x = torch.from_numpy(rng.standard_normal((T, H), dtype=np.float32)).to(dev(), torch.bfloat16)
    w13 = (torch.randn(E, 2 * I, H, device=dev()) * 0.03).to(torch.bfloat16).transpose(1, 2)
    w2 = (torch.randn(E, H, I, device=dev()) * 0.03).to(torch.bfloat16).transpose(1, 2)
    ids, wts = O.synthetic_routing("zipf1.2", T, E, k, 4)
    ids = ids.copy()
    ids[[0, 7, 23]] = -1            # tokens with every slot dropped
    ids[3, :4] = E + 5              # a token with two slots left
    scales = None
    if quant:
        w13, w2, scales = mb.quantize_weights_int8(w13, w2)
    y = mb.fused_moe_mlp(x, w13, w2, torch.from_numpy(wts).to(dev()), torch.from_numpy(ids).to(dev()),
                         scales=scales)
    yf = y.float().cpu().numpy()
    assert (yf[[0, 7, 23]] == 0).all()
    xf = x.float().cpu().numpy()
    if quant:
        ref = O.moe_mlp_w8a8(xf, w13.transpose(1, 2).cpu().numpy(), scales[0].cpu().numpy(),
                             w2.transpose(1, 2).cpu().numpy(), scales[1].cpu().numpy(), wts, ids,
                             round_hidden=O.round_bf16)
    else:
        ref = O.moe_mlp_topk(xf, w13.float().cpu().numpy(), w2.float().cpu().numpy(), wts, ids,
                             round_hidden=O.round_bf16)
    assert max_abs_rel(yf, ref) < TOL
    assert mb.device_error(dev()) == 0


def test_graph_bound_to_resident_inputs():
    """CapturedMoeMLP with inputs=(x, w, ids): replays read those tensors
    directly; rewriting them in place changes the next result."""
    T, H, I, E, k = 8, 2048, 768, 128, 8
    w13 = (torch.randn(E, 2 * I, H, device=dev()) * 0.02).to(torch.bfloat16).transpose(1, 2)
    w2 = (torch.randn(E, H, I, device=dev()) * 0.02).to(torch.bfloat16).transpose(1, 2)
    x = torch.randn(T, H, device=dev()).to(torch.bfloat16)
    ids0, wts0 = O.synthetic_routing("zipf1.2", T, E, k, 1)
    ids = torch.from_numpy(ids0).to(dev())
    wts = torch.from_numpy(wts0).to(dev())
    cap = mb.CapturedMoeMLP(w13, w2, T, k, dtype=torch.bfloat16, inputs=(x, wts, ids))
    for seed in range(3):
        ids_n, wts_n = O.synthetic_routing("zipf1.2", T, E, k, 10 + seed)
        x.copy_(torch.randn(T, H, device=dev()))
        ids.copy_(torch.from_numpy(ids_n))
        wts.copy_(torch.from_numpy(wts_n))
        got = cap(x, wts, ids).float()
        ref = mb.fused_moe_mlp(x, w13, w2, wts, ids).float()
        assert max_abs_rel(got.cpu().numpy(), ref.cpu().numpy()) < 1e-2
    assert mb.device_error(dev()) == 0
