"""GPU parity on the workload's own bars and shapes:

* int8 GEMM accumulations exact in int32: the down GEMM's raw accumulators
  (int8 x int8, unit scales, fp32 row store) equal numpy integer dot products
  bit for bit, and the gate_up GEMM's SwiGLU output on exactly dequantised
  accumulators (power-of-two scales) matches a float64 reference to 1e-6 of
  its largest element — on all three GEMM variants, with odd last tiles,
  ragged N and a reduction length that is not a multiple of 128;
* the DeepSeek-V3 layer shape (H=7168, I=2048, E=256, top-8 sigmoid, w8a8)
  and the load-imbalance stress shape (H=4096, I=1536, E=64, top-6, a quarter
  of the tokens on one hot expert, T=65536) against the oracle on sampled
  tokens (each token's output depends on its own row only, so a sample is an
  exact check of those rows).
"""
import numpy as np
import pytest
import torch

import mail_b200 as mb
from mail_b200 import _lib
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

TOL = 1e-2  # max-abs-rel bound for bf16 outputs against the fp32 oracle


def dev():
    return torch.device("cuda", 0)


def stream():
    return torch.cuda.current_stream(dev()).cuda_stream


def max_abs_rel(y, ref):
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


@pytest.fixture(params=[(1, 1, 0), (1, 0, 0), (0, 1, 0), (2, 1, 1)],
                ids=["cta_pair", "cta_pair_no_half_units", "single_cta", "swapped_operands"])
def gemm_variant(request):
    """CTA pairs (with and without M=128 half units), one CTA per tile, and
    the swapped-operand kernel (forced on the stand-alone GEMM calls)."""
    lib = _lib.load()
    opts = (_lib.OPT_GEMM_CTA_PAIR, _lib.OPT_GEMM_HALF_UNITS, _lib.OPT_GEMM_SWAP_AB)
    old = [lib.moe_get_option(o) for o in opts]
    for o, v in zip(opts, request.param):
        assert lib.moe_set_option(o, v) == 0
    yield request.param
    for o, v in zip(opts, old):
        lib.moe_set_option(o, v)


def tile_table(group_sizes):
    """The compact tile table of pre-grouped rows (moe_tile_schedule)."""
    gs = torch.tensor(group_sizes, dtype=torch.int64, device=dev())
    E, T = len(group_sizes), int(sum(group_sizes))
    grid = int(_lib.query("moe_tile_grid", T, E, 128))
    table = torch.zeros(int(_lib.query("moe_tile_table_ints", E, grid)), dtype=torch.int32, device=dev())
    _lib.call("moe_tile_schedule", gs.data_ptr(), _lib.I64, E, T, 128, None, None, None, table.data_ptr(), stream())
    return table, grid


def expert_of_rows(group_sizes):
    return np.repeat(np.arange(len(group_sizes)), group_sizes)


# odd last tiles (3.04 and 1 tiles), an empty expert, a single row, whole tiles
GROUPS = [389, 0, 1, 257, 128, 64, 200]


@pytest.mark.parametrize("K,N", [(1040, 520), (272, 256)])
def test_down_gemm_int8_accumulators_exact(K, N, gemm_variant):
    rng = np.random.default_rng(K + N)
    E, T = len(GROUPS), sum(GROUPS)
    h = rng.integers(-127, 128, size=(T, K), dtype=np.int8)
    w2 = rng.integers(-127, 128, size=(E, N, K), dtype=np.int8)   # K-major [E, H, I]
    table, grid = tile_table(GROUPS)
    h_d, w2_d = torch.from_numpy(h).to(dev()), torch.from_numpy(w2).to(dev())
    ones_h = torch.ones(T, device=dev())
    ones_w = torch.ones(E, N, device=dev())
    out = torch.full((T, N), float("nan"), device=dev())
    _lib.call("moe_gemm2", h_d.data_ptr(), _lib.I8, T, K, w2_d.data_ptr(), E, N, ones_h.data_ptr(), ones_w.data_ptr(),
              table.data_ptr(), grid, _lib.EPI_STORE_ROWS, None, None, 1, out.data_ptr(), _lib.F32, T, stream())
    got = out.cpu().numpy()
    ex = expert_of_rows(GROUPS)
    ref = np.empty((T, N), np.int64)
    for e in range(E):
        rows = np.nonzero(ex == e)[0]
        if rows.size:
            ref[rows] = h[rows].astype(np.int64) @ w2[e].astype(np.int64).T
    assert np.abs(ref).max() < 2 ** 24  # fp32 holds every accumulator exactly
    np.testing.assert_array_equal(got, ref.astype(np.float32))
    assert mb.device_error(dev()) == 0


@pytest.mark.parametrize("K,I", [(1040, 136), (272, 256)])
def test_gate_up_gemm_int8_swiglu_on_exact_accumulators(K, I, gemm_variant):
    rng = np.random.default_rng(K * 3 + I)
    E, T = len(GROUPS), sum(GROUPS)
    a = rng.integers(-127, 128, size=(T, K), dtype=np.int8)
    w13 = rng.integers(-127, 128, size=(E, 2 * I, K), dtype=np.int8)
    # power-of-two scales: the dequantised accumulators are exact in fp32
    a_scale = np.ldexp(np.ones(T, np.float32), -rng.integers(11, 14, size=T)).astype(np.float32)
    w_scale = np.ldexp(np.ones((E, 2 * I), np.float32), -rng.integers(0, 3, size=(E, 2 * I))).astype(np.float32)
    table, grid = tile_table(GROUPS)
    a_d, w_d = torch.from_numpy(a).to(dev()), torch.from_numpy(w13).to(dev())
    as_d, ws_d = torch.from_numpy(a_scale).to(dev()), torch.from_numpy(w_scale).to(dev())
    h = torch.full((T, I), float("nan"), device=dev())
    _lib.call("moe_gemm1_swiglu", a_d.data_ptr(), _lib.I8, T, K, w_d.data_ptr(), E, I, as_d.data_ptr(),
              ws_d.data_ptr(), table.data_ptr(), grid, h.data_ptr(), _lib.F32, stream())
    got = h.cpu().numpy().astype(np.float64)
    ex = expert_of_rows(GROUPS)
    ref = np.empty((T, I), np.float64)
    for e in range(E):
        rows = np.nonzero(ex == e)[0]
        if rows.size == 0:
            continue
        acc = a[rows].astype(np.int64) @ w13[e].astype(np.int64).T            # exact integers
        assert np.abs(acc).max() < 2 ** 24
        gu = acc.astype(np.float64) * a_scale[rows, None] * w_scale[e][None, :]
        g, u = gu[:, :I], gu[:, I:]
        ref[rows] = g / (1.0 + np.exp(-g)) * u
    scale = np.abs(ref).max()
    assert np.abs(got - ref).max() <= 1e-6 * scale
    assert (np.abs(got - ref) <= 2e-5 * np.abs(ref) + 1e-7 * scale).all()
    assert mb.device_error(dev()) == 0


class ExpertsOnDevice:
    """Int8 expert weights left on the GPU and copied to the host one expert
    at a time, only for the experts the oracle touches ([E, N, K] K-major)."""

    def __init__(self, w_logical):
        self.w = w_logical.transpose(1, 2)  # [E, N, K] view of the K-major storage
        self.shape = tuple(self.w.shape)

    def __getitem__(self, e):
        return self.w[e].cpu().numpy()


def big_w8a8_layer(E, H, I, seed):
    g = torch.Generator(device=dev()).manual_seed(seed)
    w13 = torch.empty(E, 2 * I, H, device=dev(), dtype=torch.bfloat16)
    w2 = torch.empty(E, H, I, device=dev(), dtype=torch.bfloat16)
    for e0 in range(0, E, 16):  # N(0, 0.02) weights, generated a few experts at a time
        n = min(16, E - e0)
        w13[e0:e0 + n] = (torch.randn(n, 2 * I, H, device=dev(), generator=g) * 0.02).to(torch.bfloat16)
        w2[e0:e0 + n] = (torch.randn(n, H, I, device=dev(), generator=g) * 0.02).to(torch.bfloat16)
    q13, q2, scales = mb.quantize_weights_int8(w13.transpose(1, 2), w2.transpose(1, 2))
    del w13, w2
    torch.cuda.empty_cache()
    return q13, q2, scales


def check_sampled_w8a8(x, q13, q2, scales, ids, wts, y, sample):
    ref = O.moe_mlp_w8a8(x[sample].float().cpu().numpy(), ExpertsOnDevice(q13), scales[0].cpu().numpy(),
                         ExpertsOnDevice(q2), scales[1].cpu().numpy(), wts[sample], ids[sample],
                         round_hidden=O.round_bf16)
    err = max_abs_rel(y[torch.from_numpy(sample).to(dev())].float().cpu().numpy(), ref)
    assert err < TOL, err


@pytest.mark.parametrize("variant", ["auto", "pair"])
def test_deepseek_v3_shape_w8a8(variant):
    """H=7168, I=2048, E=256, top-8 sigmoid, w8a8: about 2 M tiles per expert
    (the one-CTA path under auto, forced CTA pairs otherwise)."""
    T, H, I, E, k = 1024, 7168, 2048, 256, 8
    lib = _lib.load()
    old = lib.moe_get_option(_lib.OPT_GEMM_CTA_PAIR)
    lib.moe_set_option(_lib.OPT_GEMM_CTA_PAIR, 2 if variant == "auto" else 1)
    try:
        q13, q2, scales = big_w8a8_layer(E, H, I, seed=40)
        g = torch.Generator(device=dev()).manual_seed(41)
        x = torch.randn(T, H, device=dev(), generator=g).to(torch.bfloat16)
        ids, wts = O.synthetic_routing("sigmoid", T, E, k, 42)
        y = mb.fused_moe_mlp(x, q13, q2, torch.from_numpy(wts).to(dev()), torch.from_numpy(ids).to(dev()),
                             scales=scales)
        torch.cuda.synchronize()
        assert torch.isfinite(y).all()
        sample = np.random.default_rng(43).choice(T, size=4, replace=False)
        check_sampled_w8a8(x, q13, q2, scales, ids, wts, y, sample)
    finally:
        lib.moe_set_option(_lib.OPT_GEMM_CTA_PAIR, old)
    assert mb.device_error(dev()) == 0


def test_stress_shape_hot_expert_w8a8():
    """T=65536, H=4096, I=1536, E=64, top-6, a quarter of the tokens forced
    onto one hot expert (>= 128 M tiles of it), w8a8, the row-store combine
    (the fp32 accumulator would be 1 GiB); deterministic across calls."""
    T, H, I, E, k = 65536, 4096, 1536, 64, 6
    q13, q2, scales = big_w8a8_layer(E, H, I, seed=50)
    g = torch.Generator(device=dev()).manual_seed(51)
    x = torch.randn(T, H, device=dev(), generator=g).to(torch.bfloat16)
    ids, wts = O.synthetic_routing("hot25-zipf1.0", T, E, k, 52)
    counts = np.bincount(ids.reshape(-1), minlength=E)
    hot = int(counts.argmax())
    assert counts[hot] >= T // 4 and -(-counts[hot] // 128) >= 128
    ids_d, wts_d = torch.from_numpy(ids).to(dev()), torch.from_numpy(wts).to(dev())
    y = mb.fused_moe_mlp(x, q13, q2, wts_d, ids_d, scales=scales)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()
    rng = np.random.default_rng(53)
    on_hot = np.nonzero((ids == hot).any(axis=1))[0]
    sample = np.concatenate([rng.choice(on_hot, 6, replace=False), rng.choice(T, 6, replace=False)])
    check_sampled_w8a8(x, q13, q2, scales, ids, wts, y, sample)
    y2 = mb.fused_moe_mlp(x, q13, q2, wts_d, ids_d, scales=scales)
    assert torch.equal(y, y2)
    assert mb.device_error(dev()) == 0
