"""GPU parity: the sm_100a kernels (through the C ABI) against the oracle and
the reference's golden vectors.

Bars: integer/index work (tile schedule, align, int8 quant) bit-exact;
floating-point outputs within max-abs-rel error 1e-2 of an fp32 reference
(max |y - ref| / max |ref|), the tolerance the workload sets for bf16 outputs.
"""
import os

import numpy as np
import pytest
import torch

import mail_b200 as mb
from mail_b200 import _lib
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
TOL = 1e-2  # max-abs-rel error bound for bf16/fp16/tf32 outputs


def max_abs_rel(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


def npf(t):
    return t.detach().float().cpu().numpy()


def dev():
    return torch.device("cuda", 0)


def assert_no_device_error():
    assert mb.device_error(dev()) == 0


@pytest.fixture(params=[(1, 1), (1, 0), (0, 1)], ids=["cta_pair", "cta_pair_no_half_units", "single_cta"])
def gemm_variant(request):
    """Runs a test with the CTA-pair (cta_group::2) GEMMs — each expert's odd
    last tile as an M=128 pair MMA (half unit), and as an M=256 one with half
    of it idle — and with one CTA per tile."""
    lib = _lib.load()
    pair, half = request.param
    old = lib.moe_get_option(_lib.OPT_GEMM_CTA_PAIR), lib.moe_get_option(_lib.OPT_GEMM_HALF_UNITS)
    assert lib.moe_set_option(_lib.OPT_GEMM_CTA_PAIR, pair) == 0
    assert lib.moe_set_option(_lib.OPT_GEMM_HALF_UNITS, half) == 0
    yield pair
    lib.moe_set_option(_lib.OPT_GEMM_CTA_PAIR, old[0])
    lib.moe_set_option(_lib.OPT_GEMM_HALF_UNITS, old[1])


# --------------------------------------------------------------------------- tile schedule


def schedule_cases():
    t = np.load(os.path.join(GOLDEN, "tile_schedule.npz"))
    names = sorted({k.split("/")[0] for k in t.files})
    return [(n, bm) for n in names for bm in (16, 32, 64, 128, 256)]


@pytest.mark.parametrize("name,bm", schedule_cases())
def test_tile_schedule_matches_reference_bit_exact(name, bm):
    t = np.load(os.path.join(GOLDEN, "tile_schedule.npz"))
    gs = t[f"{name}/group_sizes"]
    for dt in (torch.int64, torch.int32):
        g = torch.tensor(gs, dtype=dt, device=dev())
        te, ts, tc, grid = mb.build_tile_schedule(g, int(gs.sum()), bm)
        assert grid == int(t[f"{name}/bm{bm}/grid"])
        np.testing.assert_array_equal(te.cpu().numpy(), t[f"{name}/bm{bm}/expert"])
        np.testing.assert_array_equal(ts.cpu().numpy(), t[f"{name}/bm{bm}/row_start"])
        np.testing.assert_array_equal(tc.cpu().numpy(), t[f"{name}/bm{bm}/row_count"])
        exact = int(t[f"{name}/bm{bm}/exact_grid"])
        np.testing.assert_array_equal(ts.cpu().numpy()[:exact], t[f"{name}/bm{bm}/exact_row_start"])


# --------------------------------------------------------------------------- align


ALIGN_CASES = [
    ("uniform", 64, 2, 8), ("uniform", 4096, 2, 8), ("uniform", 1, 8, 128), ("zipf", 257, 8, 128),
    ("uniform", 8192, 8, 256), ("hot", 5000, 6, 64), ("invalid", 300, 4, 16), ("one_expert", 1000, 1, 32),
    ("uniform", 3, 8, 1024),
]


def make_ids(kind, T, k, E, seed=0):
    rng = np.random.default_rng(seed)
    if kind == "uniform":
        return np.argsort(rng.random((T, E)), axis=1)[:, :k].astype(np.int32)
    if kind == "zipf":
        return O.synthetic_routing("zipf1.2", T, E, k, seed)[0]
    if kind == "hot":
        return O.synthetic_routing("hot25-zipf1.0", T, E, k, seed)[0]
    if kind == "invalid":
        return rng.integers(-2, E + 3, size=(T, k)).astype(np.int32)
    if kind == "one_expert":
        return np.full((T, k), E - 1, np.int32)
    raise ValueError(kind)


@pytest.mark.parametrize("kind,T,k,E", ALIGN_CASES)
def test_align_bit_exact(kind, T, k, E):
    ids = make_ids(kind, T, k, E)
    ref = O.align(ids, E, 128)
    got = mb.moe_align(torch.from_numpy(ids).to(dev()), E, 128)
    table = got["tile_table"].cpu().numpy()
    n = ref["num_tiles"]
    total = int(ref["padded_offsets"][-1])
    assert table[0] == n and table[1] == total and table[2] == ref["dropped"]
    np.testing.assert_array_equal(got["group_sizes"].cpu().numpy(), ref["group_sizes"])
    np.testing.assert_array_equal(got["padded_offsets"].cpu().numpy(), ref["padded_offsets"])
    np.testing.assert_array_equal(got["sorted_slots"].cpu().numpy()[:total], ref["sorted_slots"])
    np.testing.assert_array_equal(got["slot_pos"].cpu().numpy(), ref["slot_pos"])
    mt = got["max_tiles"]
    np.testing.assert_array_equal(table[4:4 + E + 1], ref["tile_cumsum"])
    np.testing.assert_array_equal(table[5 + E:5 + E + n], ref["tile_row_start"])
    np.testing.assert_array_equal(table[5 + E + mt:5 + E + mt + n], ref["tile_row_count"])


# --------------------------------------------------------------------------- router


@pytest.mark.parametrize("T,E,k,scoring,renorm,dtype", [
    (64, 8, 2, "softmax", True, torch.float32), (4096, 8, 2, "softmax", True, torch.bfloat16),
    (777, 128, 8, "softmax", False, torch.float32), (300, 256, 8, "sigmoid", True, torch.float32),
    (5, 64, 6, "sigmoid", False, torch.float16), (33, 1000, 4, "softmax", True, torch.float32),
    # more tokens than warps resident at once: four tokens per warp (E <= 256), odd T; one per warp above
    (20000, 64, 6, "softmax", True, torch.float32), (30001, 256, 8, "sigmoid", True, torch.bfloat16),
    (12000, 1000, 4, "softmax", False, torch.float32),
])
def test_route_topk_matches_oracle(T, E, k, scoring, renorm, dtype):
    rng = np.random.default_rng(E + k)
    lg = rng.standard_normal((T, E), dtype=np.float32)
    lg[0, :] = 0.25          # all tied: lowest ids win
    lg[1, 3] = lg[1, 5] = 9  # a tie at the top
    if T > 2 and E > 6:      # -0 and +0 compare equal: a tie, the lower id first
        lg[2, :] = -1.0
        lg[2, 6], lg[2, 2] = -0.0, 0.0
    lt = torch.from_numpy(lg).to(dev(), dtype)
    ids, w = mb.route_topk(lt, k, scoring, renorm)
    ids_ref, w_ref = O.route_topk(npf(lt), k, scoring, renorm)
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_ref)
    np.testing.assert_allclose(w.cpu().numpy(), w_ref, rtol=2e-6, atol=1e-7)


# --------------------------------------------------------------------------- quant / gather


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_quant_int8_rows_bit_exact(dtype):
    rng = np.random.default_rng(4)
    x = rng.standard_normal((300, 1024), dtype=np.float32) * rng.uniform(0.01, 10, size=(300, 1)).astype(np.float32)
    x[7] = 0.0
    x[11, :5] = [0.5, -0.5, 1.5, 2.5, 127.0]
    xt = torch.from_numpy(x).to(dev(), dtype)
    q, s = mb.quant_int8_rows(xt)
    q_ref, s_ref = O.quant_int8_rows(npf(xt))
    np.testing.assert_array_equal(s.cpu().numpy(), s_ref)
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)


def test_gather_rows_bit_exact():
    rng = np.random.default_rng(5)
    T, k, H, E = 100, 3, 256, 7
    x = torch.from_numpy(rng.standard_normal((T, H), dtype=np.float32)).to(dev(), torch.bfloat16)
    ids = make_ids("uniform", T, k, E)
    a = mb.moe_align(torch.from_numpy(ids).to(dev()), E, 128)
    rows = a["capacity"]
    xp = mb.gather_rows(x, a["sorted_slots"], k, rows, rows_dev=a["tile_table"][1:2])
    ref = O.align(ids, E, 128)
    total = int(ref["padded_offsets"][-1])
    xs = ref["sorted_slots"]
    expect = np.where(xs[:, None] >= 0, npf(x)[np.maximum(xs, 0) // k], 0.0)
    np.testing.assert_array_equal(npf(xp[:total]), expect)
    qp, sp = mb.gather_rows(x, a["sorted_slots"], k, rows, out_dtype=torch.int8, rows_dev=a["tile_table"][1:2])
    q_ref, s_ref = O.quant_int8_rows(expect)
    np.testing.assert_array_equal(qp[:total].cpu().numpy(), q_ref)
    np.testing.assert_array_equal(sp[:total].cpu().numpy(), s_ref)


# --------------------------------------------------------------------------- pre-routed form


@pytest.mark.parametrize("case", ["mlp_selfcheck_f32", "mlp_selftest_f16", "mlp_ragged_f32"])
@pytest.mark.parametrize("dtype", [None, torch.bfloat16])
def test_pre_routed_matches_reference_golden(case, dtype, gemm_variant):
    d = np.load(os.path.join(GOLDEN, case + ".npz"))
    dt = dtype or {np.float16: torch.float16, np.float32: torch.float32}[d["x"].dtype.type]
    x = torch.from_numpy(d["x"]).to(dev(), dt)
    # reference layout: logical (E, K, N) view over nn.Linear-style storage
    w13 = torch.from_numpy(d["w13"]).to(dev(), dt).transpose(1, 2).contiguous().transpose(1, 2)
    w2 = torch.from_numpy(d["w2"]).to(dev(), dt).transpose(1, 2).contiguous().transpose(1, 2)
    gs = torch.from_numpy(d["group_sizes"]).to(dev())
    out = mb.fused_moe_mlp(x, w13, w2, gs)
    assert out.dtype == dt and out.shape == x.shape
    if dtype is None:
        ref = d["ref_golden_loop"]  # the reference's own fp32 golden loop
    else:
        ref = O.moe_mlp_grouped(npf(x), npf(w13), npf(w2), d["group_sizes"])
    err = max_abs_rel(npf(out), ref)
    assert err < TOL, err
    assert_no_device_error()


def test_pre_routed_non_kmajor_weights_and_tail_rows(gemm_variant):
    rng = np.random.default_rng(9)
    E, H, I = 3, 256, 384
    gs = np.array([100, 0, 77])
    T = int(gs.sum()) + 20  # 20 rows no group covers -> zero (reference zero-inits its output)
    x = torch.from_numpy(rng.standard_normal((T, H), dtype=np.float32)).to(dev(), torch.bfloat16)
    w13 = (torch.randn(E, H, 2 * I, device=dev()) * 0.05).to(torch.bfloat16)  # N-contiguous: copied
    w2 = (torch.randn(E, I, H, device=dev()) * 0.05).to(torch.bfloat16)
    out = mb.fused_moe_mlp(x, w13, w2, torch.from_numpy(gs).to(dev()))
    ref = O.moe_mlp_grouped(npf(x), npf(w13), npf(w2), gs)
    assert max_abs_rel(npf(out), ref) < TOL
    assert (npf(out)[int(gs.sum()):] == 0).all()


def test_pre_routed_odd_and_even_tile_counts(gemm_variant):
    """Experts with odd and even numbers of 128-row tiles (and an empty one):
    in a CTA pair each odd last tile is a half unit (64 rows per CTA), with
    rows past the expert's end inside the tile."""
    rng = np.random.default_rng(17)
    E, H, I = 5, 512, 640
    gs = np.array([128 * 3 + 5, 256, 7, 0, 128 * 4 + 100])  # 4, 2, 1, 0, 5 tiles
    T = int(gs.sum())
    x = torch.from_numpy(rng.standard_normal((T, H), dtype=np.float32)).to(dev(), torch.bfloat16)
    w13 = (torch.randn(E, 2 * I, H, device=dev()) * 0.03).to(torch.bfloat16).transpose(1, 2)
    w2 = (torch.randn(E, H, I, device=dev()) * 0.03).to(torch.bfloat16).transpose(1, 2)
    out = mb.fused_moe_mlp(x, w13, w2, torch.from_numpy(gs).to(dev()))
    ref = O.moe_mlp_grouped(npf(x), npf(w13), npf(w2), gs)
    assert max_abs_rel(npf(out), ref) < TOL
    assert_no_device_error()


# --------------------------------------------------------------------------- top-k form


def topk_case(T, H, I, E, k, routing, dtype, seed=0, w_std=0.02):
    rng = np.random.default_rng(seed)
    x = torch.from_numpy(rng.standard_normal((T, H), dtype=np.float32)).to(dev(), dtype)
    w13 = torch.from_numpy((rng.standard_normal((E, 2 * I, H), dtype=np.float32) * w_std)).to(dev(), dtype)
    w2 = torch.from_numpy((rng.standard_normal((E, H, I), dtype=np.float32) * w_std)).to(dev(), dtype)
    ids, wts = O.synthetic_routing(routing, T, E, k, seed)
    return x, w13.transpose(1, 2), w2.transpose(1, 2), ids, wts


def run_topk(x, w13, w2, ids, wts, scales=None):
    return mb.fused_moe_mlp(x, w13, w2, torch.from_numpy(wts).to(dev()), torch.from_numpy(ids).to(dev()),
                            scales=scales)


@pytest.mark.parametrize("T,H,I,E,k,routing,dtype", [
    (64, 1024, 512, 8, 2, "uniform-softmax", torch.float32),    # config 1: tiny fp32 (tf32 tensor cores)
    (64, 1024, 512, 8, 2, "uniform-softmax", torch.bfloat16),
    (300, 512, 384, 16, 4, "sigmoid", torch.float16),
    (1, 2048, 768, 128, 8, "zipf1.2", torch.bfloat16),          # config 3 decode shapes
    (32, 2048, 768, 128, 8, "zipf1.2", torch.bfloat16),
    (256, 2048, 768, 128, 8, "zipf1.2", torch.bfloat16),
    (777, 256, 136, 6, 3, "uniform-softmax", torch.bfloat16),   # ragged I (not a multiple of 128)
])
def test_topk_matches_oracle(T, H, I, E, k, routing, dtype, gemm_variant):
    x, w13, w2, ids, wts = topk_case(T, H, I, E, k, routing, dtype)
    y = run_topk(x, w13, w2, ids, wts)
    assert y.dtype == dtype and y.shape == (T, H)
    rnd = None if dtype == torch.float32 else (O.round_bf16 if dtype == torch.bfloat16 else O.round_fp16)
    ref = O.moe_mlp_topk(npf(x), npf(w13), npf(w2), wts, ids, round_hidden=rnd)
    err = max_abs_rel(npf(y), ref)
    assert err < TOL, err
    assert_no_device_error()


def test_topk_max_experts(gemm_variant):
    """1024 experts (the GEMMs' and router's limit), 8 per token, through the
    GPU router and the fused op."""
    T, H, I, E, k = 96, 256, 128, 1024, 8
    rng = np.random.default_rng(11)
    x = torch.from_numpy(rng.standard_normal((T, H), dtype=np.float32)).to(dev(), torch.bfloat16)
    w13 = (torch.randn(E, 2 * I, H, device=dev()) * 0.05).to(torch.bfloat16).transpose(1, 2)
    w2 = (torch.randn(E, H, I, device=dev()) * 0.05).to(torch.bfloat16).transpose(1, 2)
    logits = torch.from_numpy(rng.standard_normal((T, E), dtype=np.float32)).to(dev())
    ids, wts = mb.route_topk(logits, top_k=k)
    ids_ref, _ = O.route_topk(npf(logits), k, "softmax")
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_ref)
    y = mb.fused_moe_mlp(x, w13, w2, wts, ids)
    ref = O.moe_mlp_topk(npf(x), npf(w13), npf(w2), wts.cpu().numpy(), ids.cpu().numpy(), round_hidden=O.round_bf16)
    assert max_abs_rel(npf(y), ref) < TOL
    assert_no_device_error()


def test_empty_batch_returns_empty():
    """Zero tokens in either form: an empty [0, H] output, as the reference
    returns for an empty batch."""
    E, H, I = 4, 256, 128
    w13 = (torch.randn(E, 2 * I, H, device=dev()) * 0.05).to(torch.bfloat16).transpose(1, 2)
    w2 = (torch.randn(E, H, I, device=dev()) * 0.05).to(torch.bfloat16).transpose(1, 2)
    x = torch.empty((0, H), dtype=torch.bfloat16, device=dev())
    y = mb.fused_moe_mlp(x, w13, w2, torch.empty((0, 2), device=dev()),
                         torch.empty((0, 2), dtype=torch.int32, device=dev()))
    assert tuple(y.shape) == (0, H)
    y = mb.fused_moe_mlp(x, w13, w2, torch.zeros(E, dtype=torch.int64, device=dev()))
    assert tuple(y.shape) == (0, H)
    assert_no_device_error()


def test_topk_drops_out_of_range_ids(gemm_variant):
    x, w13, w2, ids, wts = topk_case(128, 256, 128, 4, 2, "uniform-softmax", torch.bfloat16)
    ids = ids.copy()
    ids[::3, 1] = -1      # expert-parallel style "not mine"
    ids[5, 0] = 99
    y = run_topk(x, w13, w2, ids, wts)
    ref = O.moe_mlp_topk(npf(x), npf(w13), npf(w2), wts, ids, round_hidden=O.round_bf16)
    assert max_abs_rel(npf(y), ref) < TOL


def test_w8a8_matches_oracle(gemm_variant):
    T, H, I, E, k = 256, 512, 256, 16, 4
    x, w13, w2, ids, wts = topk_case(T, H, I, E, k, "sigmoid", torch.bfloat16, seed=3)
    w13q, w2q, scales = mb.quantize_weights_int8(w13, w2)
    q13, s13 = O.quantize_weight_per_channel(np.swapaxes(npf(w13), 1, 2))
    np.testing.assert_array_equal(w13q.transpose(1, 2).cpu().numpy(), q13)
    np.testing.assert_array_equal(scales[0].cpu().numpy(), s13)
    q2, s2 = O.quantize_weight_per_channel(np.swapaxes(npf(w2), 1, 2))
    y = run_topk(x, w13q, w2q, ids, wts, scales=scales)
    ref = O.moe_mlp_w8a8(npf(x), q13, s13, q2, s2, wts, ids, round_hidden=O.round_bf16)
    err = max_abs_rel(npf(y), ref)
    assert err < TOL, err
    # and against the unquantised fp32 MLP (quantisation error only)
    ref_f = O.moe_mlp_topk(npf(x), npf(w13), npf(w2), wts, ids)
    assert max_abs_rel(npf(y), ref_f) < 5e-2
    assert_no_device_error()


# --------------------------------------------------------------------------- full size (Mixtral layer)


def test_mixtral_full_size_sampled_and_properties():
    """T=4096, H=4096, I=14336, E=8, top-2, bf16: sampled tokens against an fp32
    torch reference of the same op, plus size-independent properties."""
    T, H, I, E, k = 4096, 4096, 14336, 8, 2
    g = torch.Generator(device=dev()).manual_seed(0)
    x = torch.randn(T, H, device=dev(), generator=g).to(torch.bfloat16)
    w13 = (torch.randn(E, 2 * I, H, device=dev(), generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, device=dev(), generator=g) * 0.02).to(torch.bfloat16)
    ids, wts = O.synthetic_routing("uniform-softmax", T, E, k, 0)
    ids_t, wts_t = torch.from_numpy(ids).to(dev()), torch.from_numpy(wts).to(dev())
    y = mb.fused_moe_mlp(x, w13.transpose(1, 2), w2.transpose(1, 2), wts_t, ids_t)
    torch.cuda.synchronize()
    # 512 sampled tokens (every expert among them), against a torch fp32
    # reference of the same op computed expert by expert
    rng = np.random.default_rng(1)
    sample = np.sort(rng.choice(T, size=512, replace=False))
    assert len(np.unique(ids[sample])) == E
    ref = torch.zeros(len(sample), H, device=dev())
    xs = x[torch.from_numpy(sample).to(dev())].float()
    for e in range(E):
        rows, js = np.nonzero(ids[sample] == e)
        if rows.size == 0:
            continue
        gu = xs[torch.from_numpy(rows).to(dev())] @ w13[e].float().t()
        h = (torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]).to(torch.bfloat16).float()
        o = h @ w2[e].float().t()
        wv = torch.from_numpy(wts[sample][rows, js]).to(dev())[:, None]
        ref.index_add_(0, torch.from_numpy(rows).to(dev()), wv * o)
    err = max_abs_rel(npf(y[torch.from_numpy(sample).to(dev())]), npf(ref))
    assert err < TOL, err
    # linearity in the routing weights
    y2 = mb.fused_moe_mlp(x, w13.transpose(1, 2), w2.transpose(1, 2), wts_t * 2, ids_t)
    assert max_abs_rel(npf(y2), 2 * npf(y)) < 1e-2
    # token permutation equivariance
    perm = torch.randperm(T, device=dev(), generator=g)
    y3 = mb.fused_moe_mlp(x[perm], w13.transpose(1, 2), w2.transpose(1, 2), wts_t[perm], ids_t[perm])
    assert max_abs_rel(npf(y3), npf(y[perm])) < 1e-2
    assert torch.isfinite(y).all()
    assert_no_device_error()


@pytest.mark.parametrize("quant", [False, True])
def test_large_output_uses_row_store_combine(quant, gemm_variant):
    """T x H fp32 accumulator above 80 MiB: GEMM2 stores rows and the
    deterministic combine sums them (the path a DeepSeek-V3-sized batch takes)."""
    T, H, I, E, k = 4096, 7168, 256, 32, 8   # 4096 x 7168 x 4 B = 117 MB
    x, w13, w2, ids, wts = topk_case(T, H, I, E, k, "sigmoid", torch.bfloat16, seed=6)
    scales = None
    if quant:
        w13, w2, scales = mb.quantize_weights_int8(w13, w2)
    y = run_topk(x, w13, w2, ids, wts, scales=scales)
    assert _lib.load().moe_fused_experts_workspace_size(T, H, I, E, k, _lib.BF16, _lib.I8 if quant else _lib.BF16) > 0
    sample = np.random.default_rng(0).choice(T, size=64, replace=False)
    if quant:
        q13, s13 = (npf(w13.transpose(1, 2)).astype(np.int8), npf(scales[0]))
        q2, s2 = (npf(w2.transpose(1, 2)).astype(np.int8), npf(scales[1]))
        ref = O.moe_mlp_w8a8(npf(x)[sample], q13, s13, q2, s2, wts[sample], ids[sample], round_hidden=O.round_bf16)
    else:
        ref = O.moe_mlp_topk(npf(x)[sample], npf(w13), npf(w2), wts[sample], ids[sample], round_hidden=O.round_bf16)
    err = max_abs_rel(npf(y)[sample], ref)
    assert err < TOL, err
    # deterministic path: bit-identical on a second call
    y2 = run_topk(x, w13, w2, ids, wts, scales=scales)
    assert torch.equal(y, y2)
    assert_no_device_error()


@pytest.mark.parametrize("dtype,quant", [(torch.bfloat16, False), (torch.bfloat16, True), (torch.float32, False)])
def test_fused_expert_rows_matches_oracle(dtype, quant, gemm_variant):
    R, H, I, E = 333, 512, 384, 6
    rng = np.random.default_rng(8)
    x = torch.from_numpy(rng.standard_normal((R, H), dtype=np.float32)).to(dev(), dtype)
    w13 = torch.from_numpy(rng.standard_normal((E, 2 * I, H), dtype=np.float32) * 0.03).to(dev(), dtype)
    w2 = torch.from_numpy(rng.standard_normal((E, H, I), dtype=np.float32) * 0.03).to(dev(), dtype)
    w13, w2 = w13.transpose(1, 2), w2.transpose(1, 2)
    ids = rng.integers(0, E, size=(R, 1)).astype(np.int32)
    ones = np.ones((R, 1), np.float32)
    scales = None
    if quant:
        w13, w2, scales = mb.quantize_weights_int8(w13, w2)
    out = mb.fused_expert_rows(x, w13, w2, torch.from_numpy(ids).to(dev()), scales=scales)
    rnd = None if dtype == torch.float32 else O.round_bf16
    if quant:
        ref = O.moe_mlp_w8a8(npf(x), npf(w13.transpose(1, 2)).astype(np.int8), npf(scales[0]),
                             npf(w2.transpose(1, 2)).astype(np.int8), npf(scales[1]), ones, ids, round_hidden=rnd)
    else:
        ref = O.moe_mlp_topk(npf(x), npf(w13), npf(w2), ones, ids, round_hidden=rnd)
    assert max_abs_rel(npf(out), ref) < TOL
    assert_no_device_error()


@pytest.mark.parametrize("T,k,E,kernels", [
    (2, 8, 64, 1),      # <= 16 tokens and 128 slots: the one-launch decode kernel
    (20, 1, 64, 3),     # <= 32 slots: prep + gate_up + down converting the output itself
    (64, 2, 4, 4),      # <= 4096 slots: prep + gate_up + down + convert
    (2100, 2, 4, 6),    # align + scatter + gate_up + output clear + down + convert
])
def test_launch_counter_counts_kernels(T, k, E, kernels):
    x, w13, w2, ids, wts = topk_case(T, 256, 128, E, k, "uniform-softmax", torch.bfloat16)
    lib = _lib.load()
    before = lib.moe_launch_count()
    run_topk(x, w13, w2, ids, wts)
    assert lib.moe_launch_count() - before == kernels


@pytest.mark.parametrize("T", [1, 256])
def test_programmatic_dependent_launch_matches_serial(T):
    """Kernels chained by programmatic dependent launch (the default) give the
    results of plain stream-ordered launches: every kernel waits for its
    predecessors before touching memory."""
    lib = _lib.load()
    H, I, E, k = 2048, 768, 128, 8
    x, w13, w2, ids, wts = topk_case(T, H, I, E, k, "zipf1.2", torch.bfloat16, seed=40 + T)
    gs = torch.from_numpy(np.bincount(ids.reshape(-1), minlength=E)).to(dev())
    order = np.argsort(ids.reshape(-1), kind="stable")
    xg = x[torch.from_numpy(order // k).to(dev())].contiguous()
    outs = {}
    for pdl in (1, 0):
        assert lib.moe_set_option(_lib.OPT_PDL, pdl) == 0
        try:
            ys = [run_topk(x, w13, w2, ids, wts) for _ in range(3)]  # back to back on one stream
            pre = mb.fused_moe_mlp(xg, w13, w2, gs)
        finally:
            lib.moe_set_option(_lib.OPT_PDL, 1)
        outs[pdl] = (ys, pre)
    ref = O.moe_mlp_topk(npf(x), npf(w13), npf(w2), wts, ids, round_hidden=O.round_bf16)
    for y in outs[1][0] + outs[0][0]:
        assert max_abs_rel(npf(y), ref) < TOL
    # the pre-routed form has no atomics: bit-identical with and without
    assert torch.equal(outs[1][1], outs[0][1])
    assert_no_device_error()


def test_bounded_wait_expires_and_context_survives():
    """A pipeline wait that nothing satisfies gives up after its limit and
    reports through the device error flag; the GPU context stays usable."""
    assert mb.device_error(dev()) == 0
    _lib.call("moe_selftest_wait_timeout", 200_000_000, torch.cuda.current_stream().cuda_stream)  # 0.2 s
    assert mb.device_error(dev()) == 6
    assert mb.device_error(dev()) == 0  # reading clears it
    x, w13, w2, ids, wts = topk_case(64, 256, 128, 4, 2, "uniform-softmax", torch.bfloat16)
    y = run_topk(x, w13, w2, ids, wts)
    ref = O.moe_mlp_topk(npf(x), npf(w13), npf(w2), wts, ids, round_hidden=O.round_bf16)
    assert max_abs_rel(npf(y), ref) < TOL
    assert_no_device_error()


@pytest.mark.parametrize("T", [1, 32])
def test_cuda_graph_replay_matches_eager(T):
    """Decode-sized calls captured once and replayed with new inputs."""
    H, I, E, k = 2048, 768, 128, 8
    x, w13, w2, ids, wts = topk_case(T, H, I, E, k, "zipf1.2", torch.bfloat16, seed=T)
    cap = mb.CapturedMoeMLP(w13, w2, T, k)
    for seed in (T + 1, T + 2):  # two replays with different tokens and routing
        x2, _, _, ids2, wts2 = topk_case(T, H, I, E, k, "zipf1.2", torch.bfloat16, seed=seed)
        y = cap(x2, torch.from_numpy(wts2).to(dev()), torch.from_numpy(ids2).to(dev())).clone()
        y_ref = run_topk(x2, w13, w2, ids2, wts2)
        # the fused combine adds the k expert rows with fp32 atomics, so two
        # runs can differ by the order of those additions: after the bf16
        # rounding, by one rounding step (2^-8 of an element, bounded here
        # by 2^-7 of the largest)
        assert max_abs_rel(npf(y), npf(y_ref)) <= 2.0 ** -7
    assert_no_device_error()


def test_cuda_graph_replay_pair_gemms():
    """A layer large enough for CTA pairs (experts with odd tile counts, so
    half units too), captured once and replayed with new inputs."""
    T, H, I, E, k = 2048, 1024, 1024, 4, 2  # ~1024 slots per expert: pairs, odd tile counts
    x, w13, w2, ids, wts = topk_case(T, H, I, E, k, "uniform-softmax", torch.bfloat16, seed=3)
    cap = mb.CapturedMoeMLP(w13, w2, T, k)
    for seed in (4, 5):
        x2, _, _, ids2, wts2 = topk_case(T, H, I, E, k, "uniform-softmax", torch.bfloat16, seed=seed)
        y = cap(x2, torch.from_numpy(wts2).to(dev()), torch.from_numpy(ids2).to(dev())).clone()
        y_ref = run_topk(x2, w13, w2, ids2, wts2)
        assert max_abs_rel(npf(y), npf(y_ref)) <= 2.0 ** -7  # fp32 atomic order, as above
        ref = O.moe_mlp_topk(npf(x2), npf(w13), npf(w2), wts2, ids2, round_hidden=O.round_bf16)
        assert max_abs_rel(npf(y), ref) < TOL
    assert_no_device_error()


@pytest.mark.parametrize("pair", [1, 0])
def test_stream_k_combine_matches_whole_tiles(pair):
    """With MOE_OPT_GEMM_STREAM_K the down GEMM's combine epilogue splits the
    partial last wave's (tile, K block) work over the grid; partial sums must
    add up to the whole-tile result (fp32 atomics: equal up to summation
    order)."""
    lib = _lib.load()
    T, H, I, E, k = 1000, 1024, 1536, 8, 2  # K = I: 24 blocks per tile, tiles not a multiple of the grid
    x, w13, w2, ids, wts = topk_case(T, H, I, E, k, "uniform-softmax", torch.bfloat16, seed=21)
    old_pair = lib.moe_get_option(_lib.OPT_GEMM_CTA_PAIR)
    lib.moe_set_option(_lib.OPT_GEMM_CTA_PAIR, pair)
    try:
        lib.moe_set_option(_lib.OPT_GEMM_STREAM_K, 1)
        y_sk = run_topk(x, w13, w2, ids, wts)
        lib.moe_set_option(_lib.OPT_GEMM_STREAM_K, 0)
        y_tiles = run_topk(x, w13, w2, ids, wts)
    finally:
        lib.moe_set_option(_lib.OPT_GEMM_STREAM_K, 0)
        lib.moe_set_option(_lib.OPT_GEMM_CTA_PAIR, old_pair)
    # partial sums reach the fp32 accumulator in another order: the bf16
    # outputs may differ by one rounding step (2^-7 relative)
    assert max_abs_rel(npf(y_sk), npf(y_tiles)) <= 2.0 ** -7
    ref = O.moe_mlp_topk(npf(x), npf(w13), npf(w2), wts, ids, round_hidden=O.round_bf16)
    assert max_abs_rel(npf(y_sk), ref) < TOL
    assert_no_device_error()


def test_kernel_clocks_time_each_gemm_launch():
    """MOE_OPT_KERNEL_CLOCKS: every gate_up and down launch is timed on the
    device; the summed busy time fits inside the CUDA-event time of the calls
    and each class counts exactly its launches."""
    import ctypes
    lib = _lib.load()
    x, w13, w2, ids, wts = topk_case(512, 1024, 1024, 8, 2, "uniform-softmax", torch.bfloat16, seed=21)
    tot = (ctypes.c_uint64 * _lib.NUM_CLOCKS)()
    cnt = (ctypes.c_uint64 * _lib.NUM_CLOCKS)()
    st = torch.cuda.current_stream().cuda_stream
    lib.moe_set_option(_lib.OPT_KERNEL_CLOCKS, 1)
    try:
        run_topk(x, w13, w2, ids, wts)
        _lib.call("moe_kernel_clocks", tot, cnt, _lib.NUM_CLOCKS, 1, st)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(3):
            run_topk(x, w13, w2, ids, wts)
        e1.record()
        torch.cuda.synchronize()
        _lib.call("moe_kernel_clocks", tot, cnt, _lib.NUM_CLOCKS, 1, st)
    finally:
        lib.moe_set_option(_lib.OPT_KERNEL_CLOCKS, 0)
    assert list(cnt) == [3, 3]
    assert all(t > 0 for t in tot)
    assert (tot[0] + tot[1]) / 1e6 <= e0.elapsed_time(e1) * 1.02
    _lib.call("moe_kernel_clocks", tot, cnt, _lib.NUM_CLOCKS, 0, st)
    assert list(cnt) == [0, 0]  # the read above cleared them; clocks off since
    assert_no_device_error()
