"""The oracle against the golden vectors produced by the reference itself
(tests/golden/make_golden.py), plus self-consistency of the oracle stages the
reference does not contain."""
import os

import numpy as np
import pytest

from oracle import moe_oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
MLP_CASES = ["mlp_selfcheck_f32", "mlp_selftest_f16", "mlp_ragged_f32"]
REF_KEYS = ["ref_golden_loop", "ref_fixed_kernel", "ref_linear_layout", "ref_golden_vectorized",
            "ref_triton_interpreted"]


def load(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))


@pytest.mark.parametrize("case", MLP_CASES)
def test_grouped_mlp_matches_reference(case):
    d = load(case)
    f16 = d["x"].dtype == np.float16
    for key in REF_KEYS:
        # the reference's Triton kernels round h to the weight dtype
        # (partially_fused_moe_mlp_triton.py:111); its torch loops do not
        rnd = (O.round_fp16 if f16 else None) if key == "ref_triton_interpreted" else None
        out = O.moe_mlp_grouped(d["x"], d["w13"], d["w2"], d["group_sizes"], round_hidden=rnd)
        if f16:
            out = O.round_fp16(out)
        ref = d[key]
        scale = np.abs(ref).max()
        # fp32 paths agree to summation-order noise; fp16 outputs to one fp16 ulp
        tol = (1e-3 if f16 else 2e-5) * scale
        assert np.abs(out - ref).max() <= tol, (key, np.abs(out - ref).max(), scale)


def test_reference_layouts_agree():
    d = load("mlp_selftest_f16")
    np.testing.assert_array_equal(d["ref_fixed_kernel"], d["ref_linear_layout"])


def schedule_cases():
    t = load("tile_schedule")
    names = sorted({k.split("/")[0] for k in t.files})
    return [(n, bm) for n in names for bm in (16, 32, 64, 128, 256)]


@pytest.mark.parametrize("name,bm", schedule_cases())
def test_tile_schedule_bit_exact(name, bm):
    t = load("tile_schedule")
    gs = t[f"{name}/group_sizes"]
    e, s, c, grid = O.build_tile_schedule(gs, int(gs.sum()), bm)
    assert grid == int(t[f"{name}/bm{bm}/grid"])
    np.testing.assert_array_equal(e, t[f"{name}/bm{bm}/expert"])
    np.testing.assert_array_equal(s, t[f"{name}/bm{bm}/row_start"])
    np.testing.assert_array_equal(c, t[f"{name}/bm{bm}/row_count"])
    e2, s2, c2, g2 = O.tile_schedule_exact(gs, bm)
    assert g2 == int(t[f"{name}/bm{bm}/exact_grid"])
    np.testing.assert_array_equal(e2, t[f"{name}/bm{bm}/exact_expert"])
    np.testing.assert_array_equal(s2, t[f"{name}/bm{bm}/exact_row_start"])
    np.testing.assert_array_equal(c2, t[f"{name}/bm{bm}/exact_row_count"])


@pytest.mark.parametrize("seed,T,E,k", [(0, 64, 8, 2), (1, 37, 5, 3), (2, 300, 64, 6), (3, 1, 128, 8)])
def test_align_is_stable_padded_sort(seed, T, E, k):
    rng = np.random.default_rng(seed)
    ids = rng.integers(-1, E + 1, size=(T, k)).astype(np.int32)   # includes out-of-range ids
    a = O.align(ids, E, 128)
    flat = ids.reshape(-1)
    valid = (flat >= 0) & (flat < E)
    assert a["dropped"] == int((~valid).sum())
    expected = [s for e in range(E) for s in range(flat.size) if flat[s] == e]
    got = a["sorted_slots"][a["sorted_slots"] >= 0]
    np.testing.assert_array_equal(got, expected)
    for s in range(flat.size):
        p = a["slot_pos"][s]
        assert (p == -1) == (not valid[s])
        if p >= 0:
            assert a["sorted_slots"][p] == s
    assert (np.diff(a["padded_offsets"]) % 128 == 0).all()
    np.testing.assert_array_equal(a["group_sizes"], np.bincount(flat[valid], minlength=E))


def test_route_topk_matches_torch():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(5)
    logits = rng.standard_normal((200, 64), dtype=np.float32)
    for scoring in ("softmax", "sigmoid"):
        ids, w = O.route_topk(logits, 6, scoring)
        lt = torch.from_numpy(logits)
        p = torch.softmax(lt, dim=1) if scoring == "softmax" else torch.sigmoid(lt)
        tw, ti = torch.topk(p, 6, dim=1)
        tw = tw / tw.sum(dim=1, keepdim=True)
        np.testing.assert_array_equal(ids, ti.numpy())
        np.testing.assert_allclose(w, tw.numpy(), rtol=1e-6, atol=1e-7)


def test_quant_int8_semantics():
    x = np.array([[0.0, 0.0, 0.0, 0.0], [1.0, -2.0, 0.5, 127.0], [-3.0, 1.5, 0.75, 0.0]], np.float32)
    q, s = O.quant_int8_rows(x)
    assert s[0] == 0 and (q[0] == 0).all()
    assert s[1] == np.float32(127.0) / np.float32(127.0)
    np.testing.assert_array_equal(q[1], [1, -2, 0, 127])  # 0.5 rounds half to even -> 0
    assert np.abs(q).max() <= 127


def test_w8a8_oracle_close_to_float():
    rng = np.random.default_rng(3)
    T, H, I, E, k = 32, 64, 48, 4, 2
    x = rng.standard_normal((T, H), dtype=np.float32)
    w13 = (rng.standard_normal((E, H, 2 * I), dtype=np.float32) * 0.05)
    w2 = (rng.standard_normal((E, I, H), dtype=np.float32) * 0.05)
    ids, wts = O.synthetic_routing("uniform-softmax", T, E, k, seed=1)
    yf = O.moe_mlp_topk(x, w13, w2, wts, ids)
    q13, s13 = O.quantize_weight_per_channel(np.swapaxes(w13, 1, 2))
    q2, s2 = O.quantize_weight_per_channel(np.swapaxes(w2, 1, 2))
    yq = O.moe_mlp_w8a8(x, q13, s13, q2, s2, wts, ids)
    assert np.abs(yq - yf).max() / np.abs(yf).max() < 3e-2


def test_topk_mlp_equals_grouped_mlp():
    rng = np.random.default_rng(11)
    T, H, I, E, k = 40, 32, 24, 5, 2
    x = rng.standard_normal((T, H), dtype=np.float32)
    w13 = rng.standard_normal((E, H, 2 * I), dtype=np.float32) * 0.1
    w2 = rng.standard_normal((E, I, H), dtype=np.float32) * 0.1
    ids, wts = O.synthetic_routing("uniform-softmax", T, E, k, seed=2)
    a = O.align(ids, E, 1)
    rows = a["sorted_slots"]
    xp = x[rows // k]
    outp = O.moe_mlp_grouped(xp, w13, w2, a["group_sizes"])
    y = np.zeros((T, H), np.float32)
    for p, s in enumerate(rows):
        y[s // k] += wts.reshape(-1)[s] * outp[p]
    np.testing.assert_allclose(O.moe_mlp_topk(x, w13, w2, wts, ids), y, rtol=1e-5, atol=1e-5)
