"""Property tests of the oracle's align and expert-parallel receive layout on
random inputs (CPU). The GPU kernels are checked bit-exactly against these
functions, so their invariants are checked here on their own."""
import numpy as np
from hypothesis import given, settings
from hypothesis import strategies as st

from oracle import moe_oracle as O


@settings(max_examples=60, deadline=None)
@given(T=st.integers(0, 300), E=st.integers(1, 64), k=st.integers(1, 8), seed=st.integers(0, 2**31 - 1),
       bm=st.sampled_from([1, 16, 128]))
def test_align_invariants(T, E, k, seed, bm):
    """Every valid slot appears once, grouped by expert in slot order; each
    expert's segment starts on a tile boundary; padding rows are -1; slot_pos
    inverts sorted_slots; invalid ids are dropped."""
    rng = np.random.default_rng(seed)
    ids = rng.integers(-1, E + 1, size=(T, k)).astype(np.int32)  # includes out-of-range ids
    a = O.align(ids, E, bm)
    flat = ids.reshape(-1)
    valid = (flat >= 0) & (flat < E)
    poff = np.asarray(a["padded_offsets"], np.int64)
    ss = np.asarray(a["sorted_slots"], np.int64)
    assert poff[0] == 0 and np.all(np.diff(poff) >= 0) and np.all(poff % bm == 0)
    for e in range(E):
        want = np.nonzero(flat == e)[0]  # stable: slot order
        seg = ss[poff[e]:poff[e + 1]]
        assert np.array_equal(seg[:len(want)], want)
        assert np.all(seg[len(want):] == -1) and len(seg) - len(want) < bm
    pos = np.asarray(a["slot_pos"], np.int64)
    assert np.all(pos[~valid] == -1)
    assert np.array_equal(ss[pos[valid]], np.nonzero(valid)[0])


@settings(max_examples=60, deadline=None)
@given(W=st.sampled_from([1, 2, 4, 8]), EL=st.integers(1, 4), seed=st.integers(0, 2**31 - 1))
def test_ep_receive_layout_is_a_partition(W, EL, seed):
    """Over all source ranks, the rows each source writes into an owner's
    buffer are disjoint, lie inside their expert's padded segment in source
    order, and the owner's tiles cover exactly the rows received."""
    rng = np.random.default_rng(seed)
    E = W * EL
    C = rng.integers(0, 300, size=(W, E))
    C[rng.random((W, E)) < 0.3] = 0  # empty (source, expert) pairs
    plans = [O.ep_plan(C, r, EL) for r in range(W)]
    for d in range(W):
        owner = plans[d]
        used = np.zeros(owner["total_rows"], np.int64)
        for e in range(d * EL, (d + 1) * EL):
            seg0 = sum(int((C[:, x].sum() + 127) // 128 * 128) for x in range(d * EL, e))
            nxt = None
            for s in range(W):
                b = int(plans[s]["dest_base"][e])
                assert nxt is None or b == nxt  # source s follows source s-1
                used[b:b + C[s, e]] += 1
                nxt = b + C[s, e]
                assert seg0 <= b and b + C[s, e] <= seg0 + (C[:, e].sum() + 127) // 128 * 128
        assert used.max(initial=0) <= 1
        covered = np.zeros_like(used)
        for st_, cnt in zip(owner["tile_row_start"], owner["tile_row_count"]):
            covered[st_:st_ + cnt] += 1
        assert np.array_equal(covered, used)
