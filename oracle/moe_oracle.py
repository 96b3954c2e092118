"""CPU oracle for the fused MoE MLP path — TEST INFRASTRUCTURE ONLY.

This module restates, in numpy on the CPU, the algorithm of the reference
(CrDem/mail) for the fused MoE MLP and defines the stages of the top-k form
(routing, align, int8 quant, weighted combine) that the reference does not
contain. It is what the parity tests, smoke() and
the CPU-baseline leg of bench.py compare against; the product path
(mail_b200 / libmoe_b200.so) never imports it.

Pinning
  * moe_mlp_grouped, build_tile_schedule, tile_schedule_exact are pinned by
    golden vectors generated from the reference's own Python functions
    (tests/golden/make_golden.py -> tests/golden/*.npz).
  * route_topk, align, quant_int8_rows, combine, the w8a8 MLP: the reference
    has no code for these (routing/quant/combine live in the absent sglang /
    torch_npu ops), so their parity is UNPINNED against the reference; the
    semantics below are the definitions the CUDA kernels must match
    bit-exactly (integer/index work) or within tolerance (floating point).

Reference citations are file:line within the CrDem/mail project.
"""
from __future__ import annotations

import numpy as np

# ---------------------------------------------------------------------------
# Tile schedule


def build_tile_schedule(group_sizes, num_tokens: int, block_m: int):
    """Static-grid tile schedule, restating fused_moe_mlp_triton.py:91-119.

    Returns int64 arrays (tile_expert, tile_row_start, tile_row_count) of
    length grid = ceil(num_tokens / block_m) + E, and grid. Tiles past the
    real schedule carry expert E-1, row_start 0, row_count 0 (:105-112).
    """
    gs = np.asarray(group_sizes, dtype=np.int64)
    E = gs.shape[0]
    offsets = np.zeros(E + 1, np.int64)
    offsets[1:] = np.cumsum(gs)                                     # :95-96
    tiles = (gs + block_m - 1) // block_m                           # :98
    tcum = np.zeros(E + 1, np.int64)
    tcum[1:] = np.cumsum(tiles)                                     # :99-100
    grid = -(-num_tokens // block_m) + E                            # :102
    idx = np.arange(grid, dtype=np.int64)
    expert = np.searchsorted(tcum[1:], idx, side="right")           # :105
    valid = expert < E                                              # :106
    expert = np.minimum(expert, E - 1)                              # :107
    local = idx - tcum[expert]                                      # :109
    start = np.where(valid, offsets[expert] + local * block_m, 0)   # :110
    count = np.clip(offsets[expert + 1] - start, 0, block_m)        # :111
    count = np.where(valid, count, 0)                               # :112
    return expert.astype(np.int64), start.astype(np.int64), count.astype(np.int64), int(grid)


def tile_schedule_exact(group_sizes, block_m: int):
    """Exact-grid variant, restating fixed_kernel.py:126-163 (grid = sum of
    ceil(gs / block_m), obtained there with a host sync at :140)."""
    gs = np.asarray(group_sizes, dtype=np.int64)
    grid = int(((gs + block_m - 1) // block_m).sum())
    e, s, c, _ = build_tile_schedule(gs, max(int(gs.sum()), 0), block_m)
    return e[:grid], s[:grid], c[:grid], grid


# ---------------------------------------------------------------------------
# Expert MLP


def silu(x):
    with np.errstate(over="ignore"):
        return x / (np.float32(1.0) + np.exp(-x))


def moe_mlp_grouped(x, w13, w2, group_sizes, round_hidden=None):
    """Per-expert loop over pre-grouped rows, restating fixed_kernel.py:232-249
    and independent_test.py:50-90: fp32 math, gate = first I columns of
    x @ w13[e] (w13 logical [E, H, 2I], w2 logical [E, I, H]).

    round_hidden, if given, is applied to h before the down projection (the
    reference's Triton kernels round h to the weight dtype,
    fused_moe_mlp_triton.py:66). Returns float32 [S, H]; rows no group covers
    are zero (the reference zero-initialises its output, :142-143).
    """
    x = np.asarray(x, np.float32)
    w13 = np.asarray(w13, np.float32)
    w2 = np.asarray(w2, np.float32)
    gs = np.asarray(group_sizes, np.int64)
    inter = w13.shape[2] // 2
    out = np.zeros((x.shape[0], w2.shape[2]), np.float32)
    row = 0
    for e in range(w13.shape[0]):
        n = int(gs[e])
        if n == 0:
            continue
        gate_up = x[row:row + n] @ w13[e]
        h = silu(gate_up[:, :inter]) * gate_up[:, inter:]
        if round_hidden is not None:
            h = round_hidden(h)
        out[row:row + n] = h @ w2[e]
        row += n
    return out


# ---------------------------------------------------------------------------
# Routing (ABSENT in the reference: external npu_moe_init_routing_v2)


def route_topk(logits, top_k: int, scoring: str = "softmax", renormalize: bool = True):
    """logits [T, E] -> (topk_ids int32 [T, k], topk_weights fp32 [T, k]).

    The k largest logits are chosen in descending order, ties towards the
    lower expert id (softmax and sigmoid are monotonic, so these are the
    top-k scores). Weights in fp32: softmax exp(l - max) / sum over all
    experts, or over the k chosen when renormalising; sigmoid 1/(1+exp(-l)),
    divided by the sum over the k chosen when renormalising.
    """
    lg = np.asarray(logits, np.float32)
    order = np.argsort(-lg, axis=1, kind="stable")[:, :top_k]
    top = np.take_along_axis(lg, order, axis=1)
    with np.errstate(over="ignore"):
        if scoring == "softmax":
            m = lg.max(axis=1, keepdims=True)
            sc = np.exp(top - m).astype(np.float32)
            den = sc.sum(axis=1, keepdims=True) if renormalize else \
                np.exp(lg - m).astype(np.float32).sum(axis=1, keepdims=True)
            w = sc / den
        elif scoring == "sigmoid":
            sc = (np.float32(1.0) / (np.float32(1.0) + np.exp(-top))).astype(np.float32)
            w = sc / sc.sum(axis=1, keepdims=True) if renormalize else sc
        else:
            raise ValueError(scoring)
    return order.astype(np.int32), w.astype(np.float32)


def align(topk_ids, num_experts: int, block_m: int):
    """Stable counting sort of the T*k slots by expert, padded per expert.

    Slot s = t * k + j. Slots of expert e occupy padded rows
    [poff[e], poff[e] + count[e]) in increasing slot order; each segment is
    padded with -1 up to a multiple of block_m. Ids outside [0, E) are dropped.
    Returns dict(sorted_slots [padded_total], slot_pos [S], group_sizes [E],
    padded_offsets [E+1], tile_row_start, tile_row_count, tile_cumsum [E+1],
    num_tiles, dropped).
    """
    ids = np.asarray(topk_ids).reshape(-1).astype(np.int64)
    S = ids.shape[0]
    valid = (ids >= 0) & (ids < num_experts)
    counts = np.bincount(ids[valid], minlength=num_experts).astype(np.int64)
    tiles = (counts + block_m - 1) // block_m
    poff = np.zeros(num_experts + 1, np.int64)
    poff[1:] = np.cumsum(tiles * block_m)
    tcum = np.zeros(num_experts + 1, np.int64)
    tcum[1:] = np.cumsum(tiles)
    sorted_slots = np.full(int(poff[-1]), -1, np.int32)
    slot_pos = np.full(S, -1, np.int32)
    slots = np.nonzero(valid)[0]
    order = slots[np.argsort(ids[slots], kind="stable")]
    seg_start = np.concatenate([[0], np.cumsum(counts)])
    for e in range(num_experts):
        sl = order[seg_start[e]:seg_start[e + 1]]
        pos = poff[e] + np.arange(sl.shape[0])
        sorted_slots[pos] = sl
        slot_pos[sl] = pos
    n = int(tcum[-1])
    row_start = np.zeros(n, np.int64)
    row_count = np.zeros(n, np.int64)
    for e in range(num_experts):
        for j in range(int(tiles[e])):
            i = int(tcum[e]) + j
            row_start[i] = poff[e] + j * block_m
            row_count[i] = min(block_m, counts[e] - j * block_m)
    return dict(sorted_slots=sorted_slots, slot_pos=slot_pos, group_sizes=counts.astype(np.int32),
                padded_offsets=poff.astype(np.int32), tile_row_start=row_start, tile_row_count=row_count,
                tile_cumsum=tcum.astype(np.int32), num_tiles=n, dropped=int((~valid).sum()))


# ---------------------------------------------------------------------------
# int8 (ABSENT in the reference)


def _quant_rows_last_axis(x):
    """Symmetric int8 along the last axis: s = absmax / 127 and
    inv = 127 / absmax (both fp32, correctly rounded), q = clamp(rint(x * inv),
    -127, 127) with round-half-to-even; all-zero rows give s = 0, q = 0."""
    x = np.asarray(x, np.float32)
    amax = np.abs(x).max(axis=-1).astype(np.float32) if x.shape[-1] else np.zeros(x.shape[:-1], np.float32)
    s = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        inv = np.where(amax > 0, np.float32(127.0) / amax, np.float32(0.0)).astype(np.float32)
    q = np.rint(x * inv[..., None]).astype(np.float32)
    return np.clip(q, -127, 127).astype(np.int8), s


def quant_int8_rows(x):
    """Per-token (per-row) int8 activation quantisation; see
    _quant_rows_last_axis for the exact arithmetic."""
    return _quant_rows_last_axis(x)


def quantize_weight_per_channel(w):
    """w [..., N, K] (K-major rows = output channels) -> int8 + fp32 scale
    [..., N] = absmax / 127 over each row, same arithmetic as the per-token
    activation quantisation."""
    return _quant_rows_last_axis(w)


# ---------------------------------------------------------------------------
# Top-k MoE MLP (routing align + weighted combine around the expert MLP)


def _accumulate_rows(y, rows, vals):
    """y[rows] += vals, correct for repeated rows (an id listed twice)."""
    if np.unique(rows).size == rows.size:
        y[rows] += vals
    else:
        np.add.at(y, rows, vals)


def moe_mlp_topk(x, w13, w2, topk_weights, topk_ids, round_hidden=None):
    """y[t] = sum_j topk_weights[t, j] * MLP_{topk_ids[t, j]}(x[t]) in fp32.

    w13 logical [E, H, 2I], w2 logical [E, I, H] (fixed_kernel.py:6-13);
    the per-expert MLP is the same restatement as moe_mlp_grouped. Slots with
    ids outside [0, E) contribute nothing.
    """
    x = np.asarray(x, np.float32)
    T, H = x.shape
    E = w13.shape[0]
    k = topk_ids.shape[1]
    ids = np.asarray(topk_ids).reshape(-1)
    wts = np.asarray(topk_weights, np.float32).reshape(-1)
    y = np.zeros((T, H), np.float32)
    inter = w13.shape[2] // 2
    for e in range(E):
        slots = np.nonzero(ids == e)[0]
        if slots.size == 0:
            continue
        tok = slots // k
        gu = x[tok] @ np.asarray(w13[e], np.float32)
        h = silu(gu[:, :inter]) * gu[:, inter:]
        if round_hidden is not None:
            h = round_hidden(h)
        o = h @ np.asarray(w2[e], np.float32)
        _accumulate_rows(y, tok, wts[slots, None] * o)
    return y


def moe_mlp_w8a8(x, w13_q, w13_s, w2_q, w2_s, topk_weights, topk_ids, round_hidden=None):
    """w8a8 top-k MoE MLP with the quantisation points of the CUDA path:

    x rows quantised per token (quant_int8_rows); GEMM1 accumulated exactly
    in integers, dequantised by x_scale[t] * w13_s[e, n]; SwiGLU in fp32;
    h optionally rounded (round_hidden, bf16 on the GPU path) then quantised
    per row; GEMM2 exact in integers, dequantised by h_scale * w2_s[e, c];
    weighted combine in fp32.
    w13_q: int8 [E, 2I, H] (K-major), w13_s [E, 2I]; w2_q int8 [E, H, I],
    w2_s [E, H].
    """
    x = np.asarray(x, np.float32)
    T, H = x.shape
    E = w13_q.shape[0]
    inter = w13_q.shape[1] // 2
    k = topk_ids.shape[1]
    ids = np.asarray(topk_ids).reshape(-1)
    wts = np.asarray(topk_weights, np.float32).reshape(-1)
    xq, xs = quant_int8_rows(x)
    y = np.zeros((T, H), np.float32)
    for e in range(E):
        slots = np.nonzero(ids == e)[0]
        if slots.size == 0:
            continue
        tok = slots // k
        # integer products summed in float64: exact while |acc| < 2**53
        acc = xq[tok].astype(np.float64) @ w13_q[e].astype(np.float64).T
        gu = (acc.astype(np.float32) * xs[tok, None]) * w13_s[e][None, :]
        h = silu(gu[:, :inter]) * gu[:, inter:]
        if round_hidden is not None:
            h = round_hidden(h)
        hq, hs = quant_int8_rows(h)
        acc2 = hq.astype(np.float64) @ w2_q[e].astype(np.float64).T
        o = (acc2.astype(np.float32) * hs[:, None]) * w2_s[e][None, :]
        _accumulate_rows(y, tok, wts[slots, None] * o)
    return y


def round_bf16(a):
    """Round fp32 to the nearest bfloat16 (ties to even), returned as fp32."""
    a = np.ascontiguousarray(a, np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(a), a, out)


def round_fp16(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


# ---------------------------------------------------------------------------
# Seeded synthetic inputs with the shapes/distributions of the five workloads


def zipf_topk(rng, T: int, E: int, k: int, s: float, perm=None):
    """Sample k distinct experts per token from a Zipf(s) popularity over a
    seeded permutation of the expert ids (without replacement)."""
    ranks = np.arange(1, E + 1, dtype=np.float64)
    p = ranks ** (-s)
    p /= p.sum()
    perm = rng.permutation(E) if perm is None else perm
    ids = np.empty((T, k), np.int32)
    for t in range(T):
        ids[t] = perm[rng.choice(E, size=k, replace=False, p=p)]
    return ids


def synthetic_routing(name: str, T: int, E: int, k: int, seed: int = 0):
    """(topk_ids, topk_weights) for a workload.

    uniform-softmax: logits ~ N(0,1), softmax, top-k, renormalise
    sigmoid:         logits ~ N(0,1), sigmoid, top-k, renormalise
    zipf1.2:         Zipf(1.2) expert choice, softmax over sampled logits
    hot25-zipf1.0:   25% of tokens forced to one hot expert, rest Zipf(1.0)
    """
    rng = np.random.default_rng(seed)
    if name in ("uniform-softmax", "sigmoid"):
        logits = rng.standard_normal((T, E), dtype=np.float32)
        return route_topk(logits, k, "softmax" if name == "uniform-softmax" else "sigmoid")
    if name == "zipf1.2" or name == "hot25-zipf1.0":
        s = 1.2 if name == "zipf1.2" else 1.0
        ids = zipf_topk(rng, T, E, k, s)
        if name == "hot25-zipf1.0":
            hot = int(rng.integers(E))
            forced = rng.choice(T, size=T // 4, replace=False)
            for t in forced:
                if hot not in ids[t]:
                    ids[t, k - 1] = hot
        logits = rng.standard_normal((T, k), dtype=np.float32)
        w = np.exp(logits - logits.max(axis=1, keepdims=True))
        w = (w / w.sum(axis=1, keepdims=True)).astype(np.float32)
        return ids.astype(np.int32), w
    raise ValueError(name)


# ---------------------------------------------------------------------------
# Expert-parallel receive layout (no reference counterpart)


def ep_plan(counts_all, rank: int, experts_per_rank: int, block_m: int = 128):
    """Receive layout of expert parallelism over W ranks.

    counts_all [W, E]: slots each rank routes to each global expert. Owner d
    of expert e = e // EL stores expert e's rows at padded rows
    [P(e), P(e) + pad(N_e)) of its buffer (P = exclusive prefix of the padded
    totals within d's experts, N_e = sum over ranks), source s's rows after
    those of ranks < s. Returns dest_base [E] for `rank` as the source and
    the tile rows (row_start, row_count, tile_cumsum, total_rows) of `rank`
    as the owner.
    """
    C = np.asarray(counts_all, np.int64)
    W, E = C.shape
    EL = experts_per_rank
    tot = C.sum(axis=0)
    pad = (tot + block_m - 1) // block_m * block_m
    dest_base = np.zeros(E, np.int64)
    for e in range(E):
        d = e // EL
        dest_base[e] = pad[d * EL:e].sum() + C[:rank, e].sum()
    local = np.arange(rank * EL, (rank + 1) * EL)
    tiles = (tot[local] + block_m - 1) // block_m
    tcum = np.concatenate([[0], np.cumsum(tiles)])
    starts, counts = [], []
    for i, e in enumerate(local):
        base = pad[rank * EL:e].sum()
        for j in range(int(tiles[i])):
            starts.append(base + j * block_m)
            counts.append(min(block_m, tot[e] - j * block_m))
    return dict(dest_base=dest_base.astype(np.int32), tile_row_start=np.array(starts, np.int64),
                tile_row_count=np.array(counts, np.int64), tile_cumsum=tcum.astype(np.int32),
                total_rows=int(pad[local].sum()))
