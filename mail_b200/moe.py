"""Host-side mirror of the reference's fused_moe_mlp interface.

`fused_moe_mlp` keeps the reference's call signature
(fused_moe_mlp_triton.py:121-130, called from sglang at unquant_diff.txt:13-18)
and adds the sglang fused_experts-style top-k form (routing align and
weighted combine inside):

    fused_moe_mlp(x, w13, w2, group_sizes)                      # pre-routed rows
    fused_moe_mlp(hidden_states, w13, w2, topk_weights, topk_ids, scales=None)

Weights use the reference's logical "(E, K, N)" layout: w13[E, H, 2I] (gate =
first I columns) and w2[E, I, H]. The sm_100a kernels read them K-major, i.e.
physically [E, 2I, H] / [E, H, I] — exactly what transpose(1, 2) of nn.Linear
weights gives (kernel_bench.py:229-235) — so such views are used without a
copy; any other stride pattern is made K-major with one copy per call (use
`prepack_weights` once at load time instead).

Every op runs the CUDA kernels of libmoe_b200.so through its C ABI on the
current torch stream. There is no CPU or PyTorch fallback: a missing library
or a non-CUDA tensor raises.
"""
from __future__ import annotations

import warnings

import torch

from . import _lib

_DT = {torch.float32: _lib.F32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16, torch.int8: _lib.I8,
       torch.int32: _lib.I32, torch.int64: _lib.I64}
BLOCK_M = 128  # M tile of the tcgen05 kernels


def _code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}") from None


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("mail_b200 ops run on CUDA tensors only (no CPU fallback)")


def _workspace(nbytes: int, dev) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=dev)


_warned_copy = False


def kmajor(w: torch.Tensor) -> torch.Tensor:
    """Logical (E, K, N) weight -> contiguous K-major [E, N, K] storage."""
    global _warned_copy
    wt = w.transpose(1, 2)
    if wt.is_contiguous():
        return wt
    if not _warned_copy:
        warnings.warn("fused_moe_mlp: weights are not K-major; copying them on every call "
                      "(call prepack_weights once at load time)", stacklevel=3)
        _warned_copy = True
    return wt.contiguous()


def prepack_weights(w13: torch.Tensor, w2: torch.Tensor):
    """Returns (w13, w2) logical views whose storage is K-major, copying once
    if needed; pass the results to fused_moe_mlp."""
    return (w13.transpose(1, 2).contiguous().transpose(1, 2), w2.transpose(1, 2).contiguous().transpose(1, 2))


def weights_from_linear(w13_linear: torch.Tensor, w2_linear: torch.Tensor):
    """nn.Linear-layout weights (w13 [E, 2I, H], w2 [E, H, I]) -> logical
    (E, K, N) views with no copy (kernel_bench.py:229-235)."""
    return w13_linear.transpose(1, 2), w2_linear.transpose(1, 2)


def weights_from_checkpoint(gate_proj, up_proj, down_proj, device=None, dtype=None, quantize: bool = False):
    """Per-expert checkpoint tensors -> the op's weight storage, once at load.

    gate_proj[e] and up_proj[e] are the HF `experts.{e}.gate_proj.weight` /
    `up_proj.weight` matrices ([I, H], nn.Linear layout) and down_proj[e] is
    `down_proj.weight` ([H, I]); each argument is a sequence of E tensors or
    one stacked [E, ...] tensor. The reference's loader concatenates gate and
    up on dim 0, stacks the experts and transposes (kernel_bench.py:212-235),
    giving logical w13 [E, H, 2I] (gate = first I columns) and w2 [E, I, H].
    This returns the same logical tensors, built by copying each expert
    straight into K-major storage ([E, 2I, H] / [E, H, I] contiguous, the
    layout the kernels' TMA reads) on `device` (default: the tensors' own),
    cast to `dtype` if given — no concatenated or stacked intermediate.

    quantize=True (CUDA device) converts to w8a8 weights with per-output-
    channel scales (quantize_weights_int8) and returns (w13_q, w2_q, scales);
    otherwise (w13, w2)."""
    E = len(gate_proj)
    if len(up_proj) != E or len(down_proj) != E or E == 0:
        raise ValueError("weights_from_checkpoint: gate_proj, up_proj and down_proj need one entry per expert")
    I, H = gate_proj[0].shape
    if tuple(down_proj[0].shape) != (H, I):
        raise ValueError(f"weights_from_checkpoint: down_proj is {tuple(down_proj[0].shape)}, expected {(H, I)}")
    dev = torch.device(device) if device is not None else gate_proj[0].device
    dt = dtype or gate_proj[0].dtype
    w13 = torch.empty((E, 2 * I, H), dtype=dt, device=dev)
    w2 = torch.empty((E, H, I), dtype=dt, device=dev)
    for e in range(E):
        if tuple(gate_proj[e].shape) != (I, H) or tuple(up_proj[e].shape) != (I, H):
            raise ValueError(f"weights_from_checkpoint: expert {e}: gate/up must both be {(I, H)}")
        if tuple(down_proj[e].shape) != (H, I):
            raise ValueError(f"weights_from_checkpoint: expert {e}: down_proj must be {(H, I)}")
        w13[e, :I].copy_(gate_proj[e])
        w13[e, I:].copy_(up_proj[e])
        w2[e].copy_(down_proj[e])
    w13l, w2l = w13.transpose(1, 2), w2.transpose(1, 2)
    if not quantize:
        return w13l, w2l
    _require_cuda(w13l)
    return quantize_weights_int8(w13l, w2l)


# ---------------------------------------------------------------------------
# Building blocks (each one C-ABI call)


def build_tile_schedule(group_sizes: torch.Tensor, num_tokens: int, BLOCK_M: int = BLOCK_M):
    """Device restatement of build_tile_schedule (fused_moe_mlp_triton.py:91-119).

    Returns (tile_expert, tile_row_start, tile_row_count) int64 tensors on
    group_sizes' device and the static grid size cdiv(num_tokens, BLOCK_M) + E.
    """
    _require_cuda(group_sizes)
    gs = group_sizes.contiguous()
    if gs.dtype not in (torch.int32, torch.int64):
        gs = gs.to(torch.int64)
    E = gs.numel()
    grid = int(_lib.query("moe_tile_grid", int(num_tokens), E, int(BLOCK_M)))
    if grid < 0:
        raise ValueError("build_tile_schedule: bad arguments")
    dev = gs.device
    te = torch.empty(grid, dtype=torch.int64, device=dev)
    ts = torch.empty(grid, dtype=torch.int64, device=dev)
    tc = torch.empty(grid, dtype=torch.int64, device=dev)
    _lib.call("moe_tile_schedule", gs.data_ptr(), _code(gs), E, int(num_tokens), int(BLOCK_M), te.data_ptr(),
              ts.data_ptr(), tc.data_ptr(), None, _stream(dev))
    return te, ts, tc, grid


def route_topk(logits: torch.Tensor, top_k: int, scoring: str = "softmax", renormalize: bool = True):
    """Router on the GPU: logits [T, E] -> (topk_ids int32 [T, k],
    topk_weights fp32 [T, k]); the k largest logits, ties to the lower expert
    id; softmax or sigmoid weights, optionally renormalised over the k."""
    _require_cuda(logits)
    lg = logits.contiguous()
    T, E = lg.shape
    ids = torch.empty((T, top_k), dtype=torch.int32, device=lg.device)
    w = torch.empty((T, top_k), dtype=torch.float32, device=lg.device)
    sc = {"softmax": 0, "sigmoid": 1}[scoring]
    _lib.call("moe_route_topk", lg.data_ptr(), _code(lg), T, E, top_k, sc, int(renormalize), ids.data_ptr(),
              w.data_ptr(), _stream(lg.device))
    return ids, w


def moe_align(topk_ids: torch.Tensor, num_experts: int, block_m: int = BLOCK_M) -> dict:
    """Stable block-padded sort of the T*k slots by expert (see moe_b200.h).

    Returns dict(sorted_slots, slot_pos, group_sizes, padded_offsets,
    tile_table, capacity, max_tiles).
    """
    _require_cuda(topk_ids)
    ids = topk_ids.to(torch.int32).contiguous()
    T, k = ids.shape
    S = T * k
    dev = ids.device
    cap = int(_lib.query("moe_align_capacity", S, num_experts, block_m))
    max_tiles = cap // block_m
    sorted_slots = torch.empty(max(cap, 1), dtype=torch.int32, device=dev)
    slot_pos = torch.empty(max(S, 1), dtype=torch.int32, device=dev)
    gs = torch.empty(num_experts, dtype=torch.int32, device=dev)
    poff = torch.empty(num_experts + 1, dtype=torch.int32, device=dev)
    table = torch.empty(int(_lib.query("moe_tile_table_ints", num_experts, max_tiles)), dtype=torch.int32,
                        device=dev)
    ws = _workspace(_lib.query("moe_align_workspace_size", T, k, num_experts, block_m), dev)
    _lib.call("moe_align", ids.data_ptr(), T, k, num_experts, block_m, sorted_slots.data_ptr(), slot_pos.data_ptr(),
              gs.data_ptr(), poff.data_ptr(), table.data_ptr(), ws.data_ptr(), ws.numel(), _stream(dev))
    return dict(sorted_slots=sorted_slots, slot_pos=slot_pos[:S], group_sizes=gs, padded_offsets=poff,
                tile_table=table, capacity=cap, max_tiles=max_tiles)


def quant_int8_rows(x: torch.Tensor):
    """Per-row int8: s = absmax / 127, q = clamp(rint(x * (127 / absmax)), -127, 127)."""
    _require_cuda(x)
    x = x.contiguous()
    R, C = x.shape
    q = torch.empty((R, C), dtype=torch.int8, device=x.device)
    s = torch.empty(max(R, 1), dtype=torch.float32, device=x.device)
    _lib.call("moe_quant_rows", x.data_ptr(), _code(x), R, C, None, q.data_ptr(), s.data_ptr(), _stream(x.device))
    return q, s[:R]


def gather_rows(src: torch.Tensor, sorted_slots: torch.Tensor, top_k: int, rows: int, out_dtype=None,
                rows_dev: torch.Tensor | None = None):
    """dst[p] = src[sorted_slots[p] // top_k] (zero rows for negative slots);
    out_dtype=torch.int8 quantises each row (returns (q, scale))."""
    _require_cuda(src, sorted_slots)
    src = src.contiguous()
    out_dtype = out_dtype or src.dtype
    dst = torch.empty((rows, src.shape[1]), dtype=out_dtype, device=src.device)
    scale = torch.empty(max(rows, 1), dtype=torch.float32, device=src.device) if out_dtype == torch.int8 else None
    _lib.call("moe_gather_rows", src.data_ptr(), _code(src), src.shape[1], sorted_slots.data_ptr(), top_k, rows,
              _ptr(rows_dev), dst.data_ptr(), _code(dst), _ptr(scale), _stream(src.device))
    return (dst, scale[:rows]) if scale is not None else dst


def quantize_weights_int8(w13: torch.Tensor, w2: torch.Tensor):
    """Load-time w8a8 weight prep: logical (E, K, N) weights -> int8 logical
    views with K-major storage and per-output-channel fp32 scales
    s = absmax / 127, q = clamp(rint(w * (127 / absmax)), -127, 127) — the per-row int8
    kernel applied to the K-major rows. Returns
    (w13_q, w2_q, (w13_scale [E, 2I], w2_scale [E, H]))."""
    def q(w):
        wk = kmajor(w)                                  # [E, N, K] contiguous
        E, N, K = wk.shape
        qq, s = quant_int8_rows(wk.reshape(E * N, K))
        return qq.view(E, N, K).transpose(1, 2), s.view(E, N)
    a, sa = q(w13)
    b, sb = q(w2)
    return a, b, (sa, sb)


# ---------------------------------------------------------------------------
# The op


def _check_shapes(x, w13, w2):
    if x.dim() != 2 or w13.dim() != 3 or w2.dim() != 3:
        raise ValueError("fused_moe_mlp: expected x [T, H], w13 [E, H, 2I], w2 [E, I, H]")
    T, H = x.shape
    E, Hw, two_i = w13.shape
    inter = two_i // 2
    if Hw != H or two_i != 2 * inter or tuple(w2.shape) != (E, inter, H):
        raise ValueError(f"fused_moe_mlp: shape mismatch x{tuple(x.shape)} w13{tuple(w13.shape)} "
                         f"w2{tuple(w2.shape)} (expected w13 [E, H, 2I], w2 [E, I, H])")
    return T, H, E, inter


def _prerouted_impl(x, w13, w2, group_sizes):
    """moe_fused_mlp: the reference's call on pre-grouped rows."""
    _require_cuda(x, w13, w2, group_sizes)
    T, H, E, inter = _check_shapes(x, w13, w2)
    x = x.contiguous()
    w13k, w2k = kmajor(w13), kmajor(w2)
    dev = x.device
    gs = group_sizes
    if gs.numel() != E:
        raise ValueError("fused_moe_mlp: group_sizes must have E entries")
    if gs.dtype not in (torch.int32, torch.int64):
        gs = gs.to(torch.int64)
    gs = gs.contiguous()
    if w13.dtype != x.dtype or w2.dtype != x.dtype:
        raise TypeError("fused_moe_mlp: x, w13 and w2 must share a dtype")
    out = torch.empty((T, H), dtype=x.dtype, device=dev)
    ws = _workspace(_lib.query("moe_fused_mlp_workspace_size", T, H, inter, E, _code(x), 128), dev)
    _lib.call("moe_fused_mlp", x.data_ptr(), _code(x), T, H, w13k.data_ptr(), w2k.data_ptr(), E, inter,
              gs.data_ptr(), _code(gs), 128, out.data_ptr(), ws.data_ptr(), ws.numel(), _stream(dev))
    return out


def _weight_scales(x, w13, w2, w13_scale, w2_scale, E, H, inter):
    """(w_code, w13_scale, w2_scale) of a top-k call, checked: int8 weights
    need fp32 scales [E, 2I] and [E, H]; other weights share x's dtype."""
    s13 = s2 = None
    if w13.dtype == torch.int8:
        if w13_scale is None or w2_scale is None:
            raise ValueError("fused_moe_mlp: int8 weights need scales=(w13_scale, w2_scale)")
        s13, s2 = w13_scale.to(torch.float32).contiguous(), w2_scale.to(torch.float32).contiguous()
        if tuple(s13.shape) != (E, 2 * inter) or tuple(s2.shape) != (E, H):
            raise ValueError("fused_moe_mlp: scales must be w13_scale [E, 2I] and w2_scale [E, H]")
    elif w13.dtype != x.dtype or w2.dtype != x.dtype:
        raise TypeError("fused_moe_mlp: weights must share x's dtype or be int8")
    return _code(w13), s13, s2


def _topk_impl(x, w13, w2, topk_weights, topk_ids, w13_scale, w2_scale):
    """moe_fused_experts: align -> GEMMs -> weighted combine."""
    _require_cuda(x, w13, w2, topk_weights, topk_ids)
    T, H, E, inter = _check_shapes(x, w13, w2)
    x = x.contiguous()
    w13k, w2k = kmajor(w13), kmajor(w2)
    dev = x.device
    topk_weights = topk_weights.to(torch.float32).contiguous()
    ids = topk_ids.to(torch.int32).contiguous()
    if topk_weights.shape != ids.shape or ids.dim() != 2 or ids.shape[0] != T:
        raise ValueError("fused_moe_mlp: topk_weights/topk_ids must both be [T, k]")
    k = ids.shape[1]
    w_code, s13, s2 = _weight_scales(x, w13, w2, w13_scale, w2_scale, E, H, inter)
    y = torch.empty((T, H), dtype=x.dtype, device=dev)
    ws = _workspace(_lib.query("moe_fused_experts_workspace_size", T, H, inter, E, k, _code(x), w_code), dev)
    _lib.call("moe_fused_experts", x.data_ptr(), _code(x), T, H, w13k.data_ptr(), w2k.data_ptr(), w_code, E, inter,
              topk_weights.data_ptr(), ids.data_ptr(), k, _ptr(s13), _ptr(s2), y.data_ptr(), ws.data_ptr(),
              ws.numel(), _stream(dev))
    return y


# The two forms (and the logits-in call below) as PyTorch operators (torch.ops.mail_b200.*), so a
# torch.compile'd MoE layer sees one opaque op per call instead of a graph
# break; the fake (meta) kernels give the output shape and dtype for tracing.
@torch.library.custom_op("mail_b200::fused_moe_mlp", mutates_args=())
def _op_prerouted(x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor, group_sizes: torch.Tensor) -> torch.Tensor:
    return _prerouted_impl(x, w13, w2, group_sizes)


@_op_prerouted.register_fake
def _(x, w13, w2, group_sizes):
    T, H, E, _ = _check_shapes(x, w13, w2)
    if group_sizes.numel() != E:
        raise ValueError("fused_moe_mlp: group_sizes must have E entries")
    return x.new_empty((T, H))


@torch.library.custom_op("mail_b200::fused_experts", mutates_args=())
def _op_topk(x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor, topk_weights: torch.Tensor,
             topk_ids: torch.Tensor, w13_scale: torch.Tensor | None, w2_scale: torch.Tensor | None) -> torch.Tensor:
    return _topk_impl(x, w13, w2, topk_weights, topk_ids, w13_scale, w2_scale)


@_op_topk.register_fake
def _(x, w13, w2, topk_weights, topk_ids, w13_scale, w2_scale):
    T, H, _, _ = _check_shapes(x, w13, w2)
    if topk_weights.shape != topk_ids.shape or topk_ids.dim() != 2 or topk_ids.shape[0] != T:
        raise ValueError("fused_moe_mlp: topk_weights/topk_ids must both be [T, k]")
    return x.new_empty((T, H))


def fused_moe_mlp(x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor, group_sizes_or_topk_weights: torch.Tensor,
                  topk_ids: torch.Tensor | None = None, scales=None, BLOCK_M: int = 128, BLOCK_N: int = 128,
                  BLOCK_N2: int = 256, BLOCK_K: int = 256) -> torch.Tensor:
    """Fused expert MLP: grouped GEMM(x, w13) -> silu(gate) * up -> grouped GEMM(., w2).

    Pre-routed form (topk_ids is None) — drop-in for the reference
    (fused_moe_mlp_triton.py:121-160): x [S, H] grouped by expert,
    group_sizes [E]; returns [S, H] in x.dtype (rows beyond sum(group_sizes)
    are zero). dtypes: bf16, fp16, fp32 (fp32 runs on tf32 tensor cores).

    Top-k form: x [T, H], topk_weights [T, k] (fp32), topk_ids [T, k]; returns
    y [T, H] = sum_j topk_weights[t, j] * MLP_{topk_ids[t, j]}(x[t]) in x.dtype.
    int8 w13/w2 select w8a8 with scales=(w13_scale [E, 2I], w2_scale [E, H])
    and dynamic per-token activation quantisation. The combine adds each
    token's k weighted rows with fp32 atomics while the [T, H] fp32
    accumulator fits in L2 (T * H * 4 <= 80 MiB), so the order of those adds,
    and with it the last bit of a bf16 output, can differ from run to run
    (by at most one bf16 rounding step); larger outputs use a deterministic
    row-store combine.

    Under torch.compile the call is one operator (torch.ops.mail_b200.
    fused_moe_mlp / fused_experts); eager calls go straight to the library.
    BLOCK_* are accepted for signature compatibility; the sm_100a kernels use
    fixed 128 x 256 tiles and results do not depend on them.
    """
    del BLOCK_M, BLOCK_N, BLOCK_N2, BLOCK_K
    compiling = torch.compiler.is_compiling()
    if topk_ids is None:
        if compiling:
            return torch.ops.mail_b200.fused_moe_mlp(x, w13, w2, group_sizes_or_topk_weights)
        return _prerouted_impl(x, w13, w2, group_sizes_or_topk_weights)
    s13, s2 = scales if scales is not None else (None, None)
    if compiling:
        return torch.ops.mail_b200.fused_experts(x, w13, w2, group_sizes_or_topk_weights, topk_ids, s13, s2)
    return _topk_impl(x, w13, w2, group_sizes_or_topk_weights, topk_ids, s13, s2)


def _check_logits(x, w13, w2, router_logits, top_k, scoring):
    T, H, E, inter = _check_shapes(x, w13, w2)
    if router_logits.dim() != 2 or tuple(router_logits.shape) != (T, E):
        raise ValueError(f"fused_moe_mlp_from_logits: router_logits must be [T, E] = [{T}, {E}]")
    if not 1 <= top_k <= min(E, 32):
        raise ValueError(f"fused_moe_mlp_from_logits: top_k {top_k} outside [1, min(E, 32)]")
    if scoring not in ("softmax", "sigmoid"):
        raise ValueError(f"fused_moe_mlp_from_logits: scoring must be softmax or sigmoid, not {scoring!r}")
    return T, H, E, inter


def _from_logits_impl(x, w13, w2, router_logits, top_k, scoring, renormalize, w13_scale, w2_scale):
    """moe_fused_experts_from_logits: router -> align -> GEMMs -> combine."""
    _require_cuda(x, w13, w2, router_logits)
    T, H, E, inter = _check_logits(x, w13, w2, router_logits, top_k, scoring)
    lg = router_logits.contiguous()
    x = x.contiguous()
    w13k, w2k = kmajor(w13), kmajor(w2)
    dev = x.device
    w_code, s13, s2 = _weight_scales(x, w13, w2, w13_scale, w2_scale, E, H, inter)
    y = torch.empty((T, H), dtype=x.dtype, device=dev)
    ids = torch.empty((T, top_k), dtype=torch.int32, device=dev)
    wts = torch.empty((T, top_k), dtype=torch.float32, device=dev)
    sc = {"softmax": 0, "sigmoid": 1}[scoring]
    ws = _workspace(_lib.query("moe_fused_experts_workspace_size", T, H, inter, E, top_k, _code(x), w_code), dev)
    _lib.call("moe_fused_experts_from_logits", x.data_ptr(), _code(x), T, H, w13k.data_ptr(), w2k.data_ptr(), w_code,
              E, inter, lg.data_ptr(), _code(lg), top_k, sc, int(renormalize), ids.data_ptr(), wts.data_ptr(),
              _ptr(s13), _ptr(s2), y.data_ptr(), ws.data_ptr(), ws.numel(), _stream(dev))
    return y, wts, ids


@torch.library.custom_op("mail_b200::fused_experts_from_logits", mutates_args=())
def _op_from_logits(x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor, router_logits: torch.Tensor, top_k: int,
                    scoring: str, renormalize: bool, w13_scale: torch.Tensor | None,
                    w2_scale: torch.Tensor | None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    return _from_logits_impl(x, w13, w2, router_logits, top_k, scoring, renormalize, w13_scale, w2_scale)


@_op_from_logits.register_fake
def _(x, w13, w2, router_logits, top_k, scoring, renormalize, w13_scale, w2_scale):
    T, H, _, _ = _check_logits(x, w13, w2, router_logits, top_k, scoring)
    return (x.new_empty((T, H)), x.new_empty((T, top_k), dtype=torch.float32),
            x.new_empty((T, top_k), dtype=torch.int32))


def fused_moe_mlp_from_logits(x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor, router_logits: torch.Tensor,
                              top_k: int, scoring: str = "softmax", renormalize: bool = True, scales=None):
    """Routing and the top-k form of fused_moe_mlp in one call: router_logits
    [T, E] (fp32/bf16/fp16) are routed as route_topk routes them (the k
    largest logits, ties to the lower expert id, softmax or sigmoid weights,
    optionally renormalised over the k), then the layer runs on that routing.
    Returns (y [T, H] in x.dtype, topk_weights fp32 [T, k], topk_ids int32
    [T, k]). A decode-sized batch (at most 16 tokens, E <= 256, bf16/fp16)
    routes inside the one-launch decode kernel: the whole layer is one launch.
    Under torch.compile the call is one operator
    (torch.ops.mail_b200.fused_experts_from_logits).
    """
    s13, s2 = scales if scales is not None else (None, None)
    if torch.compiler.is_compiling():
        return torch.ops.mail_b200.fused_experts_from_logits(x, w13, w2, router_logits, top_k, scoring, renormalize,
                                                             s13, s2)
    return _from_logits_impl(x, w13, w2, router_logits, top_k, scoring, renormalize, s13, s2)


def fused_expert_rows(x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor, expert_ids: torch.Tensor,
                      scales=None) -> torch.Tensor:
    """out[r] = MLP_{expert_ids[r]}(x[r]) — the expert MLP row by row with no
    routing weights or combine (the local pass of expert parallelism).
    Weights as in fused_moe_mlp; rows with ids outside [0, E) are left
    unwritten (uninitialised)."""
    _require_cuda(x, w13, w2, expert_ids)
    R, H = x.shape
    E, _, two_i = w13.shape
    inter = two_i // 2
    x = x.contiguous()
    ids = expert_ids.to(torch.int32).contiguous().view(-1)
    if ids.numel() != R:
        raise ValueError("fused_expert_rows: one expert id per row")
    w13k, w2k = kmajor(w13), kmajor(w2)
    s13 = s2 = None
    if w13.dtype == torch.int8:
        if scales is None:
            raise ValueError("fused_expert_rows: int8 weights need scales")
        s13, s2 = (t.to(torch.float32).contiguous() for t in scales)
    out = torch.empty((R, H), dtype=x.dtype, device=x.device)
    ws = _workspace(_lib.query("moe_fused_expert_rows_workspace_size", R, H, inter, E, _code(x), _code(w13)),
                    x.device)
    _lib.call("moe_fused_expert_rows", x.data_ptr(), _code(x), R, H, w13k.data_ptr(), w2k.data_ptr(), _code(w13),
              E, inter, ids.data_ptr(), _ptr(s13), _ptr(s2), out.data_ptr(), ws.data_ptr(), ws.numel(),
              _stream(x.device))
    return out


class CapturedMoeMLP:
    """The top-k fused_moe_mlp for one batch shape, captured in a CUDA graph.

    At decode sizes launching the op's kernels costs about as much as running
    them; a replay launches the whole captured sequence at once. By default
    the graph reads static input buffers that each call fills by copying;
    `inputs=(x, topk_weights, topk_ids)` binds the graph to those tensors
    instead (a caller that writes them in place, e.g. the previous layer,
    then calls with the same tensors and no copy happens). Every replay
    writes the same output tensor (copy it if it must outlive the next call).
    """

    def __init__(self, w13: torch.Tensor, w2: torch.Tensor, num_tokens: int, top_k: int, dtype=torch.bfloat16,
                 scales=None, inputs=None):
        dev = w13.device
        H = w13.shape[1]
        if inputs is None:
            self.x = torch.zeros((num_tokens, H), dtype=dtype, device=dev)
            self.w = torch.zeros((num_tokens, top_k), dtype=torch.float32, device=dev)
            self.ids = torch.zeros((num_tokens, top_k), dtype=torch.int32, device=dev)
        else:
            self.x, self.w, self.ids = inputs
            if (tuple(self.x.shape) != (num_tokens, H) or self.x.dtype != dtype or not self.x.is_contiguous()
                    or tuple(self.ids.shape) != (num_tokens, top_k) or self.ids.dtype != torch.int32
                    or self.w.dtype != torch.float32 or not self.ids.is_contiguous() or not self.w.is_contiguous()):
                raise ValueError("CapturedMoeMLP: bound inputs must be contiguous x [T, H] (dtype), "
                                 "topk_weights fp32 [T, k] and topk_ids int32 [T, k]")
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):  # first call outside the capture (kernel attributes, caches)
            fused_moe_mlp(self.x, w13, w2, self.w, self.ids, scales=scales)
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        before = _lib.load().moe_launch_count()
        with torch.cuda.graph(self.graph):
            self.y = fused_moe_mlp(self.x, w13, w2, self.w, self.ids, scales=scales)
        self.kernels = int(_lib.load().moe_launch_count() - before)  # library kernels per replay

    def __call__(self, x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor) -> torch.Tensor:
        for src, dst in ((x, self.x), (topk_weights, self.w), (topk_ids, self.ids)):
            if src.data_ptr() != dst.data_ptr():
                dst.copy_(src)
        self.graph.replay()
        return self.y


def device_error(device=None) -> int:
    """Reads and clears the kernels' device error flag (synchronises)."""
    import ctypes
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    code = ctypes.c_int(0)
    _lib.call("moe_get_device_error", ctypes.addressof(code), _stream(dev))
    return code.value
