"""mail_b200 — B200-native (sm_100a) fused MoE MLP behind the reference's
fused_moe_mlp interface. Kernels live in libmoe_b200.so (C ABI:
include/moe_b200.h); this package is the thin PyTorch-facing host side."""
from ._lib import MoeError, load as load_library
from .moe import (
    BLOCK_M,
    CapturedMoeMLP,
    build_tile_schedule,
    device_error,
    fused_expert_rows,
    fused_moe_mlp,
    fused_moe_mlp_from_logits,
    gather_rows,
    kmajor,
    moe_align,
    prepack_weights,
    quant_int8_rows,
    quantize_weights_int8,
    route_topk,
    weights_from_checkpoint,
    weights_from_linear,
)

__all__ = [
    "BLOCK_M", "CapturedMoeMLP", "MoeError", "build_tile_schedule", "device_error", "fused_expert_rows", "fused_moe_mlp",
    "fused_moe_mlp_from_logits", "gather_rows", "kmajor",
    "load_library", "moe_align", "prepack_weights", "quant_int8_rows", "quantize_weights_int8", "route_topk",
    "weights_from_checkpoint", "weights_from_linear",
]
