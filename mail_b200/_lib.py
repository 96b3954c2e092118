"""ctypes binding of libmoe_b200.so (the C ABI declared in include/moe_b200.h).

The library is loaded from this package directory. There is no fallback: if
the shared object is missing or fails to load, every op raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmoe_b200.so")

# dtype / status / epilogue codes (moe_b200.h)
F32, F16, BF16, I8, I32, I64 = 0, 1, 2, 3, 4, 5
EPI_STORE_ROWS, EPI_COMBINE_ADD, EPI_SCATTER_ROWS = 0, 1, 2
OPT_GEMM_CTA_PAIR, OPT_GEMM_BAND, OPT_GEMM_STREAM_K, OPT_GEMM_HALF_UNITS, OPT_PDL, OPT_KERNEL_CLOCKS = 1, 2, 3, 4, 5, 6
OPT_GEMM_SWAP_AB, OPT_GEMM_BAND_DOWN, OPT_DECODE_FUSED = 7, 8, 9
CLOCK_GATE_UP, CLOCK_DOWN, NUM_CLOCKS = 0, 1, 2
STATUS = {0: "MOE_OK", 1: "MOE_ERR_INVALID_ARG", 2: "MOE_ERR_UNSUPPORTED", 3: "MOE_ERR_CUDA",
          4: "MOE_ERR_WORKSPACE", 5: "MOE_ERR_DEVICE"}

_p = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_sz = ctypes.c_size_t

# name -> (restype, argtypes)
SIGNATURES = {
    "moe_version": (_i, []),
    "moe_last_error": (ctypes.c_char_p, []),
    "moe_get_device_error": (_i, [_p, _p]),
    "moe_launch_count": (_i64, []),
    "moe_kernel_clocks": (_i, [_p, _p, _i, _i, _p]),
    "moe_selftest_wait_timeout": (_i, [ctypes.c_uint64, _p]),
    "moe_set_option": (_i, [_i, _i]),
    "moe_get_option": (_i, [_i]),
    "moe_set_stage_events": (_i, [_p, _i]),
    "moe_tile_grid": (_i64, [_i64, _i, _i]),
    "moe_tile_table_ints": (_i64, [_i, _i64]),
    "moe_tile_schedule": (_i, [_p, _i, _i, _i64, _i, _p, _p, _p, _p, _p]),
    "moe_route_topk": (_i, [_p, _i, _i64, _i, _i, _i, _i, _p, _p, _p]),
    "moe_align_capacity": (_i64, [_i64, _i, _i]),
    "moe_align_workspace_size": (_sz, [_i64, _i, _i, _i]),
    "moe_align": (_i, [_p, _i64, _i, _i, _i, _p, _p, _p, _p, _p, _p, _sz, _p]),
    "moe_align_static": (_i, [_p, _i64, _i, _i, _i, _p, _p, _p, _p, _p, _p]),
    "moe_gather_rows": (_i, [_p, _i, _i64, _p, _i, _i64, _p, _p, _i, _p, _p]),
    "moe_quant_rows": (_i, [_p, _i, _i64, _i64, _p, _p, _p, _p]),
    "moe_gemm1_swiglu": (_i, [_p, _i, _i64, _i64, _p, _i, _i64, _p, _p, _p, _i64, _p, _i, _p]),
    "moe_gemm2": (_i, [_p, _i, _i64, _i64, _p, _i, _i64, _p, _p, _p, _i64, _i, _p, _p, _i, _p, _i, _i64, _p]),
    "moe_combine_rows": (_i, [_p, _i, _i64, _p, _p, _i64, _i, _p, _i, _p]),
    "moe_convert_f32": (_i, [_p, _i64, _p, _i, _p]),
    "moe_fused_mlp_workspace_size": (_sz, [_i64, _i64, _i64, _i, _i, _i]),
    "moe_fused_mlp": (_i, [_p, _i, _i64, _i64, _p, _p, _i, _i64, _p, _i, _i, _p, _p, _sz, _p]),
    "moe_fused_experts_workspace_size": (_sz, [_i64, _i64, _i64, _i, _i, _i, _i]),
    "moe_fused_experts": (_i, [_p, _i, _i64, _i64, _p, _p, _i, _i, _i64, _p, _p, _i, _p, _p, _p, _p, _sz, _p]),
    "moe_fused_experts_from_logits": (_i, [_p, _i, _i64, _i64, _p, _p, _i, _i, _i64, _p, _i, _i, _i, _i, _p, _p, _p,
                                           _p, _p, _p, _sz, _p]),
    "moe_ipc_malloc": (_i, [_sz, _p, _p]),
    "moe_ipc_open": (_i, [_p, _p]),
    "moe_ipc_close": (_i, [_p]),
    "moe_ipc_free": (_i, [_p]),
    "moe_ep_plan": (_i, [_p, _i, _i, _i, _p, _i64, _p, _p, _i64, _p, _i64, _p, _p]),
    "moe_ep_dispatch": (_i, [_p, _i, _i64, _i, _p, _p, _p, _p, _p, _i64, _i, _i, _i, _i64, _p, _i, _p, _p, _p,
                             _p]),
    "moe_ep_expert_pass_workspace_size": (_sz, [_i64, _i64, _i]),
    "moe_ep_expert_pass": (_i, [_p, _i, _p, _i64, _i64, _p, _p, _i, _i64, _p, _p, _p, _p, _p, _i, _i64, _i, _p,
                                _sz, _p]),
    "moe_fused_expert_rows_workspace_size": (_sz, [_i64, _i64, _i64, _i, _i, _i]),
    "moe_fused_expert_rows": (_i, [_p, _i, _i64, _i64, _p, _p, _i, _i, _i64, _p, _p, _p, _p, _p, _sz, _p]),
}

_lib = None
_lock = threading.Lock()


class MoeError(RuntimeError):
    """A libmoe_b200 call returned a non-zero status."""


def load() -> ctypes.CDLL:
    """Loads (once) and returns the library; raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise MoeError(f"{LIB_PATH} is missing: build it with `python -m mail_b200.build` "
                               "(there is no CPU fallback)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def call(name: str, *args) -> None:
    """Calls an int-returning entry point and raises MoeError on failure."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        msg = lib.moe_last_error().decode(errors="replace")
        raise MoeError(f"{name} failed with {STATUS.get(rc, rc)}: {msg}")


def query(name: str, *args):
    return getattr(load(), name)(*args)
