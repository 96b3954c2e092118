"""The C-ABI library loads, exports every symbol include/moe_b200.h declares,
and validates arguments on the host (no GPU needed for any call here)."""
import ctypes
import os
import re

import numpy as np
import pytest

from mail_b200 import _lib
from oracle import moe_oracle as O

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "moe_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^MOE_API\s+[\w\s\*]+?\b(moe_\w+)\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    syms = declared_symbols()
    assert len(syms) >= 19
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_lib.SIGNATURES), "ctypes signature table out of sync with the header"


def test_version_and_pure_host_queries():
    lib = _lib.load()
    assert lib.moe_version() >= 100
    assert lib.moe_tile_grid(120, 4, 128) == 1 + 4
    assert lib.moe_tile_grid(0, 4, 128) == 4
    assert lib.moe_align_capacity(8192, 8, 128) == 9216  # 8192 + 8 * 127, whole tiles
    assert lib.moe_align_capacity(8, 128, 128) == 1024    # decode: at most 8 experts hold a slot
    assert lib.moe_align_capacity(0, 128, 128) == 0
    assert lib.moe_tile_table_ints(8, 100) == 4 + 9 + 200
    assert lib.moe_fused_experts_workspace_size(4096, 4096, 14336, 8, 2, _lib.BF16, _lib.BF16) > 0
    assert lib.moe_fused_mlp_workspace_size(120, 256, 512, 4, _lib.F16, 64) == 0  # block_m must be 128


@pytest.mark.parametrize("call,needle", [
    (lambda L: L.moe_gemm1_swiglu(None, 99, 1, 64, None, 1, 64, None, None, None, 1, None, _lib.BF16, None),
     "unsupported dtype"),
    (lambda L: L.moe_gemm1_swiglu(None, _lib.BF16, 1, 12, None, 1, 64, None, None, None, 1, None, _lib.BF16, None),
     "multiple of 16 bytes"),
    (lambda L: L.moe_gemm2(None, _lib.BF16, 1, 64, None, 1, 64, None, None, ctypes.c_void_p(16), 1, 0, None, None,
                           1, None, _lib.BF16, 1, None), "NULL pointer"),
    (lambda L: L.moe_gemm2(None, _lib.BF16, 1, 64, None, 1, 64, None, None, ctypes.c_void_p(16), 1, 7, None, None,
                           1, ctypes.c_void_p(16), _lib.BF16, 1, None), "bad epilogue"),
    (lambda L: L.moe_align(None, 4, 2, 0, 128, None, None, None, None, None, None, 0, None), "num_experts"),
    (lambda L: L.moe_tile_schedule(None, _lib.I64, 4, 10, 128, None, None, None, None, None), "NULL"),
    (lambda L: L.moe_fused_mlp(None, _lib.I8, 10, 64, None, None, 2, 64, None, _lib.I64, 128, None, None, 0, None),
     "dtype"),
    (lambda L: L.moe_fused_experts(None, _lib.BF16, 4, 64, None, None, _lib.F16, 2, 64, None, None, 2, None, None,
                                   None, None, 0, None), "int8"),
    (lambda L: L.moe_fused_experts_from_logits(None, _lib.BF16, 4, 64, None, None, _lib.BF16, 8, 64, None, _lib.I8, 2,
                                               0, 1, None, None, None, None, ctypes.c_void_p(16), None, 0, None),
     "logits dtype"),
    (lambda L: L.moe_fused_experts_from_logits(None, _lib.BF16, 4, 64, None, None, _lib.BF16, 8, 64, None, _lib.F32,
                                               2, 5, 1, None, None, None, None, ctypes.c_void_p(16), None, 0, None),
     "bad scoring"),
    (lambda L: L.moe_fused_experts_from_logits(None, _lib.BF16, 4, 64, None, None, _lib.BF16, 8, 64, None, _lib.F32,
                                               2, 0, 1, None, None, None, None, ctypes.c_void_p(16), None, 0, None),
     "NULL pointer"),
])
def test_invalid_arguments_are_rejected_on_host(call, needle):
    lib = _lib.load()
    rc = call(lib)
    assert rc == 1, rc  # MOE_ERR_INVALID_ARG
    assert needle in lib.moe_last_error().decode()


def test_options_round_trip_and_reject_bad_values():
    """Every documented option reads back what was set; bad values and
    unknown options are rejected on the host."""
    lib = _lib.load()
    opts = {_lib.OPT_GEMM_CTA_PAIR: (0, 2), _lib.OPT_GEMM_BAND: (8, 16), _lib.OPT_GEMM_STREAM_K: (1, 0),
            _lib.OPT_GEMM_HALF_UNITS: (0, 1), _lib.OPT_PDL: (0, 1)}
    for opt, (val, default) in opts.items():
        assert lib.moe_get_option(opt) == default, opt
        assert lib.moe_set_option(opt, val) == 0
        assert lib.moe_get_option(opt) == val
        assert lib.moe_set_option(opt, default) == 0
    assert lib.moe_set_option(_lib.OPT_GEMM_CTA_PAIR, 3) == 1
    assert lib.moe_set_option(_lib.OPT_GEMM_BAND, 0) == 1
    assert lib.moe_set_option(99, 1) == 1 and "unknown option" in lib.moe_last_error().decode()
    assert lib.moe_get_option(99) == -1


def test_empty_batch_is_a_no_op():
    """Zero tokens: both fused entry points return OK without touching any
    buffer (all NULL here) and without launching work."""
    lib = _lib.load()
    before = lib.moe_launch_count()
    assert lib.moe_fused_experts(None, _lib.BF16, 0, 64, None, None, _lib.BF16, 4, 64, None, None, 2, None, None,
                                 None, None, 0, None) == 0
    assert lib.moe_fused_mlp(None, _lib.BF16, 0, 64, None, None, 4, 64, None, _lib.I64, 128, None, None, 0,
                             None) == 0
    assert lib.moe_launch_count() == before


def test_python_wrapper_raises_without_cuda_tensors():
    torch = pytest.importorskip("torch")
    import mail_b200
    x = torch.zeros(4, 8)
    with pytest.raises(ValueError, match="CUDA"):
        mail_b200.fused_moe_mlp(x, torch.zeros(2, 8, 16), torch.zeros(2, 8, 8), torch.tensor([2, 2]))


@pytest.mark.parametrize("T,E,k,routing", [(1, 128, 8, "zipf1.2"), (3, 256, 8, "sigmoid"), (4096, 8, 2, "uniform-softmax"),
                                           (300, 16, 4, "hot25-zipf1.0")])
def test_align_capacity_bounds_padded_rows(T, E, k, routing):
    """The capacity covers the padded rows of any routing (oracle align)."""
    ids, _ = O.synthetic_routing(routing, T, E, k, seed=T)
    cap = _lib.load().moe_align_capacity(T * k, E, 128)
    assert int(O.align(ids, E, 128)["padded_offsets"][-1]) <= cap
    # worst case: every slot on its own expert
    worst = np.arange(T * k, dtype=np.int32).reshape(T, k) % E
    assert int(O.align(worst, E, 128)["padded_offsets"][-1]) <= cap
