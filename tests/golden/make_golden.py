"""Generates the golden fixtures in this directory from the reference itself.

Run in a container where the CrDem/mail sources are mounted (default
/root/reference, override with MOE_REFERENCE_DIR):

    python tests/golden/make_golden.py

It imports the reference's Python files by path (their sibling imports are
broken as shipped, so a stub module stands in for the missing
`fused_moe_mlp`), runs on the CPU:
  * build_tile_schedule            fused_moe_mlp_triton.py:91-119 (static grid)
  * build_tile_schedule            fixed_kernel.py:126-163 (exact grid)
  * reference_moe_mlp              fixed_kernel.py:232-249 ((E,K,N) layout)
  * reference_moe_mlp              fused moe mlp triton.py:189-205 (nn.Linear layout)
  * golden_moe_mlp_loop            independent_test.py:50-90
  * _golden_moe_mlp_vectorized...  independent_test.py:93-124
  * fused_moe_mlp (Triton kernels under TRITON_INTERPRET=1)
                                   partially_fused_moe_mlp_triton.py:165-218
and stores inputs and outputs as .npz. Inputs come from numpy's PCG64 with
fixed seeds and are stored in the fixtures, so tests never regenerate them.
"""
from __future__ import annotations

import importlib.util
import os
import sys
import types

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

REF = os.environ.get("MOE_REFERENCE_DIR", "/root/reference")
OUT = os.path.dirname(os.path.abspath(__file__))


def load(name: str, filename: str):
    spec = importlib.util.spec_from_file_location(name, os.path.join(REF, filename))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def reference_modules():
    stub = types.ModuleType("fused_moe_mlp")
    stub.fused_moe_mlp = None  # independent_test.py:47 imports a module that does not exist
    sys.modules.setdefault("fused_moe_mlp", stub)
    return dict(
        canonical=load("ref_fused_moe_mlp_triton", "fused_moe_mlp_triton.py"),
        fixed=load("ref_fixed_kernel", "fixed_kernel.py"),
        linear=load("ref_fused_moe_mlp_linear", "fused moe mlp triton.py"),
        arbiter=load("ref_independent_test", "independent_test.py"),
        partial=load("ref_partially_fused", "partially_fused_moe_mlp_triton.py"),
    )


# group-size fixtures quoted from the reference's own tests/benches
GS_SELFTEST = [37, 12, 50, 21]                      # fixed_kernel.py:257
GS_SELFCHECK = [7, 0, 13, 4, 9]                     # independent_test.py:138
GS_128 = [                                          # independent_test.py:255-264
    13, 14, 20, 13, 10, 6, 20, 14, 29, 5, 3, 2, 2, 11, 10, 16,
    60, 18, 9, 12, 14, 16, 15, 15, 11, 13, 20, 13, 22, 6, 6, 21,
    10, 29, 13, 23, 22, 11, 9, 26, 2, 13, 4, 27, 9, 25, 5, 6,
    41, 26, 5, 39, 1, 34, 24, 6, 8, 34, 14, 7, 42, 16, 15, 45,
    8, 23, 11, 15, 7, 15, 10, 6, 14, 4, 14, 30, 34, 4, 8, 10,
    10, 11, 18, 14, 28, 37, 11, 5, 14, 31, 8, 8, 5, 4, 5, 21,
    28, 15, 7, 23, 15, 6, 70, 23, 23, 6, 1, 22, 11, 12, 38, 12,
    8, 14, 11, 15, 18, 14, 12, 4, 3, 11, 2, 37, 14, 21, 41, 18,
]
GS_EDGES = [                                        # kernel_bench.py:154-198
    0, 0, 1, 2, 3, 4, 5, 7, 8, 31, 32, 33, 63, 64, 65, 127, 128, 129, 130, 131, 150,
    255, 256, 257, 383, 384, 385, 511, 512, 513, 777, 1000, 0, 0, 17, 9, 41, 6, 11,
    126, 127, 128, 129, 130, 1023, 1024, 1025, 13, 27, 2, 19, 0, 8,
]
GS_EXTRA = {"all_zero": [0, 0, 0, 0], "single": [300], "leading_zero": [0, 0, 129, 0, 1]}


def gen_schedules(ref):
    out = {}
    cases = {"selftest": GS_SELFTEST, "selfcheck": GS_SELFCHECK, "gs128": GS_128, "edges": GS_EDGES}
    cases.update(GS_EXTRA)
    for name, gs in cases.items():
        out[f"{name}/group_sizes"] = np.asarray(gs, np.int64)
        for bm in (16, 32, 64, 128, 256):
            g = torch.tensor(gs, dtype=torch.int64)
            T = int(g.sum())
            e, s, c, grid = ref["canonical"].build_tile_schedule(g, T, bm)
            out[f"{name}/bm{bm}/expert"] = e.numpy()
            out[f"{name}/bm{bm}/row_start"] = s.numpy()
            out[f"{name}/bm{bm}/row_count"] = c.numpy()
            out[f"{name}/bm{bm}/grid"] = np.asarray(grid, np.int64)
            e2, s2, c2, grid2 = ref["fixed"].build_tile_schedule(g, T, bm)
            out[f"{name}/bm{bm}/exact_expert"] = e2.numpy()
            out[f"{name}/bm{bm}/exact_row_start"] = s2.numpy()
            out[f"{name}/bm{bm}/exact_row_count"] = c2.numpy()
            out[f"{name}/bm{bm}/exact_grid"] = np.asarray(grid2, np.int64)
    np.savez_compressed(os.path.join(OUT, "tile_schedule.npz"), **out)


def mlp_case(ref, name, E, H, I, gs, dtype, x_scale, w_scale, seed, triton_check=True):
    rng = np.random.default_rng(seed)
    T = int(sum(gs))
    np_dt = np.float16 if dtype == torch.float16 else np.float32
    x = (rng.standard_normal((T, H), dtype=np.float32) * x_scale).astype(np_dt)
    w13 = (rng.standard_normal((E, H, 2 * I), dtype=np.float32) * w_scale).astype(np_dt)
    w2 = (rng.standard_normal((E, I, H), dtype=np.float32) * w_scale).astype(np_dt)
    gs_t = torch.tensor(gs, dtype=torch.int64)
    xt, w13t, w2t = torch.from_numpy(x), torch.from_numpy(w13), torch.from_numpy(w2)
    res = dict(x=x, w13=w13, w2=w2, group_sizes=np.asarray(gs, np.int64))
    res["ref_fixed_kernel"] = ref["fixed"].reference_moe_mlp(xt, w13t, w2t, gs_t).float().numpy()
    res["ref_golden_loop"] = ref["arbiter"].golden_moe_mlp_loop(xt, w13t, w2t, gs_t).float().numpy()
    res["ref_golden_vectorized"] = (
        ref["arbiter"]._golden_moe_mlp_vectorized_for_selfcheck(xt, w13t, w2t, gs_t).float().numpy())
    # nn.Linear layout restatement of the same op (fused moe mlp triton.py:189-205)
    lin = ref["linear"].reference_moe_mlp(xt, w13t.transpose(1, 2).contiguous(), w2t.transpose(1, 2).contiguous(), gs_t)
    res["ref_linear_layout"] = lin.float().numpy()
    if triton_check:
        # reference Triton kernels run by the Triton interpreter on the CPU;
        # h is rounded to the weight dtype inside (partially_fused...:111)
        out = ref["partial"].fused_moe_mlp(xt, w13t, w2t, gs_t, BLOCK_M=16, BLOCK_N=16, BLOCK_K=16)
        res["ref_triton_interpreted"] = out.float().numpy()
    np.savez_compressed(os.path.join(OUT, f"{name}.npz"), **res)
    return res


def main():
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    ref = reference_modules()
    gen_schedules(ref)
    # independent_test.py:127-155 self-check shape (empty expert), fp32
    mlp_case(ref, "mlp_selfcheck_f32", 5, 32, 16, GS_SELFCHECK, torch.float32, 1.0, 1.0, 1234)
    # fixed_kernel.py:252-273 self-test group sizes and scaling, fp16, H/I reduced
    mlp_case(ref, "mlp_selftest_f16", 4, 128, 256, GS_SELFTEST, torch.float16, 0.1, 0.05, 0)
    # ragged groups incl. empty experts, I not a multiple of 128, fp32
    mlp_case(ref, "mlp_ragged_f32", 6, 64, 96, [0, 45, 130, 0, 1, 64], torch.float32, 1.0, 0.05, 7)
    print("fixtures written to", OUT)


if __name__ == "__main__":
    main()
