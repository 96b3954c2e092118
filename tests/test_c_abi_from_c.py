"""The public header is plain C99 and a C program links and calls the library
(what a cgo / JNI / N-API binding sees). Host-only calls: no GPU needed."""
import os
import shutil
import subprocess

import pytest

from mail_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

C_SOURCE = r"""
#include <stdio.h>
#include "moe_b200.h"
int main(void) {
  if (moe_version() < 100) return 1;
  if (moe_align_capacity(8192, 8, 128) != 9216) return 2;
  if (moe_tile_grid(120, 4, 128) != 5) return 3;
  /* an empty batch is a no-op, NULL buffers included */
  if (moe_fused_experts(NULL, MOE_BF16, 0, 64, NULL, NULL, MOE_BF16, 4, 64, NULL, NULL, 2, NULL, NULL, NULL,
                        NULL, 0, NULL) != MOE_OK) return 4;
  /* bad arguments come back as a status code with a message */
  if (moe_gemm1_swiglu(NULL, 99, 1, 64, NULL, 1, 64, NULL, NULL, NULL, 1, NULL, MOE_BF16, NULL) !=
      MOE_ERR_INVALID_ARG) return 5;
  printf("%s\n", moe_last_error());
  return 0;
}
"""


def test_header_is_c99_and_links(tmp_path):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lib = _lib.load()  # builds nothing; fails loudly if the library is missing
    del lib
    src = tmp_path / "abi.c"
    src.write_text(C_SOURCE)
    exe = tmp_path / "abi"
    libdir = os.path.dirname(_lib.LIB_PATH)
    subprocess.run([cc, "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I", os.path.join(ROOT, "include"),
                    str(src), "-L", libdir, "-lmoe_b200", f"-Wl,-rpath,{libdir}", "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, (out.returncode, out.stdout, out.stderr)
    assert "unsupported dtype 99" in out.stdout
