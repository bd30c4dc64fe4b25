"""include/fa_b200.h is plain C: a C99 program that includes it compiles
with gcc, links against libfa_b200.so and calls the host-only entry points
(no GPU needed). This is the binding a C, cgo or other FFI host makes."""

import os
import shutil
import subprocess

import pytest

from conftest import PKG_DIR, REPO

LIB_DIR = os.path.join(PKG_DIR, "flashattn_cuda")

C_SOURCE = r"""
#include <stdio.h>
#include <string.h>
#include "fa_b200.h"

int main(void) {
  int chunks = 0;
  size_t ws = 0;
  int rc = fa_prefill_host_plan(4, 14, 14, 4096, 64, &chunks, &ws);
  printf("plan %d %d %zu\n", rc, chunks, ws);
  printf("split %d\n", fa_choose_decode_split(131072, 1, 14, 296));
  printf("status %s\n", fa_status_string(FA_EINVAL));
  /* argument errors are reported before any device work */
  printf("bad %d %d\n",
         fa_prefill_ex(0, 0, 0, 0, 1, 2, 2, 16, 64, 7, 1, 0.1f, 0),
         fa_decode_ex(0, 0, 0, 0, 0, 1, 2, 2, 8, 96, FA_DTYPE_BF16, 0.1f, 0,
                      0, 0, 0, 0));
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_header_compiles_as_c99_and_links(tmp_path):
    src = tmp_path / "host.c"
    src.write_text(C_SOURCE)
    exe = tmp_path / "host"
    subprocess.run(
        ["gcc", "-std=c99", "-Wall", "-Werror", "-pedantic",
         "-I", os.path.join(REPO, "include"), str(src), "-o", str(exe),
         "-L", LIB_DIR, "-lfa_b200", "-Wl,-rpath," + LIB_DIR],
        check=True, capture_output=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True,
                         text=True).stdout.split("\n")
    assert out[0] == "plan 0 5 %d" % (3 * 14 * 4 * (512 << 10))
    assert out[1] == "split 1024"
    assert out[2].startswith("status ")
    assert out[3] == "bad 1 1"
