"""The C ABI from plain C: include/bloth_b200.h compiles as C99 with warnings
as errors, and a C program links against libbloth_b200.so and gets the
argument checks' status codes back (they run before any CUDA call, so this
needs no GPU). This is the boundary a non-Python host (cgo, JNI, a C++
runtime) binds."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_DIR = os.path.join(ROOT, "bloth_b200")

PROGRAM = r"""
#include <stdio.h>
#include "bloth_b200.h"

int main(void) {
  int bad = 0;
  /* rows wider than 65536 elements: BLOTH_ERR_SHAPE */
  int rc = bloth_rmsnorm_fwd(NULL, 0, NULL, 0.0f, NULL, 0, NULL, 1, 70000, 1e-6f, BLOTH_BF16,
                             BLOTH_BF16, NULL);
  bad |= rc != BLOTH_ERR_SHAPE;
  /* an unknown dtype code: BLOTH_ERR_DTYPE */
  rc = bloth_rmsnorm_fwd(NULL, 0, NULL, 0.0f, NULL, 0, NULL, 1, 64, 1e-6f, 7, BLOTH_BF16, NULL);
  bad |= rc != BLOTH_ERR_DTYPE;
  /* no rows: nothing to do */
  rc = bloth_rmsnorm_fwd(NULL, 0, NULL, 0.0f, NULL, 0, NULL, 0, 64, 1e-6f, BLOTH_BF16,
                         BLOTH_BF16, NULL);
  bad |= rc != BLOTH_OK;
  printf("version %d\n%s\n", bloth_version(), bloth_strerror(BLOTH_ERR_ALIGN));
  printf("%s\n", bad ? "FAIL" : "OK");
  return bad;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_header_is_c99_and_links_from_c(tmp_path):
    lib = os.path.join(LIB_DIR, "libbloth_b200.so")
    if not os.path.exists(lib):
        pytest.skip("library not built")
    src = tmp_path / "abi.c"
    src.write_text(PROGRAM)
    exe = tmp_path / "abi"
    cmd = ["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic",
           "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe),
           "-L", LIB_DIR, "-lbloth_b200", "-Wl,-rpath," + LIB_DIR]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, run.stdout + run.stderr
    lines = run.stdout.splitlines()
    assert lines[-1] == "OK"
    assert lines[0].startswith("version ")
    assert "aligned" in lines[1]
