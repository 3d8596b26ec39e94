"""The C ABI from plain C, as a foreign caller (cgo, JNI, a C engine) binds it:
include/b200moe.h compiles as strict C99, and a C program linked against
libb200moe.so calls host-only entry points (no GPU needed)."""

import os
import shutil
import subprocess

import pytest

from tests.conftest import ROOT

LIBDIR = ROOT / "moe_serving_profile_b200"

PROGRAM = r"""
#include <stdio.h>
#include "b200moe.h"

int main(void) {
  size_t bytes = 0;
  int rc = b200moe_permute_workspace(4096, 8, 128, &bytes);
  printf("%s|%d|%zu|%d\n", b200moe_version(), rc, bytes, b200moe_permute_workspace(-1, 8, 128, &bytes));
  return rc == B200MOE_OK ? 0 : 1;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_header_is_c99_and_the_library_links_from_c(tmp_path):
    src = tmp_path / "caller.c"
    src.write_text(PROGRAM)
    exe = tmp_path / "caller"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I", str(ROOT / "include"),
                    str(src), "-L", str(LIBDIR), "-lb200moe", "-o", str(exe)], check=True)
    env = dict(os.environ, LD_LIBRARY_PATH=f"{LIBDIR}:{os.environ.get('LD_LIBRARY_PATH', '')}")
    out = subprocess.run([str(exe)], env=env, capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stderr
    version, rc, nbytes, bad = out.stdout.strip().split("|")
    assert version.startswith("b200moe") and int(rc) == 0
    assert int(nbytes) == 32 * 128 * 4             # per-chunk histograms of 32 chunks
    assert int(bad) == 1                            # B200MOE_ERR_INVALID
