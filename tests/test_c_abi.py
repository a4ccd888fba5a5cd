"""The C ABI from a C host: ``include/tj.h`` compiles as C99 with warnings as
errors, a small C program links against ``libtj.so`` and its argument checks
answer without a GPU (null pointers, unsupported head_dim, bad workspace
queries) with a status code and a message, as a C/C++ host would see them."""

import re
import shutil
import subprocess
from pathlib import Path

import pytest

from techjam_b200 import _lib, build

ROOT = Path(__file__).resolve().parent.parent

C_HOST = r"""
#include <stdio.h>
#include <string.h>
#include "tj.h"

static int expect(int got, int want, const char* what) {
  if (got != want) { printf("FAIL %s: status %d, expected %d\n", what, got, want); return 1; }
  if (want != TJ_OK && strlen(tj_last_error()) == 0) { printf("FAIL %s: no message\n", what); return 1; }
  return 0;
}

int main(void) {
  int bad = 0;
  TjModel* m = NULL;
  size_t bytes = 0;
  TjConfig cfg = {1000, 16, 4096, 1, 1, 1e-5f};  /* head_dim 62.5: not an integer */
  if (tj_version() < 1) { printf("FAIL version\n"); bad = 1; }
  bad |= expect(tj_model_create(NULL, &m), TJ_ERR_INVALID, "create(NULL)");
  bad |= tj_model_create(&cfg, &m) == TJ_OK;  /* must refuse before touching a device */
  bad |= expect(tj_workspace_bytes(NULL, 1, 1, TJ_ROUTE_EXACT, &bytes), TJ_ERR_INVALID, "workspace(NULL)");
  bad |= expect(tj_model_destroy(NULL), TJ_OK, "destroy(NULL)");
  printf("%s\n", bad ? "c-host FAILED" : "c-host ok");
  return bad;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_header_compiles_as_c_and_links(tmp_path):
    build.build()
    src = tmp_path / "host.c"
    src.write_text(C_HOST)
    exe = tmp_path / "host"
    lib_dir = _lib.LIB_PATH.parent
    cmd = ["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-I", str(ROOT / "include"), str(src),
           "-L", str(lib_dir), "-l:libtj.so", f"-Wl,-rpath,{lib_dir}", "-o", str(exe)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "c-host ok" in run.stdout


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_header_compiles_as_cxx(tmp_path):
    src = tmp_path / "host.cpp"
    src.write_text('#include "tj.h"\nint main() { return tj_version() > 0 ? 0 : 1; }\n')
    res = subprocess.run(["g++", "-std=c++17", "-Wall", "-Werror", "-fsyntax-only", "-I", str(ROOT / "include"),
                          str(src)], capture_output=True, text=True)
    assert res.returncode == 0, res.stderr


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_integration_example_compiles(tmp_path):
    """The C host example of the integration guide compiles against tj.h as written."""
    text = (ROOT / "INTEGRATION.md").read_text()
    blocks = re.findall(r"```c\n(.*?)```", text, flags=re.S)
    assert blocks, "no C example in the integration guide"
    src = tmp_path / "example.c"
    src.write_text(blocks[0])
    res = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-fsyntax-only", "-I",
                          str(ROOT / "include"), str(src)], capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
