"""A plain C program can use include/rnb_moe.h and librnb_moe.so as they ship.

The boundary is a C ABI, so a C caller (or a cgo / JNI / N-API binding that
mirrors the header) must be able to compile the header as strict C11, link the
library and get the same struct layout as the Python binding.  The program
built here prints the size and every field offset of rnb_moe_desc, then makes
two host-side calls that need no GPU: rnb_version, and rnb_moe_workspace_size
with an unsupported bit width, whose error code and message must come back."""
import ctypes
import os
import re
import shutil
import subprocess

import pytest

from runnel_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "runnel_b200")


def _fields():
    text = open(os.path.join(ROOT, "include", "rnb_moe.h")).read()
    body = text[text.index("typedef struct rnb_moe_desc"):text.index("} rnb_moe_desc;")]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    return re.findall(r"\b(\w+)\s*;", body)


SOURCE = r"""
#include <stddef.h>
#include <stdio.h>
#include <string.h>
#include "rnb_moe.h"

int main(void) {
  printf("version %d\n", rnb_version());
  printf("size %zu\n", sizeof(rnb_moe_desc));
@OFFSETS@
  rnb_moe_desc d;
  memset(&d, 0, sizeof d);
  d.T = 1; d.H = 2048; d.I = 512; d.E = 256; d.E_total = 256; d.k = 8; d.bits = 3; d.group = 64;
  size_t n = 0;
  const int rc = rnb_moe_workspace_size(&d, &n);
  printf("rc %d\n", rc);
  printf("msg %s\n", rnb_last_error());
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_strict_c11_program_links_and_matches_the_binding(tmp_path):
    lib = _lib.load()  # builds nothing; the library must exist
    assert lib is not None
    fields = _fields()
    assert "router_bits" in fields and "sgate_b" in fields
    offsets = "\n".join(f'  printf("off {f} %zu\\n", offsetof(rnb_moe_desc, {f}));' for f in fields)
    src = tmp_path / "consumer.c"
    src.write_text(SOURCE.replace("@OFFSETS@", offsets))
    exe = tmp_path / "consumer"
    cc = subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-pedantic", "-I",
                         os.path.join(ROOT, "include"), str(src), "-o", str(exe), "-L", PKG, "-lrnb_moe",
                         f"-Wl,-rpath,{PKG}"], capture_output=True, text=True, timeout=300)
    assert cc.returncode == 0, cc.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stderr
    out = dict(line.split(" ", 1) for line in run.stdout.splitlines() if not line.startswith("off "))
    offs = {line.split()[1]: int(line.split()[2]) for line in run.stdout.splitlines() if line.startswith("off ")}
    assert int(out["version"]) == lib.rnb_version()
    assert int(out["size"]) == ctypes.sizeof(_lib.RnbMoeDesc)
    for name in fields:
        assert offs[name] == getattr(_lib.RnbMoeDesc, name).offset, name
    assert int(out["rc"]) == -1  # RNB_ERR_INVALID
    assert "bits" in out["msg"]
