"""The boundary from C: a plain C11 program compiled with gcc against include/kf_moe.h links
libkf_moe.so and calls its host-side entry points (no GPU needed).  This is the binding a
non-Python host (cgo, JNI, N-API, a C++ server) would make."""
import os
import shutil
import subprocess

import pytest

from kernelforge_b200 import binding as B

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

C_SRC = r"""
#include <stdio.h>
#include <string.h>
#include "kf_moe.h"

int main(void) {
  /* sizes are host-only queries */
  printf("%zu %zu %zu\n", kf_moe_workspace_bytes(16, 32), kf_moe_workspace_bytes(4096, 256),
         kf_moe_workspace_bytes(KF_MOE_MAX_TOKENS + 1, 32));
  printf("%d %d\n", kf_ep_max_send_rows(100, 8), (int)kf_ep_workspace_bytes(100, 3));
  /* argument errors are reported before any device work */
  int rc = kf_moe_forward(NULL, NULL, NULL, NULL, NULL, NULL, NULL, NULL, 4, 0, 0, 2.5f, NULL, NULL, 0, NULL);
  printf("%d %s\n", rc, kf_moe_error_string(rc));
  rc = kf_moe_forward(NULL, NULL, NULL, NULL, NULL, NULL, NULL, NULL, 0, 32, 0, 2.5f, NULL, NULL, 0, NULL);
  printf("%d %d\n", rc, kf_moe_launches_per_forward());
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_c_program_links_and_calls_the_library(tmp_path):
    lib = B.library()   # builds libkf_moe.so if needed
    libdir = os.path.join(ROOT, "kernelforge_b200")
    src = tmp_path / "caller.c"
    src.write_text(C_SRC)
    exe = tmp_path / "caller"
    cc = ["gcc", "-std=c11", "-Wall", "-Werror", "-pedantic", f"-I{os.path.join(ROOT, 'include')}", str(src),
          "-o", str(exe), f"-L{libdir}", "-l:libkf_moe.so", f"-Wl,-rpath,{libdir}"]
    r = subprocess.run(cc, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    env = dict(os.environ)
    env["LD_LIBRARY_PATH"] = os.pathsep.join(filter(None, ["/usr/local/cuda/lib64", env.get("LD_LIBRARY_PATH")]))
    r = subprocess.run([str(exe)], capture_output=True, text=True, env=env, timeout=60)
    assert r.returncode == 0, r.stderr
    lines = r.stdout.split("\n")
    ws16, ws4096, ws_over = (int(x) for x in lines[0].split())
    assert ws16 == lib.kf_moe_workspace_bytes(16, 32) and ws4096 == lib.kf_moe_workspace_bytes(4096, 256)
    assert ws_over == 0
    assert lines[1].split() == ["800", "0"]          # 100 tokens x 8 ranks; 3 ranks do not divide 256
    assert lines[2] == "1 invalid argument"
    assert lines[3].split() == ["0", "7"]
