"""Build the sm_100a shared library ``kernelforge_b200/libkf_moe.so`` with nvcc.

    python -m kernelforge_b200.build [--force]

Cross-compiles without a GPU.  The GEMM kernels split registers between warp
groups with ``setmaxnreg`` (48 for the producer/MMA group, 224 for the two
epilogue groups), which is only valid when the kernel is launched with 168
registers per thread; the build checks ptxas's report and fails otherwise.
"""
from __future__ import annotations

import os
import re
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libkf_moe.so")
SOURCES = ["kf_route_permute.cu", "kf_grouped_gemm.cu", "kf_grouped_gemm_pair.cu", "kf_moe_api.cu",
           "kf_moe_noalloc.cu", "kf_ep.cu", "kf_quant.cu"]
HEADERS = ["kf_ptx.cuh", "kf_internal.cuh", "kf_quant.cuh", "kf_fp8.cuh"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xptxas", "-v", f"-I{INCLUDE}"]
SETMAXNREG_KERNELS = ("gemm1_swiglu_kernel", "gemm2_weighted_kernel", "gemm1_pair_kernel", "gemm2_pair_kernel")
REQUIRED_REGS = 168


def _inputs():
    files = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [os.path.join(INCLUDE, "kf_moe.h")]
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def _check_registers(ptxas_log: str) -> None:
    current = None
    for line in ptxas_log.splitlines():
        m = re.search(r"Compiling entry function '([^']+)'", line)
        if m:
            current = m.group(1)
            continue
        m = re.search(r"Used (\d+) registers", line)
        if m and current and any(k in current for k in SETMAXNREG_KERNELS):
            regs = int(m.group(1))
            if regs != REQUIRED_REGS:
                raise RuntimeError(f"{current}: ptxas allotted {regs} registers, the setmaxnreg split needs "
                                   f"exactly {REQUIRED_REGS}")


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    objs = []
    log = []
    build_dir = os.path.join(PKG, "_build")
    os.makedirs(build_dir, exist_ok=True)
    for src in SOURCES:
        obj = os.path.join(build_dir, src.replace(".cu", ".o"))
        cmd = [NVCC, *ARCH, *FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        log.append(r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        objs.append(obj)
    _check_registers("\n".join(log))
    tmp = LIB + ".tmp"
    cmd = [NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    if verbose:
        print("\n".join(log))
    return LIB


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(path)
