"""Build the sm_100a shared library ``kernelforge_b200/libkf_moe.so`` with nvcc, and the PyTorch
C++ extension ``kernelforge_b200/_kf_torch.so`` that binds its C ABI for torch tensors.

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
EXT = os.path.join(PKG, "_kf_torch.so")
EXT_SOURCE = "kf_torch_ext.cpp"
SOURCES = ["kf_route_permute.cu", "kf_grouped_gemm.cu", "kf_moe_api.cu",
           "kf_moe_noalloc.cu", "kf_ep.cu", "kf_quant.cu"]
HEADERS = ["kf_ptx.cuh", "kf_internal.cuh", "kf_quant.cuh", "kf_fp8.cuh"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xptxas", "-v", f"-I{INCLUDE}"]
# ptxas's register count of each kernel whose setmaxnreg split assumes it
REQUIRED_REGS = {"gemm1_swiglu_kernel": 168, "gemm2_weighted_kernel": 168}


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
        if m and current:
            for k, need in REQUIRED_REGS.items():
                if k in current and int(m.group(1)) != need:
                    raise RuntimeError(f"{current}: ptxas allotted {m.group(1)} registers, the setmaxnreg split needs "
                                       f"exactly {need}")


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
    # the soname lets the torch extension's dependency on libkf_moe.so resolve to the
    # copy the binding has already loaded
    cmd = [NVCC, *ARCH, "-shared", "-Xlinker", "-soname=libkf_moe.so", "-o", tmp, *objs, "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    if verbose:
        print("\n".join(log))
    return LIB


def ext_up_to_date() -> bool:
    if not os.path.exists(EXT):
        return False
    t = os.path.getmtime(EXT)
    deps = [os.path.join(CSRC, EXT_SOURCE), os.path.join(INCLUDE, "kf_moe.h"), LIB]
    return all(os.path.getmtime(f) <= t for f in deps)


def build_ext(force: bool = False, verbose: bool = False) -> str:
    """The torch extension (``kf_torch_ext.cpp``), linked against ``libkf_moe.so``."""
    if not force and ext_up_to_date():
        return EXT
    import ctypes
    import shutil

    from torch.utils import cpp_extension
    ctypes.CDLL(LIB)                      # its soname satisfies the extension's dependency when imported here
    bdir = os.path.join(PKG, "_build", "torch_ext")
    os.makedirs(bdir, exist_ok=True)
    cpp_extension.load(name="_kf_torch", sources=[os.path.join(CSRC, EXT_SOURCE)], extra_include_paths=[INCLUDE],
                       extra_cflags=["-O3"], extra_ldflags=[f"-L{PKG}", "-lkf_moe"], build_directory=bdir,
                       with_cuda=True, verbose=verbose)
    tmp = EXT + ".tmp"
    shutil.copyfile(os.path.join(bdir, "_kf_torch.so"), tmp)
    os.replace(tmp, EXT)
    return EXT


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(path)
    print(build_ext(force="--force" in sys.argv, verbose="-v" in sys.argv))
