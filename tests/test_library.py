"""The C-ABI library: builds, loads and exports every entry point ``include/kf_moe.h`` declares.

No compute calls here (no GPU in the CPU tier): host-only entry points are called,
device entry points are only resolved.
"""
import ctypes
import os
import re

import pytest
import torch

from kernelforge_b200 import binding as B

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "kf_moe.h")).read()
    return sorted(set(re.findall(r"^\s*(?:[\w\s\*]+?)\b(kf_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_entry_points():
    syms = declared_symbols()
    for s in ["kf_moe_forward", "kf_moe_route", "kf_moe_experts", "kf_moe_workspace_bytes",
              "kf_moe_read_status", "kf_moe_error_string", "kf_moe_launches_per_forward"]:
        assert s in syms


def test_library_exports_every_declared_symbol():
    lib = B.library()
    for s in declared_symbols():
        assert hasattr(lib, s), s
        assert ctypes.cast(getattr(lib, s), ctypes.c_void_p).value


def test_workspace_bytes_is_host_only_and_monotone():
    lib = B.library()
    a = lib.kf_moe_workspace_bytes(16, 32)
    b = lib.kf_moe_workspace_bytes(4096, 32)
    c = lib.kf_moe_workspace_bytes(4096, 256)
    assert 0 < a < b < c
    assert lib.kf_moe_workspace_bytes(-1, 32) == 0
    assert lib.kf_moe_workspace_bytes(16, 0) == 0
    assert lib.kf_moe_workspace_bytes(16, 257) == 0
    # worst case: every token on min(8, E) local experts, each expert padded to 128 rows; per row the
    # gathered FP8 row, the hi and lo FP8 intermediate and the bf16 GEMM2 output row
    rows = ((4096 * 8 + 32 * 127) + 127) // 128 * 128
    assert b > rows * (7168 + 2 * 2048 + 7168 * 2)


def test_token_ceiling():
    """Counts above KF_MOE_MAX_TOKENS are refused on the host (no 32-bit index can wrap)."""
    text = open(os.path.join(ROOT, "include", "kf_moe.h")).read()
    m = re.search(r"#define KF_MOE_MAX_TOKENS \(1 << (\d+)\)", text)
    cap = 1 << int(m.group(1))
    lib = B.library()
    assert lib.kf_moe_workspace_bytes(cap, 256) >= lib.kf_moe_workspace_bytes(cap - 1, 256) > 0
    assert lib.kf_moe_workspace_bytes(cap + 1, 32) == 0
    assert lib.kf_moe_workspace_bytes(2 ** 31 - 1, 1) == 0
    assert lib.kf_ep_max_send_rows(cap, 8) == cap * 8
    assert lib.kf_ep_max_send_rows(cap + 1, 8) == 0
    assert lib.kf_ep_workspace_bytes(cap + 1, 8) == 0
    null = ctypes.c_void_p(0)
    rc = lib.kf_moe_forward(null, null, null, null, null, null, null, null, cap + 1, 32, 0, ctypes.c_float(1.0), null,
                            null, ctypes.c_size_t(0), null)
    assert rc == 1
    assert lib.kf_quantize_hidden(null, cap + 1, null, null, null) == 1


def test_library_calls_run_with_the_tensors_device_current(monkeypatch):
    """_call makes the given device current around the C-ABI call (the library launches on the current device)."""
    seen = []

    class Guard:
        def __init__(self, d):
            self.d = d

        def __enter__(self):
            seen.append(("enter", self.d))

        def __exit__(self, *exc):
            seen.append(("exit", self.d))

    monkeypatch.setattr(torch.cuda, "device", Guard)
    dev = torch.device("cuda", 3)
    assert B._call(dev, lambda a, b: (seen.append("call"), a + b)[1], 1, 2) == 3
    assert seen == [("enter", dev), "call", ("exit", dev)]


def test_every_device_entry_point_goes_through_the_device_guard():
    """In the binding, each call of a launching entry point is made through _call."""
    src = open(os.path.join(ROOT, "kernelforge_b200", "binding.py")).read()
    host_only = {"kf_moe_workspace_bytes", "kf_ep_workspace_bytes", "kf_ep_max_send_rows", "kf_moe_error_string",
                 "kf_moe_profile_begin", "kf_moe_profile_end", "kf_moe_launches_per_forward"}
    direct = [n for n in re.findall(r"(?:_load\(\)|lib)\.(kf_\w+)\(", src) if n not in host_only]
    assert not direct, f"called without _call: {direct}"
    routed = re.findall(r"_call\(\s*[\w.]+,\s*(?:_load\(\)|lib)\.(kf_\w+),", src)
    assert {"kf_moe_route", "kf_moe_experts", "kf_moe_experts_packed", "kf_moe_experts_packed_p2p",
            "kf_ep_dispatch", "kf_ep_combine", "kf_quantize_hidden", "kf_moe_read_status"} <= set(routed)
    # kernel() goes through the torch extension, which makes the tensors' device current the same way
    ext = open(os.path.join(ROOT, "kernelforge_b200", "csrc", "kf_torch_ext.cpp")).read()
    body = ext[ext.index("at::Tensor kernel("):]
    assert body.index("c10::cuda::CUDAGuard guard(dev)") < body.index("kf_moe_forward(")


def test_release_workspaces_empties_the_caches():
    B._workspaces[(0, 0)] = torch.empty(8, dtype=torch.uint8)
    B._ep_ws[(0, 0)] = torch.empty(8, dtype=torch.uint8)
    B.release_workspaces()
    assert not B._workspaces and not B._ep_ws


def test_error_strings():
    lib = B.library()
    assert lib.kf_moe_error_string(0) == b"ok"
    assert b"workspace" in lib.kf_moe_error_string(2)
    assert lib.kf_moe_launches_per_forward() == 7


def test_invalid_arguments_rejected_before_any_device_work():
    lib = B.library()
    null = ctypes.c_void_p(0)
    # E out of range / offset out of range / null pointers: rejected on the host
    rc = lib.kf_moe_forward(null, null, null, null, null, null, null, null, 4, 0, 0, ctypes.c_float(1.0), null,
                            null, ctypes.c_size_t(0), null)
    assert rc == 1
    rc = lib.kf_moe_forward(null, null, null, null, null, null, null, null, 4, 32, 240, ctypes.c_float(1.0), null,
                            null, ctypes.c_size_t(0), null)
    assert rc == 1
    rc = lib.kf_moe_forward(null, null, null, null, null, null, null, null, 4, 32, 0, ctypes.c_float(1.0), null,
                            null, ctypes.c_size_t(0), null)
    assert rc == 1
    # T == 0 is a no-op
    rc = lib.kf_moe_forward(null, null, null, null, null, null, null, null, 0, 32, 0, ctypes.c_float(1.0), null,
                            null, ctypes.c_size_t(0), null)
    assert rc == 0


def test_python_kernel_refuses_cpu_tensors():
    from kernelforge_b200 import synthetic as S
    ti = S.token_inputs(2, seed=0)
    wb = S.expert_bank(1, 0, only=[])
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        B.kernel(ti.routing_logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale,
                 wb.gemm1_weights, wb.gemm1_weights_scale, wb.gemm2_weights, wb.gemm2_weights_scale, 0, 2.5)


def test_noalloc_static_scratch_covers_its_limits():
    """The static scratch of the allocation-free entry point holds the workspace
    of its largest accepted call (checked on the host, so layout changes that
    outgrow it fail here rather than on a GPU)."""
    text = open(os.path.join(ROOT, "include", "kf_moe.h")).read()
    size = re.search(r"#define KF_MOE_NOALLOC_SCRATCH_BYTES \((\d+)u << (\d+)\)", text)
    max_t = int(re.search(r"#define KF_MOE_NOALLOC_MAX_TOKENS (\d+)", text).group(1))
    max_e = int(re.search(r"#define KF_MOE_NOALLOC_MAX_LOCAL_EXPERTS (\d+)", text).group(1))
    scratch = int(size.group(1)) << int(size.group(2))
    lib = B.library()
    assert all(lib.kf_moe_workspace_bytes(t, e) <= scratch for t in (1, max_t) for e in (1, max_e))


def test_torch_extension_binds_the_c_abi():
    """The PyTorch C++ extension loads beside libkf_moe.so, exposes the operator and refuses CPU tensors
    itself (no GPU needed)."""
    from kernelforge_b200 import synthetic as S
    ext = B.extension()
    assert callable(ext.kernel) and callable(ext.read_status) and callable(ext.release_workspaces)
    ti = S.token_inputs(2, seed=0)
    wb = S.expert_bank(1, 0, only=[])
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ext.kernel(ti.routing_logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale, wb.gemm1_weights,
                   wb.gemm1_weights_scale, wb.gemm2_weights, wb.gemm2_weights_scale, 0, 2.5)
    ext.release_workspaces()


def test_extension_loads_first_in_a_fresh_process():
    """A process whose first call into the binding is the extension (as kernel() is for a caller that
    never routes first) loads the library and the extension without deadlocking."""
    import subprocess
    import sys
    code = ("import sys; sys.path.insert(0, %r); from kernelforge_b200 import binding as B; "
            "ext = B.extension(); print(callable(ext.kernel))" % ROOT)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip().endswith("True"), r.stderr[-2000:]
