"""kf_moe_forward_noalloc through the C ABI: the layer for callers that cannot allocate.

Such callers (a plugin host that owns all device memory, a foreign-language
binding without a CUDA allocator, a server whose memory is fully reserved by its
own pools) cannot pass kf_moe_forward a workspace.  The allocation-free entry
point keeps its scratch in a static device array instead.  This test checks that
two calls in a row -- sharing that array, so the second sees the first's
leftovers -- give bit for bit the result of the workspace entry point (both run
the same kernels), that their status word reads back clear through the
allocation-free status reader, that a call changes neither the device's free
memory nor torch's allocation count, and that calls beyond the array's limits
are refused.

Kept in its own file, collected last, so that a stop-at-first-failure run has
already run every other test.
"""
import ctypes

import pytest
import torch

from kernelforge_b200 import binding as B
from kernelforge_b200 import synthetic as S
from oracle import moe_oracle as O
from tests.helpers import gpu_available, gpu_bank, to_cuda

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not gpu_available(), reason="needs a B200")]

KF_ERR_INVALID_ARGUMENT = 1
KF_ERR_EXCEEDS_STATIC_SCRATCH = 7


def _entry():
    fn = B.library().kf_moe_forward_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 8 + [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_float,
                                           ctypes.c_void_p, ctypes.c_void_p]
    return fn


def _read_status() -> int:
    fn = B.library().kf_moe_noalloc_read_status
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(ctypes.c_int32), ctypes.c_void_p]
    st = ctypes.c_int32(-1)
    rc = fn(ctypes.byref(st), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc in (0, 6), rc
    return int(st.value)


def _call(fn, ti, wb, offset, rsf, out):
    T = ti.routing_logits.shape[0]
    E = wb.gemm1_weights.shape[0]
    ptrs = [ctypes.c_void_p(t.data_ptr()) for t in (ti.routing_logits, ti.routing_bias, ti.hidden_states,
                                                      ti.hidden_states_scale, wb.gemm1_weights,
                                                      wb.gemm1_weights_scale, wb.gemm2_weights,
                                                      wb.gemm2_weights_scale)]
    stream = torch.cuda.current_stream()
    return fn(*ptrs, T, E, offset, ctypes.c_float(rsf), ctypes.c_void_p(out.data_ptr()),
              ctypes.c_void_p(stream.cuda_stream))


def test_noalloc_matches_workspace_entry_point_on_two_calls_in_a_row():
    fn = _entry()
    wb = gpu_bank(32, 0, seed=8)
    cases = [to_cuda(S.token_inputs(16, seed=31)), to_cuda(S.token_inputs(5, seed=32))]
    refs = [B.kernel(ti.routing_logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale,
                     wb.gemm1_weights, wb.gemm1_weights_scale, wb.gemm2_weights, wb.gemm2_weights_scale, 0, 2.5)
            for ti in cases]
    outs = [torch.full_like(r, float("nan")) for r in refs]
    torch.cuda.synchronize()
    for k, (ti, out) in enumerate(zip(cases, outs)):     # two consecutive calls sharing the static scratch
        if k == 1:    # the first call looked the array up; from here on nothing may allocate
            free0 = torch.cuda.mem_get_info()[0]
            allocs0 = torch.cuda.memory_stats().get("allocation.all.allocated", 0)
        assert _call(fn, ti, wb, 0, 2.5, out) == 0
        torch.cuda.synchronize()
        assert _read_status() == 0
    assert torch.cuda.mem_get_info()[0] == free0
    assert torch.cuda.memory_stats().get("allocation.all.allocated", 0) == allocs0
    for out, ref in zip(outs, refs):
        assert torch.equal(out, ref)      # the same kernels as kf_moe_forward: identical bits
        assert O.check_tolerance(out, ref)["ok"]


def test_noalloc_refuses_calls_beyond_its_limits():
    fn = _entry()
    null = ctypes.c_void_p(0)
    args = [null] * 8
    assert fn(*args, 17, 32, 0, ctypes.c_float(1.0), null, null) == KF_ERR_EXCEEDS_STATIC_SCRATCH
    assert fn(*args, 16, 33, 0, ctypes.c_float(1.0), null, null) == KF_ERR_EXCEEDS_STATIC_SCRATCH
    # what kf_moe_forward refuses is refused here too, as an invalid argument
    assert fn(*args, 16, 257, 0, ctypes.c_float(1.0), null, null) == KF_ERR_INVALID_ARGUMENT
    assert fn(*args, 0, 32, 240, ctypes.c_float(1.0), null, null) == KF_ERR_INVALID_ARGUMENT
    assert fn(*args, 0, 32, -1, ctypes.c_float(1.0), null, null) == KF_ERR_INVALID_ARGUMENT
    assert fn(*args, 0, 32, 0, ctypes.c_float(1.0), null, null) == 0
