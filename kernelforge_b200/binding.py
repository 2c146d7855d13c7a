"""Python mirror of the reference operator ``kernel(...)`` over the C ABI of ``libkf_moe.so``.

``kernel`` keeps the reference's signature, argument meaning and value-returning
style (``solution/triton/kernel.py:1817-1828``): ten positional arguments, the
two scalars given as Python numbers or 0-d tensors, a new bf16 ``[T, 7168]``
tensor returned on the input device.  Errors raise ``RuntimeError``.  It is a
thin wrapper over the PyTorch C++ extension ``_kf_torch`` (``csrc/kf_torch_ext.cpp``),
which checks the tensors and calls ``kf_moe_forward`` on the current torch
stream; the other entry points (routing, experts, expert-parallel exchange,
quantiser) reach the same C ABI through ``ctypes``.

PyTorch is only plumbing here: it owns device memory (outputs and the cached
workspace come from its caching allocator) and the current stream.  All compute
runs in the CUDA kernels of ``libkf_moe.so``; there is no CPU or PyTorch
fallback -- without the library or a B200 the call fails.
"""
from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional

import torch

H = 7168
I = 2048
E_GLOBAL = 256
TOP_K = 8

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libkf_moe.so")
_lib = None
_lib_lock = threading.RLock()   # extension() loads the library while holding it

KF_OK = 0
KF_ERR_DEVICE_STATUS = 6

# Device status bits (kf_moe.h KF_STATUS_*): set by the kernels, read back by the host.
STATUS_BITS = {
    0x01: "a TMA producer timed out waiting for a free stage",
    0x02: "the MMA issuer timed out waiting for data or tensor memory",
    0x04: "a promotion/epilogue warp timed out",
    0x08: "a routed expert id outside [0, 256)",
    0x10: "a permuted row index beyond the workspace capacity",
    0x20: "a peer rank did not reach a barrier in time",
}


def status_message(status: int) -> str:
    """Text for a non-zero device status word."""
    what = [v for k, v in STATUS_BITS.items() if status & k]
    if status & ~sum(STATUS_BITS):
        what.append("unknown bits")
    return f"device status {status:#x}: " + "; ".join(what)


def _load():
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(_LIB_PATH):
            from . import build as _build
            _build.build()
        lib = ctypes.CDLL(_LIB_PATH)
        vp, i32, f32, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_float, ctypes.c_size_t
        lib.kf_moe_workspace_bytes.restype = sz
        lib.kf_moe_workspace_bytes.argtypes = [i32, i32]
        lib.kf_moe_forward.restype = ctypes.c_int
        lib.kf_moe_forward.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, f32, vp, vp, sz, vp]
        lib.kf_moe_route.restype = ctypes.c_int
        lib.kf_moe_route.argtypes = [vp, vp, i32, f32, vp, vp, vp]
        lib.kf_moe_experts.restype = ctypes.c_int
        lib.kf_moe_experts.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, vp, i32, vp, sz, vp]
        lib.kf_moe_read_status.restype = ctypes.c_int
        lib.kf_moe_read_status.argtypes = [vp, ctypes.POINTER(i32), vp]
        lib.kf_moe_error_string.restype = ctypes.c_char_p
        lib.kf_moe_error_string.argtypes = [ctypes.c_int]
        lib.kf_moe_launches_per_forward.restype = i32
        lib.kf_moe_launches_per_forward.argtypes = []
        lib.kf_moe_experts_packed.restype = ctypes.c_int
        lib.kf_moe_experts_packed.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, vp, i32, vp, sz, vp]
        lib.kf_ep_workspace_bytes.restype = sz
        lib.kf_ep_workspace_bytes.argtypes = [i32, i32]
        lib.kf_ep_max_send_rows.restype = i32
        lib.kf_ep_max_send_rows.argtypes = [i32, i32]
        lib.kf_ep_dispatch.restype = ctypes.c_int
        lib.kf_ep_dispatch.argtypes = [vp, vp, vp, vp, i32, i32, vp, vp, vp, vp, sz, vp]
        lib.kf_ep_combine.restype = ctypes.c_int
        lib.kf_ep_combine.argtypes = [vp, i32, vp, i32, i32, vp, vp]
        lib.kf_ep_plan_p2p.restype = ctypes.c_int
        lib.kf_ep_plan_p2p.argtypes = [vp, i32, i32, i32, vp, vp, sz, vp]
        lib.kf_ep_pack_p2p.restype = ctypes.c_int
        lib.kf_ep_pack_p2p.argtypes = [vp, vp, vp, vp, i32, i32, i32, vp, vp, i32, vp, vp, vp, sz, vp]
        lib.kf_ep_return_p2p.restype = ctypes.c_int
        lib.kf_ep_return_p2p.argtypes = [vp, i32, i32, i32, vp, vp, vp]
        lib.kf_moe_experts_packed_p2p.restype = ctypes.c_int
        lib.kf_moe_experts_packed_p2p.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, vp, i32, i32, vp, vp, sz, vp]
        lib.kf_ep_barrier.restype = ctypes.c_int
        lib.kf_ep_barrier.argtypes = [vp, vp, i32, i32, i32, vp, vp]
        lib.kf_quantize_hidden.restype = ctypes.c_int
        lib.kf_quantize_hidden.argtypes = [vp, i32, vp, vp, vp]
        lib.kf_moe_profile_begin.restype = ctypes.c_int
        lib.kf_moe_profile_begin.argtypes = []
        lib.kf_moe_profile_end.restype = ctypes.c_int
        lib.kf_moe_profile_end.argtypes = [ctypes.POINTER(f32), ctypes.POINTER(i32), i32]
        _lib = lib
    return _lib


def library():
    """The loaded ``ctypes.CDLL`` (loads it on first use)."""
    return _load()


_ext_mod = None


def extension():
    """The torch extension module ``_kf_torch`` (built on first use if missing); ``libkf_moe.so``
    is loaded first, so the extension's dependency on it resolves to that copy."""
    global _ext_mod
    if _ext_mod is not None:
        return _ext_mod
    with _lib_lock:
        if _ext_mod is None:
            import importlib.machinery
            import importlib.util

            from . import build as _build
            _load()
            if not _build.ext_up_to_date():
                _build.build_ext()
            loader = importlib.machinery.ExtensionFileLoader("_kf_torch", _build.EXT)
            spec = importlib.util.spec_from_file_location("_kf_torch", _build.EXT, loader=loader)
            mod = importlib.util.module_from_spec(spec)
            loader.exec_module(mod)
            _ext_mod = mod
    return _ext_mod


def _call(device: torch.device, fn, *args) -> int:
    """One C-ABI call with ``device`` current: the library launches on, and sets
    itself up for, the current CUDA device, while the tensors of a call may live
    on any device (as with the reference's operator)."""
    with torch.cuda.device(device):
        return fn(*args)


def _check(rc: int, what: str) -> None:
    if rc != KF_OK:
        msg = _load().kf_moe_error_string(rc).decode()
        raise RuntimeError(f"{what} failed: {msg} (code {rc})")


# One workspace per (device, stream): calls queued on one stream run in order, so
# they can share scratch memory; calls on different streams get their own.
_workspaces: dict = {}
_ws_lock = threading.Lock()

# Device errors raise on the host without a synchronisation per call: after each
# launch the workspace's status word (its first 4 bytes, written by the kernels,
# cleared by the next call on that workspace) is copied asynchronously into a
# pinned host word and an event is recorded.  Every later call on the workspace
# first looks at the copies whose events have completed and raises RuntimeError
# for a non-zero word; read_status() synchronises and reports at once.
_pending: dict = {}      # workspace key -> [(pinned int32 [1], event)] in launch order
_free_mirrors: list = []


def _check_pending(key) -> None:
    q = _pending.get(key)
    while q and q[0][1].query():
        mirror, ev = q.pop(0)
        v = int(mirror[0])
        _free_mirrors.append((mirror, ev))
        if v:
            raise RuntimeError("an earlier call on this stream failed on the device: " + status_message(v))


def _mirror_status(key, buf: torch.Tensor, stream) -> None:
    if torch.cuda.is_current_stream_capturing():
        return        # a captured call's status is not mirrored (the graph replays without host checks)
    mirror, ev = _free_mirrors.pop() if _free_mirrors else (torch.zeros(1, dtype=torch.int32).pin_memory(),
                                                            torch.cuda.Event())
    with torch.cuda.stream(stream):
        mirror.copy_(buf[:4].view(torch.int32), non_blocking=True)
    ev.record(stream)
    _pending.setdefault(key, []).append((mirror, ev))


def workspace(num_tokens: int, num_local: int, device: torch.device, stream: Optional[torch.cuda.Stream] = None):
    need = int(_load().kf_moe_workspace_bytes(int(num_tokens), int(num_local)))
    stream = stream or torch.cuda.current_stream(device)
    key = (device.index, stream.cuda_stream)
    with _ws_lock:
        _check_pending(key)
        buf = _workspaces.get(key)
        if buf is None or buf.numel() < need:
            buf = torch.empty(need, dtype=torch.uint8, device=device)
            _workspaces[key] = buf
    return buf


def _launched(device: torch.device, stream, buf: torch.Tensor) -> None:
    """Bookkeeping after a successful launch on ``buf``: mirror its status word."""
    with _ws_lock:
        _mirror_status((device.index, stream.cuda_stream), buf, stream)


def release_workspaces() -> None:
    """Drop the cached scratch buffers of every device and stream (they return to
    torch's caching allocator); the next call allocates again.  Call it only when
    no library work is pending on those streams."""
    with _ws_lock:
        _workspaces.clear()
        _ep_ws.clear()
        _pending.clear()
    if _ext_mod is not None:
        _ext_mod.release_workspaces()


def _ptr(t: Optional[torch.Tensor]):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _scalar_int(v) -> int:
    return int(v.item()) if isinstance(v, torch.Tensor) else int(v)


def _scalar_float(v) -> float:
    return float(v.item()) if isinstance(v, torch.Tensor) else float(v)


def _expect(t: torch.Tensor, name: str, dtype, shape, device):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {tuple(shape)}, got {tuple(t.shape)}")
    if t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")
    return t.contiguous()


def _weights(gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, device):
    if gemm1_weights.dim() != 3:
        raise ValueError("gemm1_weights must be [E, 4096, 7168]")
    E = int(gemm1_weights.shape[0])
    w13 = _expect(gemm1_weights, "gemm1_weights", torch.float8_e4m3fn, (E, 2 * I, H), device)
    w13s = _expect(gemm1_weights_scale, "gemm1_weights_scale", torch.float32, (E, 2 * I // 128, H // 128), device)
    w2 = _expect(gemm2_weights, "gemm2_weights", torch.float8_e4m3fn, (E, H, I), device)
    w2s = _expect(gemm2_weights_scale, "gemm2_weights_scale", torch.float32, (E, H // 128, I // 128), device)
    return E, w13, w13s, w2, w2s


def kernel(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
           gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
           routed_scaling_factor):
    """Fused DeepSeek-V3 FP8 block-scale MoE layer; returns bf16 ``[T, 7168]``.

    Same contract as the reference ``kernel`` (``solution/triton/kernel.py:1817``):
    routing_logits f32 [T,256], routing_bias bf16 [256], hidden_states e4m3
    [T,7168], hidden_states_scale f32 [56,T], gemm1_weights e4m3 [E,4096,7168],
    gemm1_weights_scale f32 [E,32,56], gemm2_weights e4m3 [E,7168,2048],
    gemm2_weights_scale f32 [E,56,16]; local_expert_offset / routed_scaling_factor
    as numbers or 0-d tensors.  E (local experts) is taken from the weights.
    """
    if hidden_states.device.type != "cuda":
        raise RuntimeError("kernelforge_b200.kernel needs CUDA tensors on a B200 (sm_100a); no CPU fallback")
    return extension().kernel(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                              gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                              _scalar_int(local_expert_offset), _scalar_float(routed_scaling_factor))


def route(routing_logits, routing_bias, routed_scaling_factor):
    """Routing only: ``(topk_idx int32 [T,8], topk_weight f32 [T,8])``, descending score order."""
    device = routing_logits.device
    T = int(routing_logits.shape[0])
    logits = _expect(routing_logits, "routing_logits", torch.float32, (T, E_GLOBAL), device)
    bias = _expect(routing_bias.reshape(-1), "routing_bias", torch.bfloat16, (E_GLOBAL,), device)
    idx = torch.empty((T, TOP_K), dtype=torch.int32, device=device)
    w = torch.empty((T, TOP_K), dtype=torch.float32, device=device)
    if T:
        stream = torch.cuda.current_stream(device)
        rc = _call(device, _load().kf_moe_route, _ptr(logits), _ptr(bias), T,
                   ctypes.c_float(_scalar_float(routed_scaling_factor)), _ptr(idx), _ptr(w),
                   ctypes.c_void_p(stream.cuda_stream))
        _check(rc, "kf_moe_route")
    return idx, w


def experts(topk_idx, topk_weight, hidden_states, hidden_states_scale, gemm1_weights, gemm1_weights_scale,
            gemm2_weights, gemm2_weights_scale, local_expert_offset, out_dtype=torch.bfloat16):
    """Experts on pre-routed rows: ``out[t] = sum_k w[t,k] * FFN_{e[t,k]}(x[t])`` over local experts.

    ``topk_idx`` int32 [T,8] holds global expert ids or -1; ids outside the local
    range contribute nothing.  Returns ``out_dtype`` (bf16 or f32) ``[T, 7168]``.
    """
    device = hidden_states.device
    T = int(hidden_states.shape[0])
    idx = _expect(topk_idx, "topk_idx", torch.int32, (T, TOP_K), device)
    w = _expect(topk_weight, "topk_weight", torch.float32, (T, TOP_K), device)
    hid = _expect(hidden_states, "hidden_states", torch.float8_e4m3fn, (T, H), device)
    hs = _expect(hidden_states_scale, "hidden_states_scale", torch.float32, (H // 128, T), device)
    E, w13, w13s, w2, w2s = _weights(gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, device)
    offset = _scalar_int(local_expert_offset)
    if out_dtype not in (torch.bfloat16, torch.float32):
        raise TypeError("out_dtype must be bfloat16 or float32")
    out = torch.empty((T, H), dtype=out_dtype, device=device)
    if T == 0:
        return out
    stream = torch.cuda.current_stream(device)
    ws = workspace(T, E, device, stream)
    rc = _call(device, _load().kf_moe_experts, _ptr(idx), _ptr(w), _ptr(hid), _ptr(hs), _ptr(w13), _ptr(w13s),
               _ptr(w2), _ptr(w2s), T, E, offset, _ptr(out), 1 if out_dtype == torch.float32 else 0, _ptr(ws),
               ctypes.c_size_t(ws.numel()), ctypes.c_void_p(stream.cuda_stream))
    _check(rc, "kf_moe_experts")
    _launched(device, stream, ws)
    return out


def read_status(device: Optional[torch.device] = None) -> int:
    """Synchronise and return (then clear) the device status word of the current stream's workspace.

    Also settles the asynchronous status copies of earlier calls on that workspace, so a
    non-zero word is reported here once rather than raised again by the next call.
    """
    device = device or torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream(device)
    key = (device.index, stream.cuda_stream)
    from_ext = int(_ext_mod.read_status(device.index)) if _ext_mod is not None else 0   # kernel() calls
    buf = _workspaces.get(key)
    if buf is None:
        return from_ext
    st = ctypes.c_int32(0)
    rc = _call(device, _load().kf_moe_read_status, _ptr(buf), ctypes.byref(st), ctypes.c_void_p(stream.cuda_stream))
    if rc not in (KF_OK, KF_ERR_DEVICE_STATUS):
        _check(rc, "kf_moe_read_status")
    earlier = 0
    with _ws_lock:
        for mirror, ev in _pending.pop(key, []):
            earlier |= int(mirror[0])
            _free_mirrors.append((mirror, ev))
    return int(st.value) | earlier | from_ext


def check(device: Optional[torch.device] = None) -> None:
    """Synchronise and raise ``RuntimeError`` if a call on the current stream set a device status bit."""
    st = read_status(device)
    if st:
        raise RuntimeError(status_message(st))


KERNEL_NAMES = ["route", "masks_from_topk", "permute_scan", "permute_assign", "gather_rows", "gemm1_swiglu",
                "gemm2_weighted", "unpermute_reduce", "front_small", "swiglu_quant"]


def profile_begin() -> None:
    """Start bracketing every library kernel launch with CUDA events."""
    _check(_load().kf_moe_profile_begin(), "kf_moe_profile_begin")


def profile_end() -> dict:
    """Stop profiling; returns ``{kernel: (total_ms, launches)}`` (synchronises the events)."""
    n = len(KERNEL_NAMES)
    ms = (ctypes.c_float * n)()
    cnt = (ctypes.c_int32 * n)()
    _check(_load().kf_moe_profile_end(ms, cnt, n), "kf_moe_profile_end")
    return {KERNEL_NAMES[i]: (float(ms[i]), int(cnt[i])) for i in range(n)}


PACKED_ROW_BYTES = H + (H // 128) * 4 + TOP_K * 4 + TOP_K * 4   # 7456


def experts_packed(rows, gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                   local_expert_offset, out_dtype=torch.bfloat16):
    """Experts on packed expert-parallel rows (uint8 ``[R, 7456]``, as ``ep_dispatch`` writes them)."""
    device = rows.device
    R = int(rows.shape[0])
    if rows.dtype != torch.uint8 or rows.dim() != 2 or rows.shape[1] != PACKED_ROW_BYTES:
        raise ValueError("rows must be uint8 [R, 7456]")
    rows = rows.contiguous()
    E, w13, w13s, w2, w2s = _weights(gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, device)
    out = torch.empty((R, H), dtype=out_dtype, device=device)
    if R == 0:
        return out
    stream = torch.cuda.current_stream(device)
    ws = workspace(R, E, device, stream)
    rc = _call(device, _load().kf_moe_experts_packed, _ptr(rows), _ptr(w13), _ptr(w13s), _ptr(w2), _ptr(w2s), R, E,
               _scalar_int(local_expert_offset), _ptr(out), 1 if out_dtype == torch.float32 else 0, _ptr(ws),
               ctypes.c_size_t(ws.numel()), ctypes.c_void_p(stream.cuda_stream))
    _check(rc, "kf_moe_experts_packed")
    _launched(device, stream, ws)
    return out


def experts_packed_p2p(rows, gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                       local_expert_offset, counts, rank: int, world: int, peer_back) -> None:
    """``experts_packed`` whose reduce stores each row's bf16 partial into its source rank's return buffer.

    ``counts``: this rank's int32 ``[world * world]`` count matrix; ``peer_back``:
    int64 device tensor of the ``world`` ranks' return-buffer addresses.
    """
    device = rows.device
    R = int(rows.shape[0])
    if rows.dtype != torch.uint8 or rows.dim() != 2 or rows.shape[1] != PACKED_ROW_BYTES:
        raise ValueError("rows must be uint8 [R, 7456]")
    if R == 0:
        return
    rows = rows.contiguous()
    E, w13, w13s, w2, w2s = _weights(gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, device)
    stream = torch.cuda.current_stream(device)
    ws = workspace(R, E, device, stream)
    rc = _call(device, _load().kf_moe_experts_packed_p2p, _ptr(rows), _ptr(w13), _ptr(w13s), _ptr(w2), _ptr(w2s), R,
               E, _scalar_int(local_expert_offset), _ptr(counts), int(rank), int(world), _ptr(peer_back), _ptr(ws),
               ctypes.c_size_t(ws.numel()), ctypes.c_void_p(stream.cuda_stream))
    _check(rc, "kf_moe_experts_packed_p2p")
    _launched(device, stream, ws)


_ep_ws: dict = {}


def _ep_workspace(device: torch.device, need: int) -> torch.Tensor:
    """Cached scratch of the expert-parallel kernels for (device, current stream)."""
    stream = torch.cuda.current_stream(device)
    key = (device.index, stream.cuda_stream)
    buf = _ep_ws.get(key)
    if buf is None or buf.numel() < need:
        buf = torch.empty(max(need, 256), dtype=torch.uint8, device=device)
        _ep_ws[key] = buf
    return buf


def ep_dispatch(topk_idx, topk_weight, hidden_states, hidden_states_scale, world: int):
    """Device-side expert-parallel dispatch: ``(send_rows [S_max, 7456] u8, send_counts i64 [world], pos i32 [T, world])``."""
    device = hidden_states.device
    T = int(hidden_states.shape[0])
    lib = _load()
    idx = _expect(topk_idx, "topk_idx", torch.int32, (T, TOP_K), device)
    w = _expect(topk_weight, "topk_weight", torch.float32, (T, TOP_K), device)
    hid = _expect(hidden_states, "hidden_states", torch.float8_e4m3fn, (T, H), device)
    hs = _expect(hidden_states_scale, "hidden_states_scale", torch.float32, (H // 128, T), device)
    send = torch.empty((int(lib.kf_ep_max_send_rows(T, world)), PACKED_ROW_BYTES), dtype=torch.uint8, device=device)
    counts = torch.empty((world,), dtype=torch.int64, device=device)
    pos = torch.empty((T, world), dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream(device)
    need = int(lib.kf_ep_workspace_bytes(T, world))
    key = (device.index, stream.cuda_stream)
    buf = _ep_ws.get(key)
    if buf is None or buf.numel() < need:
        buf = torch.empty(max(need, 256), dtype=torch.uint8, device=device)
        _ep_ws[key] = buf
    rc = _call(device, lib.kf_ep_dispatch, _ptr(idx), _ptr(w), _ptr(hid), _ptr(hs), T, int(world), _ptr(send),
               _ptr(counts), _ptr(pos), _ptr(buf), ctypes.c_size_t(buf.numel()),
               ctypes.c_void_p(stream.cuda_stream))
    _check(rc, "kf_ep_dispatch")
    return send, counts, pos


def ep_combine(partials, pos, world: int):
    """bf16 ``[T, 7168]``: per token, the sum of its destinations' partial rows in ascending rank order."""
    device = pos.device
    T = int(pos.shape[0])
    out = torch.empty((T, H), dtype=torch.bfloat16, device=device)
    if T == 0:
        return out
    if partials.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError("partials must be bf16 or f32")
    partials = partials.contiguous()
    pos = pos.to(torch.int32).contiguous()
    stream = torch.cuda.current_stream(device)
    rc = _call(device, _load().kf_ep_combine, _ptr(partials) if partials.numel() else ctypes.c_void_p(0),
               1 if partials.dtype == torch.float32 else 0, _ptr(pos), T, int(world), _ptr(out),
               ctypes.c_void_p(stream.cuda_stream))
    _check(rc, "kf_ep_combine")
    return out


def quantize_hidden(x: torch.Tensor):
    """bf16 rows ``[T, 7168]`` -> (e4m3 ``[T, 7168]``, f32 scales ``[56, T]``): the input format of ``kernel``.

    Per row and 128 columns: scale = absmax / 448 (1 for an all-zero block),
    q = e4m3(x / scale) -- the reference's ``_quantize_fp8_block_rows``
    (``solution/triton/kernel.py:126-141``), computed by ``kf_quantize_hidden``.
    """
    if x.dim() != 2 or x.shape[1] != H or x.dtype != torch.bfloat16 or not x.is_cuda:
        raise RuntimeError("quantize_hidden expects a CUDA bf16 tensor [T, 7168]")
    x = x.contiguous()
    T = x.shape[0]
    q = torch.empty((T, H), dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty((H // 128, T), dtype=torch.float32, device=x.device)
    rc = _call(x.device, _load().kf_quantize_hidden, _ptr(x), T, _ptr(q), _ptr(s),
               torch.cuda.current_stream(x.device).cuda_stream)
    _check(rc, "kf_quantize_hidden")
    return q, s
