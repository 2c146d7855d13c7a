"""Expert-parallel MoE layer: 256 experts sharded over N GPUs, peer-memory (or NCCL) dispatch/combine.

Rank r owns global experts ``[r*256/N, (r+1)*256/N)`` (``local_expert_offset``
in the reference's data contract, ``solution/triton/kernel.py:1826``; the
reference itself has no multi-GPU code).  Every rank routes its own tokens with
the CUDA routing kernel, then:

1. dispatch: each token is sent ONCE to every rank that owns at least one of
   its 8 experts (with N = 8 a rank owns exactly one routing group, so a token
   reaches at most ``topk_group`` = 4 ranks).  A dispatched row carries the FP8
   hidden row, its 56 fp32 scales and the token's 8 (expert id, weight) pairs
   with the experts the receiver does not own masked to -1 (7456 bytes);
2. the receiver runs the grouped expert kernels (``kf_moe_experts_packed``) on
   the rows it got, producing one partial sum per row;
3. combine: the partials travel back to their sources and each token's output
   is the sum of its partials in ascending rank order (fixed order, no
   atomics), rounded to bf16 once.

By default the rows and the partials move by stores into the ranks' symmetric
buffers (``PeerExchange``): the pack kernel writes each row straight into its
destination's receive area and the expert stage's reduce kernel writes each
partial back into its source's return area, with the library's bounded barrier
between the phases.  The host reads the count matrix (it sizes the expert
call) from an asynchronous copy, waiting only for the plan, not for the pack
that the GPU runs meanwhile.
With ``exchange="nccl"`` the same kernels run around ``torch.distributed``
all-to-alls over NCCL (split sizes first, then rows).
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

import torch
import torch.distributed as dist

H = 7168
HB = H // 128
E_GLOBAL = 256
TOP_K = 8
ROW_BYTES = H + HB * 4 + TOP_K * 4 + TOP_K * 4   # 7456: fp8 row | 56 scales | 8 ids | 8 weights


class PeerExchange:
    """This rank's symmetric buffer for the peer-to-peer exchange (``kf_ep_*_p2p``).

    One allocation per rank with the same layout, mapped into every peer by
    ``torch.distributed``'s symmetric memory (plain NVLink loads and stores; no
    multicast object is requested).  Layout: barrier flags int32 ``[world]`` |
    count matrix int32 ``[world, world]`` + status int32 | receive rows
    ``[recv_cap, 7456]`` u8 | return rows bf16 ``[send_cap, 7168]``.  The
    capacities are the same on every rank.  The flags and counts are zeroed and
    all ranks synchronise once (on the host) before the first barrier.
    """

    def __init__(self, recv_cap: int, send_cap: int, world: int, rank: int, group, device: torch.device):
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        import torch.distributed._symmetric_memory as symm
        self.recv_cap, self.send_cap = int(recv_cap), int(send_cap)
        self.world, self.rank, self.device = int(world), int(rank), device
        al = lambda n: (n + 255) // 256 * 256
        self.off_flags = 0
        self.off_meta = al(world * 4)
        self.off_recv = self.off_meta + al((world * world + 1) * 4)
        self.off_back = self.off_recv + al(self.recv_cap * ROW_BYTES)
        total = self.off_back + al(max(self.send_cap, 1) * H * 2)
        self.buf = symm.empty(total, dtype=torch.uint8, device=device)
        self.buf[:self.off_recv].zero_()
        torch.cuda.synchronize(device)
        pg = group if group is not None else dist.group.WORLD
        self.handle = symm.rendezvous(self.buf, pg.group_name)
        dist.barrier(group=group)
        ptrs = [int(x) for x in self.handle.buffer_ptrs]
        dev_ptrs = lambda off: torch.tensor([p_ + off for p_ in ptrs], dtype=torch.int64, device=device)
        self.peer_flags = dev_ptrs(self.off_flags)
        self.peer_counts = dev_ptrs(self.off_meta)
        self.peer_recv = dev_ptrs(self.off_recv)
        self.peer_back = dev_ptrs(self.off_back)
        self.flags = self.buf[self.off_flags:self.off_flags + world * 4].view(torch.int32)
        self.meta = self.buf[self.off_meta:self.off_meta + (world * world + 1) * 4].view(torch.int32)
        self.counts = self.meta[:world * world]
        self.status = self.meta[world * world:]
        self.recv = self.buf[self.off_recv:self.off_recv + self.recv_cap * ROW_BYTES].view(self.recv_cap, ROW_BYTES)
        self.back = self.buf[self.off_back:self.off_back + self.send_cap * H * 2].view(torch.bfloat16).view(-1, H)
        self.meta_host = torch.empty(world * world + 1, dtype=torch.int32).pin_memory()   # count matrix + status
        self.epoch = 0

    def barrier(self, stream) -> None:
        from . import binding as B
        self.epoch += 1
        rc = B.library().kf_ep_barrier(self.peer_flags.data_ptr(), self.flags.data_ptr(), self.rank, self.world,
                                       self.epoch, self.status.data_ptr(), stream)
        B._check(rc, "kf_ep_barrier")


def peer_capacity_needs(counts: torch.Tensor):
    """Rows the largest receive area and the largest return area must hold for a step.

    ``counts[s, d]`` = rows source s sends to destination d (every rank holds
    the same matrix after the first barrier, so every rank computes the same
    answer).  Receive area of d: the sum of column d; return area of s: the sum
    of row s.
    """
    return int(counts.sum(0).max()), int(counts.sum(1).max())


STATUS_SLOT_OVERFLOW = 0x10   # KF_STATUS_SLOT_OVERFLOW: a row beyond a receive area was dropped
STATUS_TIMEOUT_PEER = 0x20    # KF_STATUS_TIMEOUT_PEER: a rank did not reach a barrier in time


def peer_status_error(status: int) -> Optional[str]:
    """The error a non-zero status word of the peer exchange stands for (None for 0)."""
    if not status:
        return None
    what = []
    if status & STATUS_TIMEOUT_PEER:
        what.append("a rank did not reach a barrier in time")
    if status & STATUS_SLOT_OVERFLOW:
        what.append("a receive area overflowed")
    if status & ~(STATUS_TIMEOUT_PEER | STATUS_SLOT_OVERFLOW):
        what.append("unknown bits")
    return f"peer exchange: device status {status:#x} ({'; '.join(what)})"


def _exchange_counts(send_counts: torch.Tensor, group) -> torch.Tensor:
    recv = torch.empty_like(send_counts)
    dist.all_to_all_single(recv, send_counts, group=group)
    return recv


class ExpertParallelMoE:
    """One rank's share of the expert-parallel layer (CUDA routing, exchange and expert kernels)."""

    def __init__(self, weights, local_expert_offset: int, num_local: int, group=None,
                 combine_dtype: torch.dtype = torch.bfloat16, exchange: str = "p2p"):
        self.w = weights
        self.offset = int(local_expert_offset)
        self.num_local = int(num_local)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.num_local * self.world != E_GLOBAL or self.offset != self.rank * self.num_local:
            raise ValueError("expert-parallel shards must be equal, contiguous and in rank order")
        self.combine_dtype = combine_dtype
        # "p2p": dispatch rows and returned partials stored straight into the peers'
        # symmetric buffers by the library's kernels (kf_ep_*_p2p), bounded device
        # barriers in place of the two all-to-alls; "nccl": the same kernels around
        # NCCL all_to_all_single
        if exchange not in ("p2p", "nccl"):
            raise ValueError("exchange must be 'p2p' or 'nccl'")
        if exchange == "p2p" and combine_dtype != torch.bfloat16:
            raise ValueError("the peer-to-peer exchange returns bf16 partials")
        self.exchange = exchange
        self._peer = None

    def local_pairs(self) -> int:
        """(row, local expert) pairs this rank's expert kernels processed in the last forward (synchronises)."""
        ids = getattr(self, "_last_ids", None)
        if callable(ids):
            ids = ids()
        if ids is None:
            return 0
        loc = ids.to(torch.int64) - self.offset
        return int(((ids >= 0) & (loc >= 0) & (loc < self.num_local)).sum().item())

    def check(self) -> None:
        """Raise ``RuntimeError`` if a device-side check of the peer exchange has failed: a barrier
        that gave up waiting for a rank, or a row dropped at a full receive area.  Synchronises with
        the device.  ``forward`` runs the same check when it reads the next step's count matrix, so a
        failure in a step's pack or return barrier surfaces one step later at the latest; calling
        this after a step reports it at once.  The status is sticky: once set, every later step
        raises, since the exchange can no longer be trusted.  No-op for the NCCL exchange (its
        collectives raise their own errors)."""
        err = peer_status_error(self.status())
        if err:
            raise RuntimeError(err)

    def status(self) -> int:
        """The peer exchange's device status word (0: no failure; synchronises), 0 for the NCCL exchange."""
        if self.exchange != "p2p" or self._peer is None:
            return 0
        return int(self._peer.status.item())

    def forward(self, routing_logits, routing_bias, hidden_states, hidden_states_scale, routed_scaling_factor):
        """The layer on this rank's tokens.  ``hidden_states`` are e4m3 with ``hidden_states_scale``
        ``[56, T]``, or bf16 rows with ``hidden_states_scale=None``: then the peer exchange quantises
        each row as it packs it (the NCCL exchange quantises the rows first).  With the peer
        exchange, a failed barrier of this step's later phases raises at the next step or at
        ``check()``."""
        from . import binding as B
        if hidden_states_scale is None and self.exchange != "p2p":
            hidden_states, hidden_states_scale = B.quantize_hidden(hidden_states)
        # the library's entry points launch on the current device: make it the rows' device
        with torch.cuda.device(hidden_states.device):
            if self.exchange == "p2p":
                return self._forward_p2p(routing_logits, routing_bias, hidden_states, hidden_states_scale,
                                         routed_scaling_factor)
            return self._forward_nccl(routing_logits, routing_bias, hidden_states, hidden_states_scale,
                                      routed_scaling_factor)

    def _forward_nccl(self, routing_logits, routing_bias, hidden_states, hidden_states_scale, routed_scaling_factor):
        from . import binding as B
        idx, w = B.route(routing_logits, routing_bias, routed_scaling_factor)
        send, send_counts, pos = B.ep_dispatch(idx, w, hidden_states, hidden_states_scale, self.world)
        recv_counts = _exchange_counts(send_counts, self.group)
        s_split = send_counts.tolist()
        r_split = recv_counts.tolist()
        S, R = sum(s_split), sum(r_split)
        recv = torch.empty((R, ROW_BYTES), dtype=torch.uint8, device=send.device)
        dist.all_to_all_single(recv, send[:S], output_split_sizes=r_split, input_split_sizes=s_split,
                               group=self.group)
        self._last_ids = recv[:, H + HB * 4:H + HB * 4 + TOP_K * 4].contiguous().view(torch.int32)
        part = B.experts_packed(recv, self.w.gemm1_weights, self.w.gemm1_weights_scale, self.w.gemm2_weights,
                                self.w.gemm2_weights_scale, self.offset, out_dtype=self.combine_dtype)
        back = torch.empty((S, H), dtype=part.dtype, device=part.device)
        dist.all_to_all_single(back, part, output_split_sizes=s_split, input_split_sizes=r_split, group=self.group)
        return B.ep_combine(back, pos, self.world)

    def _forward_p2p(self, routing_logits, routing_bias, hidden_states, hidden_states_scale, routed_scaling_factor):
        from . import binding as B
        lib = B.library()
        dev = hidden_states.device
        T = int(hidden_states.shape[0])
        world, rank = self.world, self.rank
        if self._peer is None:
            # capacities for the largest rank's token count (agreed once, on the device)
            t = torch.tensor([T], dtype=torch.int64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
            t_max = int(t.item())
            self._peer = PeerExchange(t_max * world, int(lib.kf_ep_max_send_rows(t_max, world)), world, rank,
                                      self.group, dev)
        idx, w = B.route(routing_logits, routing_bias, routed_scaling_factor)
        hid = hidden_states.contiguous()
        hs = hidden_states_scale.contiguous() if hidden_states_scale is not None else None
        if hs is None and hid.dtype != torch.bfloat16:
            raise ValueError("without hidden_states_scale, hidden_states must be bf16 rows")
        cstream = torch.cuda.current_stream(dev)
        stream = cstream.cuda_stream
        ws = B._ep_workspace(dev, int(lib.kf_ep_workspace_bytes(T, world)))
        sz = ctypes.c_size_t(ws.numel())
        pos = torch.empty((T, world), dtype=torch.int32, device=dev)

        def plan_and_pack(pe):
            """Enqueue plan, barrier, an asynchronous copy of the count matrix, pack and barrier;
            returns the event that marks the copy."""
            B._check(lib.kf_ep_plan_p2p(B._ptr(idx), T, world, rank, pe.peer_counts.data_ptr(), B._ptr(ws), sz,
                                        stream), "kf_ep_plan_p2p")
            pe.barrier(stream)                  # every rank's count row has landed here
            pe.meta_host.copy_(pe.meta, non_blocking=True)
            copied = torch.cuda.Event()
            copied.record(cstream)
            # the pack reads the counts on the device; rows beyond a receive area are dropped
            # (and flagged), which the host sees below and redoes with larger areas
            B._check(lib.kf_ep_pack_p2p(B._ptr(idx), B._ptr(w), B._ptr(hid), B._ptr(hs), T, world, rank,
                                        pe.counts.data_ptr(), pe.peer_recv.data_ptr(), pe.recv_cap, B._ptr(pos),
                                        pe.status.data_ptr(), B._ptr(ws), sz, stream), "kf_ep_pack_p2p")
            pe.barrier(stream)                  # every row sent to this rank has landed
            return copied

        def read_counts(pe, copied):
            copied.synchronize()                # the plan only; the GPU packs meanwhile
            err = peer_status_error(int(pe.meta_host[world * world]))
            if err:
                raise RuntimeError(err)
            return pe.meta_host[:world * world].clone().view(world, world)

        pe = self._peer
        counts = read_counts(pe, plan_and_pack(pe))
        # every rank holds the same count matrix, so all of them take this branch together
        need_recv, need_send = peer_capacity_needs(counts)
        if need_recv > pe.recv_cap or need_send > pe.send_cap:
            cstream.synchronize()               # the dropped pack has finished with the old areas
            self._peer = PeerExchange(max(need_recv, pe.recv_cap), max(need_send, pe.send_cap), world, rank,
                                      self.group, dev)
            pe = self._peer
            counts = read_counts(pe, plan_and_pack(pe))
        R = int(counts[:, rank].sum())
        S = int(counts[rank, :].sum())
        recv = pe.recv[:R]
        self._last_ids = lambda: recv[:, H + HB * 4:H + HB * 4 + TOP_K * 4].contiguous().view(torch.int32)
        # the experts' last kernel (the reduce) stores each row's partial straight into
        # its source's return buffer
        B.experts_packed_p2p(recv, self.w.gemm1_weights, self.w.gemm1_weights_scale, self.w.gemm2_weights,
                             self.w.gemm2_weights_scale, self.offset, pe.counts, rank, world, pe.peer_back)
        pe.barrier(stream)                      # every partial of this rank's rows is back
        return B.ep_combine(pe.back[:S], pos, world)
