"""PyTorch restatement of the expert-parallel exchange -- TEST INFRASTRUCTURE.

The product's exchange (``kernelforge_b200.ep.ExpertParallelMoE``) runs CUDA
kernels around peer-memory stores or NCCL all-to-alls.  This module states the
same data flow with tensor ops so that:

* the CPU tests can run it on gloo ranks (dispatch dedup and masking, the
  exchange in both directions, the fixed-order combine, a dropped rank), and
* the GPU tests can check the CUDA pack, unpack and combine kernels against it.

Nothing under ``kernelforge_b200/`` imports it.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist

from kernelforge_b200.ep import E_GLOBAL, H, HB, ROW_BYTES, TOP_K


@dataclass
class DispatchPlan:
    send_counts: torch.Tensor   # int64 [N]: rows sent to each rank
    send_token: torch.Tensor    # int64 [S]: source token of each send row (grouped by destination)
    send_ids: torch.Tensor      # int32 [S, 8]: expert ids, -1 where the destination does not own the expert
    send_w: torch.Tensor        # f32 [S, 8]
    pos: torch.Tensor           # int64 [T, N]: row of (token, destination) in the send buffer, -1 if not sent


def dispatch_plan(topk_idx: torch.Tensor, topk_w: torch.Tensor, world: int) -> DispatchPlan:
    """Which rows go to which rank, deduplicated per (token, destination), token order kept."""
    T = topk_idx.shape[0]
    per_rank = E_GLOBAL // world
    ids = topk_idx.to(torch.int64)
    dest = ids // per_rank                                               # [T, 8]
    member = torch.zeros(T, world, dtype=torch.bool, device=ids.device)
    member.scatter_(1, dest, True)
    send_counts = member.sum(dim=0)
    d_idx, t_idx = torch.nonzero(member.t(), as_tuple=True)             # destination-major, token order
    pos = torch.full((T, world), -1, dtype=torch.int64, device=ids.device)
    pos[t_idx, d_idx] = torch.arange(t_idx.numel(), device=ids.device)
    own = dest[t_idx] == d_idx.unsqueeze(1)
    send_ids = torch.where(own, ids[t_idx], torch.full_like(ids[t_idx], -1)).to(torch.int32)
    send_w = torch.where(own, topk_w[t_idx].to(torch.float32), torch.zeros_like(topk_w[t_idx], dtype=torch.float32))
    return DispatchPlan(send_counts, t_idx, send_ids, send_w, pos)


def pack_rows(hidden: torch.Tensor, hidden_scale: torch.Tensor, plan: DispatchPlan) -> torch.Tensor:
    """[S, 7456] uint8 rows: hidden fp8 | scales f32 [56] | ids int32 [8] | weights f32 [8]."""
    tok = plan.send_token
    parts = [hidden.index_select(0, tok).view(torch.uint8),
             hidden_scale.t().index_select(0, tok).contiguous().view(torch.uint8),
             plan.send_ids.contiguous().view(torch.uint8),
             plan.send_w.contiguous().view(torch.uint8)]
    return torch.cat(parts, dim=1)


def unpack_rows(rows: torch.Tensor):
    """Inverse of pack_rows: (hidden e4m3 [R,7168], scales f32 [56,R], ids int32 [R,8], w f32 [R,8])."""
    hid = rows[:, :H].contiguous().view(torch.float8_e4m3fn)
    sc = rows[:, H:H + HB * 4].contiguous().view(torch.float32).t().contiguous()
    ids = rows[:, H + HB * 4:H + HB * 4 + TOP_K * 4].contiguous().view(torch.int32)
    w = rows[:, H + HB * 4 + TOP_K * 4:].contiguous().view(torch.float32)
    return hid, sc, ids, w


def combine(back: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
    """out[t] = sum over destinations d (ascending) of back[pos[t, d]]; fp32 sum, one bf16 rounding."""
    T, world = pos.shape
    acc = torch.zeros(T, H, dtype=torch.float32, device=back.device)
    for d in range(world):
        p = pos[:, d]
        sel = torch.nonzero(p >= 0).flatten()
        if sel.numel():
            acc.index_copy_(0, sel, acc.index_select(0, sel) + back.index_select(0, p[sel]).to(torch.float32))
    return acc.to(torch.bfloat16)


class TorchExchangeMoE:
    """One rank of the expert-parallel layer with the exchange written in tensor ops and
    ``torch.distributed`` all-to-alls (any backend, gloo included); ``route_fn`` and
    ``experts_fn`` stand in for the CUDA routing and expert kernels."""

    def __init__(self, weights, local_expert_offset: int, num_local: int, route_fn: Callable,
                 experts_fn: Callable, group=None, combine_dtype: torch.dtype = torch.bfloat16):
        self.w = weights
        self.offset, self.num_local = int(local_expert_offset), int(num_local)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.num_local * self.world != E_GLOBAL or self.offset != self.rank * self.num_local:
            raise ValueError("expert-parallel shards must be equal, contiguous and in rank order")
        self.route_fn, self.experts_fn = route_fn, experts_fn
        self.combine_dtype = combine_dtype

    def forward(self, routing_logits, routing_bias, hidden_states, hidden_states_scale, routed_scaling_factor):
        T = routing_logits.shape[0]
        idx, w = self.route_fn(routing_logits, routing_bias, routed_scaling_factor)
        plan = dispatch_plan(idx, w, self.world)
        send = pack_rows(hidden_states, hidden_states_scale.contiguous(), plan)
        recv_counts = torch.empty_like(plan.send_counts)
        dist.all_to_all_single(recv_counts, plan.send_counts, group=self.group)
        s_split, r_split = plan.send_counts.tolist(), recv_counts.tolist()
        recv = torch.empty((sum(r_split), ROW_BYTES), dtype=torch.uint8, device=send.device)
        dist.all_to_all_single(recv, send, output_split_sizes=r_split, input_split_sizes=s_split, group=self.group)
        hid, sc, ids, ww = unpack_rows(recv)
        part = self.experts_fn(ids, ww, hid, sc, self.w.gemm1_weights, self.w.gemm1_weights_scale,
                               self.w.gemm2_weights, self.w.gemm2_weights_scale, self.offset,
                               out_dtype=self.combine_dtype)
        back = torch.empty((sum(s_split), H), dtype=part.dtype, device=part.device)
        dist.all_to_all_single(back, part.contiguous(), output_split_sizes=s_split, input_split_sizes=r_split,
                               group=self.group)
        return combine(back, plan.pos) if T else torch.empty((0, H), dtype=torch.bfloat16, device=back.device)
