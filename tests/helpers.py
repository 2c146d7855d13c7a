"""Shared test helpers: GPU input banks, routing comparison with tie analysis."""
from __future__ import annotations

import numpy as np
import torch

from kernelforge_b200 import synthetic as S
from oracle import moe_oracle as O


def gpu_available() -> bool:
    return torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0)


def gpu_bank(num_local: int, offset: int, seed: int = 0):
    """All local experts generated directly on the GPU (values differ from the CPU
    generator's but follow the same distributions; used with the GPU fp32 reference)."""
    return S.expert_bank(num_local, offset, seed=seed, device="cuda")


def to_cuda(ti: S.TokenInputs) -> S.TokenInputs:
    return S.TokenInputs(*(t.cuda() for t in (ti.routing_logits, ti.routing_bias, ti.hidden_states,
                                               ti.hidden_states_scale)))


def f32_ulp(x: float) -> float:
    return float(np.spacing(np.float32(abs(x))))


def compare_routing(gpu_idx: torch.Tensor, gpu_w: torch.Tensor, logits: torch.Tensor, bias: torch.Tensor,
                    rsf: float, ulps: int = 4):
    """Compare kernel routing with the oracle's.

    Returns ``(hard_mismatches, near_ties, max_rel_weight_err)``.  A token whose
    index set differs counts as a near tie (allowed, reported) only when every
    swapped pair of experts is within ``ulps`` float32 ulps of each other in the
    biased score, or their groups are within ``ulps`` ulps in group score: the
    GPU sigmoid may differ from the CPU one by an ulp, which can flip such ties.
    """
    logits, bias = logits.float().cpu(), bias.cpu()
    ref_idx, ref_w = O.route(logits, bias, rsf)
    g = gpu_idx.long().cpu().sort(dim=1).values
    r = ref_idx.sort(dim=1).values
    sb, gs = O.route_scores(logits, bias)
    mism = (g != r).any(dim=1)
    hard, ties = 0, 0
    for t in torch.nonzero(mism).flatten().tolist():
        a = sorted(set(g[t].tolist()) - set(r[t].tolist()))
        b = sorted(set(r[t].tolist()) - set(g[t].tolist()))
        ok = len(a) == len(b)
        for x in a:
            near = False
            for y in b:
                vx, vy = float(sb[t, x]), float(sb[t, y])
                gx, gy = float(gs[t, x // 32]), float(gs[t, y // 32])
                if abs(vx - vy) <= ulps * max(f32_ulp(vx), f32_ulp(vy)) or \
                        abs(gx - gy) <= ulps * max(f32_ulp(gx), f32_ulp(gy)):
                    near = True
            ok = ok and near
        if ok:
            ties += 1
        else:
            hard += 1
    good = ~mism
    gi = gpu_idx.long().cpu()[good]
    gw = gpu_w.float().cpu()[good]
    rw = torch.gather(ref_w[good], 1, gi)
    rel = ((gw - rw).abs() / rw.abs().clamp_min(1e-30)).max().item() if gi.numel() else 0.0
    return hard, ties, rel
