"""Seeded synthetic inputs for the DeepSeek-V3 FP8 block-scale MoE layer.

The contest dataset (``flashinfer-ai/mlsys26-contest``) is not available offline,
so every test, the smoke check and the benchmark use these generators.  They
follow the workload description of the layer
(``moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048``):

* ``routing_logits``  fp32 N(0, 1)                        ``[T, 256]``
* ``routing_bias``    bf16 N(0, 0.02)                     ``[256]``
* ``hidden_states``   bf16 N(0, 1) quantised to e4m3 with one fp32 scale per
  token and 128 columns (absmax / 448), scales stored K-block-major ``[56, T]``
  (the layout the reference reads at ``solution/triton/kernel.py:85-90``)
* ``gemm1_weights``   N(0, 0.02) ``[E, 4096, 7168]``, 128x128 block scales ``[E, 32, 56]``
* ``gemm2_weights``   N(0, 0.02) ``[E, 7168, 2048]``, 128x128 block scales ``[E, 56, 16]``

Token tensors come from one ``torch.Generator`` seeded with ``seed``.  Each
expert's weights come from their own generator keyed by the *global* expert id,
so an expert-parallel rank, a single GPU holding all 256 experts and a CPU test
that materialises only the experts a few tokens touch all see identical weights.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Iterable, Optional

import torch

H = 7168
I = 2048
E_GLOBAL = 256
BLOCK = 128
TOP_K = 8
N_GROUP = 8
TOPK_GROUP = 4
FP8_MAX = 448.0

_EXPERT_SEED_STRIDE = 1_000_003


def _quantize_blocks_2d(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantise a ``[R, C]`` fp32 matrix to e4m3 with one scale per 128x128 block."""
    r, c = w.shape
    blocks = w.view(r // BLOCK, BLOCK, c // BLOCK, BLOCK)
    absmax = blocks.abs().amax(dim=(1, 3))
    scale = torch.where(absmax > 0, absmax / FP8_MAX, torch.ones_like(absmax))
    q = (blocks / scale[:, None, :, None]).to(torch.float8_e4m3fn).view(r, c)
    return q, scale.to(torch.float32)


def quantize_rows_per_128(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantise ``[T, K]`` rows to e4m3 with one scale per row and 128 columns.

    Returns the fp8 tensor ``[T, K]`` and the scales K-block-major ``[K/128, T]``.
    """
    t, k = x.shape
    blocks = x.to(torch.float32).view(t, k // BLOCK, BLOCK)
    absmax = blocks.abs().amax(dim=2)
    scale = torch.where(absmax > 0, absmax / FP8_MAX, torch.ones_like(absmax))
    q = (blocks / scale[:, :, None]).to(torch.float8_e4m3fn).view(t, k)
    return q, scale.t().contiguous()


def expert_weights(global_expert: int, seed: int = 0, device="cpu"):
    """W13/W2 (fp8) and their block scales for one expert, keyed by global id."""
    g = torch.Generator(device=device).manual_seed(seed * _EXPERT_SEED_STRIDE + 1 + int(global_expert))
    w13 = torch.randn(2 * I, H, generator=g, device=device, dtype=torch.float32).mul_(0.02)
    w13_q, w13_s = _quantize_blocks_2d(w13)
    del w13
    w2 = torch.randn(H, I, generator=g, device=device, dtype=torch.float32).mul_(0.02)
    w2_q, w2_s = _quantize_blocks_2d(w2)
    return w13_q, w13_s, w2_q, w2_s


@dataclass
class TokenInputs:
    routing_logits: torch.Tensor       # [T, 256] f32
    routing_bias: torch.Tensor         # [256] bf16
    hidden_states: torch.Tensor        # [T, 7168] e4m3
    hidden_states_scale: torch.Tensor  # [56, T] f32


def token_inputs(T: int, seed: int = 0, device="cpu", routing_bias: Optional[torch.Tensor] = None) -> TokenInputs:
    g = torch.Generator(device=device).manual_seed(seed)
    logits = torch.randn(T, E_GLOBAL, generator=g, device=device, dtype=torch.float32)
    bias = (torch.randn(E_GLOBAL, generator=g, device=device, dtype=torch.float32) * 0.02).to(torch.bfloat16)
    if routing_bias is not None:
        bias = routing_bias.to(device=device, dtype=torch.bfloat16)
    hid = torch.randn(T, H, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
    hq, hs = quantize_rows_per_128(hid)
    return TokenInputs(logits, bias, hq, hs)


@dataclass
class ExpertWeights:
    gemm1_weights: torch.Tensor        # [E, 4096, 7168] e4m3
    gemm1_weights_scale: torch.Tensor  # [E, 32, 56] f32
    gemm2_weights: torch.Tensor        # [E, 7168, 2048] e4m3
    gemm2_weights_scale: torch.Tensor  # [E, 56, 16] f32


def expert_bank(num_local: int, local_offset: int, seed: int = 0, device="cpu",
                only: Optional[Iterable[int]] = None) -> ExpertWeights:
    """Weights for local experts ``[offset, offset+num_local)``.

    With ``only`` (local expert ids), the other experts are left as zeros so a
    CPU test can skip generating experts no token is routed to.
    """
    keep = set(range(num_local)) if only is None else set(int(e) for e in only)
    w13 = torch.zeros(num_local, 2 * I, H, dtype=torch.float8_e4m3fn, device=device)
    w13s = torch.ones(num_local, 2 * I // BLOCK, H // BLOCK, dtype=torch.float32, device=device)
    w2 = torch.zeros(num_local, H, I, dtype=torch.float8_e4m3fn, device=device)
    w2s = torch.ones(num_local, H // BLOCK, I // BLOCK, dtype=torch.float32, device=device)
    for e in sorted(keep):
        a, b, c, d = expert_weights(local_offset + e, seed, device)
        w13[e].copy_(a); w13s[e].copy_(b); w2[e].copy_(c); w2s[e].copy_(d)
    return ExpertWeights(w13, w13s, w2, w2s)


def zipf_bias(seed: int = 0, s: float = 1.2, beta: Optional[float] = None) -> torch.Tensor:
    """Routing bias that skews expert popularity towards a Zipf(s) profile.

    bias_e = -beta * ln(rank(e)) over a seeded permutation of the 256 experts.
    ``beta`` defaults to a fixed value picked so that with N(0,1) logits the
    selection histogram roughly follows Zipf(1.2) (calibrated by
    ``tests/golden/calibrate_zipf.py``).
    """
    g = torch.Generator().manual_seed(seed + 7919)
    perm = torch.randperm(E_GLOBAL, generator=g)
    rank = torch.empty(E_GLOBAL, dtype=torch.float32)
    rank[perm] = torch.arange(1, E_GLOBAL + 1, dtype=torch.float32)
    if beta is None:
        beta = ZIPF_BETA
    return (-beta * torch.log(rank)).to(torch.bfloat16)


# Calibrated by tests/golden/calibrate_zipf.py (s=1.2, 4096 tokens, seed 0).
ZIPF_BETA = 0.11

