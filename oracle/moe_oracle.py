"""CPU oracle for the DeepSeek-V3 FP8 block-scale MoE layer -- TEST INFRASTRUCTURE.

This module is a plain PyTorch (CPU, fp32) restatement of the reference's
algorithm for ``kernel(...)``.  It is the checker for the CUDA path: only the
tests, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl
reference`` legs of ``bench.py`` may import it.  The product path never calls it.

Reference (chinmay29/kernelforge), all in ``solution/triton/kernel.py``:

* routing ............ ``kernel`` lines 1842-1867 (same math as
  ``_route_topk_ids_and_weights`` lines 967-993)
* token sort ......... ``_sort_tokens`` lines 46-82
* dequantisation ..... ``_dequant_hidden_rows`` 85-90, ``_dequant_gemm1_weight``
  93-100, ``_dequant_gemm2_weight`` 118-123
* expert loop ........ ``kernel`` lines 1927-1950 (the per-expert PyTorch path
  that runs with ``KF_USE_GROUPED_TRITON=0``)
* SwiGLU ............. ``silu(X2) * X1`` with X1 = W13 rows [0, I) and X2 = rows
  [I, 2I) (lines 1940-1943)
* row quantisation ... ``_quantize_fp8_block_rows`` lines 126-141 (the FP8
  format of ``hidden_states`` / ``hidden_states_scale``: per row and 128
  columns, scale = absmax / 448, or 1 for an all-zero block)

Pinning: ``tests/golden/make_golden.py`` imports the reference ``kernel`` in the
build container and records its outputs on seeded inputs; ``tests/test_oracle.py``
checks this restatement against those fixtures.
"""
from __future__ import annotations

import torch

H = 7168
I = 2048
E_GLOBAL = 256
BLOCK = 128
TOP_K = 8
N_GROUP = 8
TOPK_GROUP = 4
GROUP_SIZE = E_GLOBAL // N_GROUP


def route(routing_logits: torch.Tensor, routing_bias: torch.Tensor, routed_scaling_factor: float):
    """DeepSeek-V3 grouped sigmoid routing (reference ``kernel.py:1842-1867``).

    Returns ``(topk_idx [T, 8] int64, weights [T, 256] f32)``.  ``topk_idx`` is in
    torch.topk's (unspecified) order; compare index *sets*.  ``weights`` is the
    dense matrix the reference indexes with ``weights[token, global_expert]``.
    """
    T = routing_logits.shape[0]
    s = torch.sigmoid(routing_logits.to(torch.float32))
    sb = s + routing_bias.to(torch.float32).reshape(-1)
    # group score = sum of the two largest biased scores in each group of 32
    top2, _ = torch.topk(sb.view(T, N_GROUP, GROUP_SIZE), k=2, dim=2, largest=True, sorted=False)
    gscore = top2.sum(dim=2)
    _, gidx = torch.topk(gscore, k=TOPK_GROUP, dim=1, largest=True, sorted=False)
    keep_group = torch.zeros_like(gscore).scatter_(1, gidx, 1.0)
    keep = keep_group.unsqueeze(2).expand(T, N_GROUP, GROUP_SIZE).reshape(T, E_GLOBAL)
    pruned = sb.masked_fill(keep == 0, torch.finfo(torch.float32).min)
    _, topk_idx = torch.topk(pruned, k=TOP_K, dim=1, largest=True, sorted=False)
    # weights use the un-biased sigmoid, normalised over the selection
    sel = torch.zeros_like(s).scatter_(1, topk_idx, 1.0)
    w = s * sel
    w = (w / (w.sum(dim=1, keepdim=True) + 1e-20)) * float(routed_scaling_factor)
    return topk_idx, w


def route_scores(routing_logits: torch.Tensor, routing_bias: torch.Tensor):
    """The biased scores and group scores the selection is made on (for tie analysis)."""
    T = routing_logits.shape[0]
    s = torch.sigmoid(routing_logits.to(torch.float32))
    sb = s + routing_bias.to(torch.float32).reshape(-1)
    top2, _ = torch.topk(sb.view(T, N_GROUP, GROUP_SIZE), k=2, dim=2)
    return sb, top2.sum(dim=2)


def sort_tokens(topk_idx: torch.Tensor, local_start: int, num_local: int):
    """Local (token, expert) pairs stably sorted by local expert (``kernel.py:46-82``).

    Returns ``(sorted_ids, sorted_local_experts, expert_starts, counts)`` as int64.
    """
    T, K = topk_idx.shape
    local = topk_idx.to(torch.int64) - int(local_start)
    valid = ((local >= 0) & (local < num_local)).reshape(-1)
    tok = torch.arange(T, dtype=torch.int64, device=topk_idx.device).unsqueeze(1).expand(T, K).reshape(-1)[valid]
    le = local.reshape(-1)[valid]
    order = torch.argsort(le, stable=True)
    sorted_ids = tok[order]
    sorted_le = le[order]
    counts = torch.bincount(sorted_le, minlength=num_local)
    starts = torch.zeros(num_local, dtype=torch.int64, device=topk_idx.device)
    if num_local > 1:
        starts[1:] = torch.cumsum(counts, 0)[:-1]
    return sorted_ids, sorted_le, starts, counts


def quantize_rows_per_128(x: torch.Tensor):
    """``kernel.py:126-141``: ``[R, K]`` -> e4m3 ``[R, K]`` and fp32 scales ``[K/128, R]``.

    absmax over each 128-wide block; scale = absmax / 448 (1 where absmax is 0);
    q = e4m3(x / scale) with torch's round-to-nearest cast.
    """
    r, k = x.shape
    blocks = x.to(torch.float32).view(r, k // BLOCK, BLOCK)
    absmax = blocks.abs().amax(dim=2)
    scale = torch.where(absmax > 0, absmax / torch.finfo(torch.float8_e4m3fn).max, torch.ones_like(absmax))
    q = (blocks / scale.unsqueeze(-1)).to(torch.float8_e4m3fn).reshape(r, k)
    return q.contiguous(), scale.t().contiguous()


def dequant_hidden_rows(hidden_states, hidden_states_scale, token_ids):
    """``kernel.py:85-90``: fp8 rows times their per-128 scale (scales are ``[56, T]``)."""
    x = hidden_states.index_select(0, token_ids).to(torch.float32)
    sc = hidden_states_scale.index_select(1, token_ids).to(torch.float32).t()
    return (x.view(-1, H // BLOCK, BLOCK) * sc.unsqueeze(-1)).reshape(-1, H)


def dequant_block_weight(w_fp8: torch.Tensor, w_scale: torch.Tensor):
    """``kernel.py:93-100`` / ``118-123``: expand a ``[R/128, C/128]`` scale grid."""
    w = w_fp8.to(torch.float32)
    sc = w_scale.to(torch.float32).repeat_interleave(BLOCK, 0).repeat_interleave(BLOCK, 1)
    return w * sc


def expert_forward(hidden_rows_f32, w13_fp8, w13_scale, w2_fp8, w2_scale):
    """One expert on already-dequantised rows: GEMM1, SwiGLU, GEMM2 (``kernel.py:1939-1946``)."""
    w13 = dequant_block_weight(w13_fp8, w13_scale)
    g1 = hidden_rows_f32.matmul(w13.t())
    x1, x2 = g1[:, :I], g1[:, I:]
    act = torch.nn.functional.silu(x2) * x1
    w2 = dequant_block_weight(w2_fp8, w2_scale)
    return act.matmul(w2.t())


def moe_layer(routing_logits, routing_bias, hidden_states, hidden_states_scale,
              gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
              local_expert_offset, routed_scaling_factor, *, return_routing: bool = False):
    """The whole layer, value-returning like the reference ``kernel`` (``kernel.py:1817-1950``).

    Output: bf16 ``[T, 7168]``.  The number of local experts comes from the weight
    shape (the reference fixes it at 32; expert-parallel shards use 32..256).
    Runs on the inputs' device: on CPU it is the oracle, on a GPU the tests use
    the same fp32 code as a full-size reference.
    """
    if isinstance(local_expert_offset, torch.Tensor):
        local_expert_offset = int(local_expert_offset.item())
    if isinstance(routed_scaling_factor, torch.Tensor):
        routed_scaling_factor = float(routed_scaling_factor.item())
    T = routing_logits.shape[0]
    E = gemm1_weights.shape[0]
    topk_idx, weights = route(routing_logits, routing_bias, routed_scaling_factor)
    sorted_ids, _, starts, counts = sort_tokens(topk_idx, local_expert_offset, E)
    acc = torch.zeros(T, H, dtype=torch.float32, device=routing_logits.device)
    for e in torch.nonzero(counts > 0).flatten().tolist():
        tok = sorted_ids[int(starts[e]): int(starts[e]) + int(counts[e])]
        rows = dequant_hidden_rows(hidden_states, hidden_states_scale, tok)
        y = expert_forward(rows, gemm1_weights[e], gemm1_weights_scale[e],
                           gemm2_weights[e], gemm2_weights_scale[e])
        rw = weights[tok, int(local_expert_offset) + e]
        acc.index_add_(0, tok, y * rw.unsqueeze(1))
    out = acc.to(torch.bfloat16)
    if return_routing:
        return out, topk_idx, weights
    return out


def moe_experts(topk_idx, topk_weight, hidden_states, hidden_states_scale, gemm1_weights,
                gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset):
    """Experts on pre-routed rows, fp32 ``[T, 7168]`` (the expert-parallel receive side).

    ``topk_idx`` holds global expert ids or -1; ids outside the local range are
    skipped.  Per expert the math is the reference loop (``kernel.py:1927-1950``)
    with the routing weight taken from ``topk_weight``; experts are accumulated
    in ascending order, as ``index_add_`` over the expert-sorted pairs does.
    """
    T = hidden_states.shape[0]
    E = gemm1_weights.shape[0]
    loc = topk_idx.to(torch.int64) - int(local_expert_offset)
    valid = (topk_idx >= 0) & (loc >= 0) & (loc < E)
    acc = torch.zeros(T, H, dtype=torch.float32, device=hidden_states.device)
    for e in sorted(set(loc[valid].tolist())):
        m = valid & (loc == e)
        tok = torch.nonzero(m.any(dim=1)).flatten()
        rw = (topk_weight.to(torch.float32) * m).sum(dim=1)[tok]
        rows = dequant_hidden_rows(hidden_states, hidden_states_scale, tok)
        y = expert_forward(rows, gemm1_weights[e], gemm1_weights_scale[e],
                           gemm2_weights[e], gemm2_weights_scale[e])
        acc.index_add_(0, tok, y * rw.unsqueeze(1))
    return acc


def active_local_experts(routing_logits, routing_bias, local_expert_offset: int, num_local: int):
    """Local expert ids that receive at least one token (lets tests skip the rest)."""
    idx, _ = route(routing_logits, routing_bias, 1.0)
    loc = idx - int(local_expert_offset)
    loc = loc[(loc >= 0) & (loc < num_local)]
    return sorted(set(loc.tolist()))


def check_tolerance(out: torch.Tensor, ref: torch.Tensor, *, atol=1e-2, rtol=2e-2,
                    max_rel=1e-2, frac=0.999) -> dict:
    """The layer's acceptance test on bf16 outputs.

    Passes when max|out-ref| <= ``max_rel``*max|ref| and at least ``frac`` of
    the elements satisfy |out-ref| <= atol + rtol*|ref|.
    """
    o = out.to(torch.float32).cpu()
    r = ref.to(torch.float32).cpu()
    d = (o - r).abs()
    ref_max = float(r.abs().max()) if r.numel() else 0.0
    max_err = float(d.max()) if d.numel() else 0.0
    within = (d <= atol + rtol * r.abs())
    frac_ok = float(within.float().mean()) if d.numel() else 1.0
    ok = (max_err <= max_rel * ref_max or max_err == 0.0) and frac_ok >= frac and bool(torch.isfinite(o).all())
    return {"ok": ok, "max_abs_err": max_err, "max_abs_ref": ref_max, "frac_within": frac_ok}
