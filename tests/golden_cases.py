"""Loaders for the committed golden fixtures (made by tests/golden/make_golden.py)."""
import hashlib
import os

import numpy as np
import torch

from kernelforge_b200 import synthetic as S

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().reshape(-1).view(torch.uint8).numpy().tobytes()).hexdigest()


def _group(npz, prefix):
    return {k.split("/", 1)[1]: npz[k] for k in npz.files if k.startswith(prefix + "/")}


def layer_cases():
    npz = np.load(os.path.join(GOLDEN, "moe_golden.npz"))
    names = sorted({k.split("/")[0] for k in npz.files})
    return {n: _group(npz, n) for n in names}


def routing_cases():
    npz = np.load(os.path.join(GOLDEN, "routing_golden.npz"))
    names = sorted({k.split("/")[0] for k in npz.files})
    return {n: _group(npz, n) for n in names}


def layer_inputs(case, num_local=32):
    """Regenerate the inputs of a golden layer case (CPU), checking their digests."""
    T, seed, offset, zipf = [int(v) for v in case["meta"]]
    bias = S.zipf_bias(seed) if zipf else None
    ti = S.token_inputs(T, seed, routing_bias=bias)
    active = [int(e) for e in case["active"]]
    wb = S.expert_bank(num_local, offset, seed=0, only=active)
    digests = [sha(ti.routing_logits), sha(ti.routing_bias), sha(ti.hidden_states), sha(ti.hidden_states_scale)]
    for e in active:
        digests += [sha(wb.gemm1_weights[e]), sha(wb.gemm2_weights[e])]
    assert list(case["sha"]) == digests, "seeded input generator drifted from the golden fixture"
    return ti, wb, offset, float(case["rsf"][0])


def routing_inputs(case):
    T, seed, zipf = [int(v) for v in case["meta"]]
    bias = S.zipf_bias(seed) if zipf else None
    ti = S.token_inputs(T, seed, routing_bias=bias)
    assert list(case["sha"]) == [sha(ti.routing_logits), sha(ti.routing_bias)]
    return ti
