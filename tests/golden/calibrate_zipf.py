"""Calibrate the Zipf routing-bias strength used by the skewed-load workload.

``kernelforge_b200.synthetic.zipf_bias`` sets bias_e = -beta * ln(rank(e)) over a
seeded permutation of the 256 experts.  This script sweeps beta, routes N(0,1)
logits with the oracle's routing restatement and reports the beta whose sorted
expert-selection histogram is closest (L1) to Zipf(s).  The chosen value is
hard-coded as ``synthetic.ZIPF_BETA``.

    python tests/golden/calibrate_zipf.py [s] [T]
"""
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from kernelforge_b200 import synthetic as S  # noqa: E402
from oracle.moe_oracle import route  # noqa: E402


def calibrate(s=1.2, T=4096, seed=0, betas=None):
    logits = torch.randn(T, S.E_GLOBAL, generator=torch.Generator().manual_seed(seed))
    target = torch.tensor([1.0 / (r ** s) for r in range(1, S.E_GLOBAL + 1)])
    target = target / target.sum()
    best = (float("inf"), None, None)
    for beta in (betas or [0.01 * i for i in range(1, 61)]):
        idx, _ = route(logits, S.zipf_bias(seed, s, beta), 1.0)
        hist = torch.bincount(idx.reshape(-1), minlength=S.E_GLOBAL).float()
        hist = hist.sort(descending=True).values / hist.sum()
        gap = float((hist - target).abs().sum())
        if gap < best[0]:
            best = (gap, beta, hist)
    return best


if __name__ == "__main__":
    s = float(sys.argv[1]) if len(sys.argv) > 1 else 1.2
    T = int(sys.argv[2]) if len(sys.argv) > 2 else 4096
    gap, beta, hist = calibrate(s, T)
    print(f"beta={beta:.3f} L1 gap={gap:.3f}")
    print("top-10 share:", [round(float(h), 4) for h in hist[:10]])
    print("experts with <0.05% of selections:", int((hist < 5e-4).sum()))
