"""Golden vectors for the hidden-state FP8 quantiser, from the REFERENCE function.

Run where a checkout of the reference (chinmay29/kernelforge) is available; it
imports ``_quantize_fp8_block_rows`` (``solution/triton/kernel.py`` lines 126-141)
from that checkout and runs it on CPU:

    python tests/golden/make_quant_golden.py <reference checkout>

Writes ``tests/golden/quant_golden.npz``: bf16 inputs (as uint16 bits), the
reference's e4m3 output (as uint8 bits) and its ``[56, R]`` fp32 scales, for
seeded rows plus edge rows: an all-zero row, a row with a single non-zero per
block, tiny magnitudes, one large spike per block, exact powers of two and
negative-only blocks.
"""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF_KERNEL = os.path.join(sys.argv[1] if len(sys.argv) > 1 else ".", "solution", "triton", "kernel.py")
H = 7168


def inputs() -> torch.Tensor:
    g = torch.Generator().manual_seed(123)
    rows = [torch.randn(6, H, generator=g) * 3.0]
    rows.append(torch.zeros(1, H))                                   # all-zero blocks -> scale 1
    one = torch.zeros(1, H)
    one[0, ::128] = torch.linspace(-5, 5, H // 128)                  # one non-zero per block (some zero)
    rows.append(one)
    rows.append(torch.randn(1, H, generator=g) * 1e-30)              # tiny magnitudes
    spike = torch.randn(1, H, generator=g) * 0.01
    spike[0, 7::128] = 1e4                                           # one spike per block
    rows.append(spike)
    rows.append(torch.full((1, H), 2.0) ** torch.randint(-20, 20, (1, H), generator=g).float())
    rows.append(-torch.rand(1, H, generator=g) * 100)                # negative only
    return torch.cat(rows).to(torch.bfloat16)


def main():
    spec = importlib.util.spec_from_file_location("ref_kernel", REF_KERNEL)
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    x = inputs()
    q, scale = ref._quantize_fp8_block_rows(x.to(torch.float32))
    np.savez_compressed(os.path.join(HERE, "quant_golden.npz"),
                        x_bits=x.view(torch.int16).numpy().view(np.uint16),
                        q_bits=q.view(torch.uint8).numpy(), scale=scale.numpy())
    print("rows", x.shape[0], "scale shape", tuple(scale.shape))


if __name__ == "__main__":
    main()
