"""The CUDA hidden-state quantiser (``kf_quantize_hidden``) against the oracle and the reference's vectors.

Integer/byte output: bit-exact e4m3 codes and bit-exact fp32 scales.
"""
import os

import numpy as np
import pytest
import torch

from kernelforge_b200 import binding as B
from kernelforge_b200 import synthetic as S
from oracle import moe_oracle as O
from tests.helpers import gpu_available, gpu_bank

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not gpu_available(), reason="needs a B200")]


def _check(x_cpu):
    q, s = B.quantize_hidden(x_cpu.cuda())
    torch.cuda.synchronize()
    q_ref, s_ref = O.quantize_rows_per_128(x_cpu)
    assert torch.equal(q.cpu().view(torch.uint8), q_ref.view(torch.uint8))
    assert torch.equal(s.cpu(), s_ref)


def test_reference_vectors_bit_exact():
    d = np.load(os.path.join(os.path.dirname(__file__), "golden", "quant_golden.npz"))
    x = torch.from_numpy(d["x_bits"].view(np.int16)).view(torch.bfloat16)
    q, s = B.quantize_hidden(x.cuda())
    assert torch.equal(q.cpu().view(torch.uint8), torch.from_numpy(d["q_bits"]))
    assert torch.equal(s.cpu(), torch.from_numpy(d["scale"]))


@pytest.mark.parametrize("T", [1, 7, 64, 4096])
def test_seeded_rows_bit_exact(T):
    g = torch.Generator().manual_seed(T)
    _check((torch.randn(T, B.H, generator=g) * 2.0).to(torch.bfloat16))


def test_empty_call():
    q, s = B.quantize_hidden(torch.empty((0, B.H), dtype=torch.bfloat16, device="cuda"))
    assert q.shape == (0, B.H) and s.shape == (56, 0)


def test_quantised_rows_feed_the_layer_unchanged():
    """bf16 rows -> kf_quantize_hidden -> kernel(...) equals the layer on the oracle-quantised rows."""
    T = 32
    g = torch.Generator().manual_seed(5)
    x = torch.randn(T, B.H, generator=g).to(torch.bfloat16)
    ti = S.token_inputs(T, seed=5)
    wb = gpu_bank(32, 0)
    q, s = B.quantize_hidden(x.cuda())
    q_ref, s_ref = O.quantize_rows_per_128(x)
    args = (ti.routing_logits.cuda(), ti.routing_bias.cuda())
    w = (wb.gemm1_weights, wb.gemm1_weights_scale, wb.gemm2_weights, wb.gemm2_weights_scale, 0, 2.5)
    out = B.kernel(*args, q, s, *w)
    ref = B.kernel(*args, q_ref.cuda(), s_ref.cuda(), *w)
    assert torch.equal(out, ref)
