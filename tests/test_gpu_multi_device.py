"""Calls whose tensors live on a GPU other than the current one, which the reference's operator
allows: the binding makes the tensors' device current for each library call."""
import pytest
import torch

from kernelforge_b200 import binding as B
from kernelforge_b200 import synthetic as S
from tests.helpers import gpu_available


def _two_b200s() -> bool:
    return gpu_available() and torch.cuda.device_count() >= 2 and torch.cuda.get_device_capability(1) == (10, 0)


pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not _two_b200s(), reason="needs two B200s")]


def test_layer_on_a_non_current_device_matches_the_current_one():
    T, E, offset = 300, 32, 0
    ti = S.token_inputs(T, seed=61)
    wb = S.expert_bank(E, offset, seed=61, device="cuda:0")
    outs = []
    for d in (0, 1):
        dev = torch.device("cuda", d)
        args = [t.to(dev) for t in (ti.routing_logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale,
                                     wb.gemm1_weights, wb.gemm1_weights_scale, wb.gemm2_weights,
                                     wb.gemm2_weights_scale)]
        with torch.cuda.device(0):          # device 0 stays current for both calls
            out = B.kernel(*args, offset, 2.5)
            idx, _ = B.route(args[0], args[1], 2.5)
        torch.cuda.synchronize(dev)
        assert out.device == dev and idx.device == dev
        assert B.read_status(dev) == 0
        outs.append((out.cpu(), idx.cpu()))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
