"""CUDA-graph replay of the layer (decode): the same bits as direct calls, and within the
layer's tolerance of the fp32 reference at every captured size."""
import pytest
import torch

from kernelforge_b200 import binding as B
from kernelforge_b200 import synthetic as S
from kernelforge_b200.graph import GraphedMoE
from oracle import moe_oracle as O
from tests.helpers import compare_routing, gpu_available, gpu_bank, to_cuda

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not gpu_available(), reason="needs a B200")]


@pytest.mark.parametrize("T", [1, 16, 48])
def test_graph_replay_matches_direct_calls_and_reference(T):
    wb = gpu_bank(32, 0, seed=12)
    layer = GraphedMoE(wb, 0, 2.5, T).capture()
    for seed in (40, 41):  # two replays with different inputs
        ti = to_cuda(S.token_inputs(T, seed=seed))
        ref = B.kernel(ti.routing_logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale,
                       wb.gemm1_weights, wb.gemm1_weights_scale, wb.gemm2_weights, wb.gemm2_weights_scale, 0, 2.5)
        out = layer(ti.routing_logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale).clone()
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        idx, w = B.route(ti.routing_logits, ti.routing_bias, 2.5)
        hard, ties, _ = compare_routing(idx, w, ti.routing_logits, ti.routing_bias, 2.5)
        assert hard == 0 and ties == 0
        f32 = O.moe_experts(idx, w, ti.hidden_states, ti.hidden_states_scale, wb.gemm1_weights,
                            wb.gemm1_weights_scale, wb.gemm2_weights, wb.gemm2_weights_scale, 0)
        res = O.check_tolerance(out, f32.to(torch.bfloat16))
        assert res["ok"], res
