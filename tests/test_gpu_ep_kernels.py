"""Expert-parallel CUDA plumbing on one GPU (ranks emulated): dispatch packing,
the packed-row experts entry point and the combine, each bit-exact against the
tensor-op restatement in kernelforge_b200.ep."""
import pytest
import torch

from kernelforge_b200 import binding as B
from kernelforge_b200 import ep
from kernelforge_b200 import synthetic as S
from tests.helpers import gpu_available, gpu_bank, to_cuda

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not gpu_available(), reason="needs a B200")]


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("T", [5, 300])
def test_dispatch_matches_restatement(world, T):
    ti = to_cuda(S.token_inputs(T, seed=70 + T))
    idx, w = B.route(ti.routing_logits, ti.routing_bias, 2.5)
    send, counts, pos = B.ep_dispatch(idx, w, ti.hidden_states, ti.hidden_states_scale, world)
    plan = ep.dispatch_plan(idx, w, world)
    ref_rows = ep.pack_rows(ti.hidden_states, ti.hidden_states_scale, plan)
    torch.cuda.synchronize()
    assert torch.equal(counts.cpu(), plan.send_counts.cpu())
    assert torch.equal(pos.long(), plan.pos)
    n = int(counts.sum())
    assert torch.equal(send[:n], ref_rows)


def test_experts_packed_matches_unpacked():
    world, r = 4, 1
    T = 200
    ti = to_cuda(S.token_inputs(T, seed=77))
    idx, w = B.route(ti.routing_logits, ti.routing_bias, 2.5)
    send, counts, _ = B.ep_dispatch(idx, w, ti.hidden_states, ti.hidden_states_scale, world)
    c = counts.tolist()
    rows = send[sum(c[:r]):sum(c[:r + 1])]
    E = 256 // world
    bank = gpu_bank(E, r * E, seed=9)
    out_p = B.experts_packed(rows, bank.gemm1_weights, bank.gemm1_weights_scale, bank.gemm2_weights,
                             bank.gemm2_weights_scale, r * E)
    hid, sc, ids, ww = ep.unpack_rows(rows)
    out_u = B.experts(ids, ww, hid, sc, bank.gemm1_weights, bank.gemm1_weights_scale, bank.gemm2_weights,
                      bank.gemm2_weights_scale, r * E)
    torch.cuda.synchronize()
    assert B.read_status() == 0
    assert torch.equal(out_p, out_u)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_combine_matches_restatement(dtype):
    world, T = 8, 300
    ti = to_cuda(S.token_inputs(T, seed=78))
    idx, w = B.route(ti.routing_logits, ti.routing_bias, 2.5)
    _, counts, pos = B.ep_dispatch(idx, w, ti.hidden_states, ti.hidden_states_scale, world)
    n = int(counts.sum())
    back = torch.randn(n, 7168, generator=torch.Generator(device="cuda").manual_seed(3), device="cuda").to(dtype)
    out = B.ep_combine(back, pos, world)
    ref = ep.combine(back, pos.long())
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
