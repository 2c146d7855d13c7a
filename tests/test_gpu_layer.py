"""Parity of the CUDA layer (through the C ABI) with the oracle and the reference goldens.

Acceptance (the layer's contract): routing index sets bit-exact (no token may
differ, not even on a near tie of a few float32 ulps), bf16 output with
max|out-ref| <= 1e-2 * max|ref| and >= 99.9% of elements within
atol 1e-2 + rtol 2e-2 * |ref|.
"""
import numpy as np
import pytest
import torch

from kernelforge_b200 import binding as B
from kernelforge_b200 import synthetic as S
from oracle import moe_oracle as O
from tests.golden_cases import layer_cases, layer_inputs, routing_cases, routing_inputs
from tests.helpers import compare_routing, gpu_available, gpu_bank, to_cuda

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not gpu_available(), reason="needs a B200")]

LAYER = layer_cases()
ROUTING = routing_cases()


def _run(ti, wb, offset, rsf, **kw):
    out = B.kernel(ti.routing_logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale,
                   wb.gemm1_weights, wb.gemm1_weights_scale, wb.gemm2_weights, wb.gemm2_weights_scale,
                   offset, rsf)
    torch.cuda.synchronize()
    assert B.read_status() == 0, "device status word set"
    return out


def _gpu_ref(ti, wb, offset, rsf):
    """fp32 reference on the GPU (the oracle's expert math on cuda tensors).

    Routing is checked against the CPU oracle first; the expert math then uses
    the kernel's (verified) routing, so a near tie that a different sigmoid
    implementation would flip cannot swap a whole expert between the two sides.
    """
    idx, w = B.route(ti.routing_logits, ti.routing_bias, rsf)
    hard, ties, rel = compare_routing(idx, w, ti.routing_logits, ti.routing_bias, rsf)
    assert hard == 0 and ties == 0 and rel < 2e-6
    ref = O.moe_experts(idx, w, ti.hidden_states, ti.hidden_states_scale, wb.gemm1_weights,
                        wb.gemm1_weights_scale, wb.gemm2_weights, wb.gemm2_weights_scale, offset)
    return ref.to(torch.bfloat16)


@pytest.mark.parametrize("name", sorted(ROUTING))
def test_routing_matches_reference_golden(name):
    case = ROUTING[name]
    ti = routing_inputs(case)
    idx, w = B.route(ti.routing_logits.cuda(), ti.routing_bias.cuda(), 2.5)
    hard, ties, rel = compare_routing(idx, w, ti.routing_logits, ti.routing_bias, 2.5)
    assert hard == 0 and ties == 0
    # the golden index sets are the reference's own
    g = idx.long().cpu().sort(dim=1).values.numpy()
    diff = (g != case["topk_sorted"].astype(np.int64)).any(axis=1).sum()
    assert diff == 0
    assert rel < 2e-6


@pytest.mark.parametrize("T", [1, 5, 128, 129, 1000, 16384])
def test_routing_random_sizes(T):
    ti = S.token_inputs(T, seed=100 + T)
    idx, w = B.route(ti.routing_logits.cuda(), ti.routing_bias.cuda(), 2.5)
    hard, ties, rel = compare_routing(idx, w, ti.routing_logits, ti.routing_bias, 2.5)
    assert hard == 0 and ties == 0 and rel < 2e-6
    # distinct experts per token, drawn from at most 4 groups
    srt = idx.long().cpu().sort(dim=1).values
    assert (srt[:, 1:] != srt[:, :-1]).all()
    groups = torch.zeros(T, 8).scatter_(1, srt // 32, 1.0).sum(dim=1)
    assert (groups <= 4).all()


@pytest.mark.parametrize("name", sorted(LAYER))
def test_layer_matches_reference_golden(name):
    case = LAYER[name]
    ti, wb, offset, rsf = layer_inputs(case)
    ti = to_cuda(ti)
    wb = S.ExpertWeights(*(t.cuda() for t in (wb.gemm1_weights, wb.gemm1_weights_scale, wb.gemm2_weights,
                                               wb.gemm2_weights_scale)))
    out = _run(ti, wb, offset, rsf)
    ref = torch.from_numpy(case["out_bf16"]).view(torch.bfloat16)
    res = O.check_tolerance(out, ref)
    assert res["ok"], res
    # the reference passed a 0-d tensor offset / scale: both forms are accepted
    out2 = B.kernel(ti.routing_logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale,
                    wb.gemm1_weights, wb.gemm1_weights_scale, wb.gemm2_weights, wb.gemm2_weights_scale,
                    torch.tensor(offset, dtype=torch.int32), torch.tensor(rsf))
    assert torch.equal(out, out2)


@pytest.mark.parametrize("T,offset,num_local", [(64, 0, 32), (300, 96, 32), (1024, 0, 32), (4096, 0, 32),
                                                (512, 0, 256), (777, 128, 128)])
def test_layer_vs_fp32_reference(T, offset, num_local):
    ti = to_cuda(S.token_inputs(T, seed=7 + T))
    wb = gpu_bank(num_local, offset, seed=1)
    out = _run(ti, wb, offset, 2.5)
    ref = _gpu_ref(ti, wb, offset, 2.5)
    res = O.check_tolerance(out, ref)
    assert res["ok"], res


def test_layer_full_prefill_16384():
    T = 16384
    ti = to_cuda(S.token_inputs(T, seed=5))
    wb = gpu_bank(32, 0, seed=2)
    out = _run(ti, wb, 0, 2.5)
    ref = _gpu_ref(ti, wb, 0, 2.5)
    res = O.check_tolerance(out, ref)
    assert res["ok"], res


@pytest.fixture(scope="module")
def bank256():
    """All 256 experts on one GPU (11.3 GB): the expert bank of config 3's layer at N = 1."""
    return gpu_bank(256, 0, seed=0)


def _sampled_gpu_ref(ti, wb, offset, rsf, n_sample, seed):
    """fp32 reference of a seeded sample of the tokens (routing checked for every token)."""
    T = ti.routing_logits.shape[0]
    idx, w = B.route(ti.routing_logits, ti.routing_bias, rsf)
    hard, ties, rel = compare_routing(idx, w, ti.routing_logits, ti.routing_bias, rsf)
    assert hard == 0 and ties == 0 and rel < 2e-6
    g = torch.Generator().manual_seed(seed)
    sel = torch.randperm(T, generator=g)[:n_sample].sort().values.cuda()
    ref = O.moe_experts(idx[sel], w[sel], ti.hidden_states[sel], ti.hidden_states_scale[:, sel], wb.gemm1_weights,
                        wb.gemm1_weights_scale, wb.gemm2_weights, wb.gemm2_weights_scale, offset)
    return sel, ref.to(torch.bfloat16)


@pytest.mark.parametrize("T,zipf", [(8192, False), (128, True), (16384, True)])
def test_layer_256_experts_one_gpu_sampled(bank256, T, zipf):
    """Config 3's layer on one GPU (T = 8192 tokens, all 256 experts local: the bench's default
    workload) and config 4's Zipf(1.2)-skewed routing at 256 experts: the whole layer runs, 384
    seeded tokens of it are checked against the fp32 reference."""
    bias = S.zipf_bias(seed=0) if zipf else None
    ti = to_cuda(S.token_inputs(T, seed=17, routing_bias=bias))
    out = _run(ti, bank256, 0, 2.5)
    sel, ref = _sampled_gpu_ref(ti, bank256, 0, 2.5, min(T, 384), seed=T)
    res = O.check_tolerance(out[sel], ref)
    assert res["ok"], res


def test_skewed_single_expert_many_tiles():
    """Every token routed to expert 3 (and 7 others): 1000 pairs in one expert -> 8 row tiles."""
    T = 1000
    ti = S.token_inputs(T, seed=3)
    logits = ti.routing_logits.clone()
    logits[:, 3] = 8.0
    logits[:, 0:32] += 2.0
    ti = to_cuda(S.TokenInputs(logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale))
    wb = gpu_bank(32, 0, seed=3)
    out = _run(ti, wb, 0, 2.5)
    ref = _gpu_ref(ti, wb, 0, 2.5)
    res = O.check_tolerance(out, ref)
    assert res["ok"], res


@pytest.mark.parametrize("T", [8, 31, 32, 33])
def test_decode_sizes_with_one_full_expert_tile(T):
    """Calls of at most 32 tokens run the GEMMs' decode layouts (32-row A slots); every token routed
    to expert 3 fills its tile with T rows, the most those layouts hold (T = 33 is the general path)."""
    ti = S.token_inputs(T, seed=40 + T)
    logits = ti.routing_logits.clone()
    logits[:, 3] = 8.0
    logits[:, 0:32] += 2.0
    ti = to_cuda(S.TokenInputs(logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale))
    wb = gpu_bank(32, 0, seed=8)
    out = _run(ti, wb, 0, 2.5)
    ref = _gpu_ref(ti, wb, 0, 2.5)
    res = O.check_tolerance(out, ref)
    assert res["ok"], res


def test_zipf_skewed_load():
    T = 4096
    ti = to_cuda(S.token_inputs(T, seed=9, routing_bias=S.zipf_bias(9)))
    wb = gpu_bank(32, 0, seed=4)
    out = _run(ti, wb, 0, 2.5)
    ref = _gpu_ref(ti, wb, 0, 2.5)
    res = O.check_tolerance(out, ref)
    assert res["ok"], res


def test_empty_and_no_local_tokens():
    wb = gpu_bank(32, 0, seed=5)
    ti = to_cuda(S.token_inputs(0, seed=1))
    out = _run(ti, wb, 0, 2.5)
    assert out.shape == (0, 7168)
    # routing confined to experts >= 32: no local pairs -> zeros
    ti = S.token_inputs(17, seed=2)
    logits = ti.routing_logits.clone()
    logits[:, :32] = -20.0
    ti = to_cuda(S.TokenInputs(logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale))
    out = _run(ti, wb, 0, 2.5)
    assert torch.count_nonzero(out) == 0


def test_repeated_calls_are_deterministic_and_noncontiguous_inputs_accepted():
    T = 333
    ti = to_cuda(S.token_inputs(T, seed=11))
    wb = gpu_bank(32, 0, seed=6)
    a = _run(ti, wb, 0, 2.5)
    b = _run(ti, wb, 0, 2.5)
    assert torch.equal(a, b)
    hs_nc = ti.hidden_states_scale.t().contiguous().t()   # same values, transposed strides
    assert not hs_nc.is_contiguous()
    c = B.kernel(ti.routing_logits, ti.routing_bias, ti.hidden_states, hs_nc, wb.gemm1_weights,
                 wb.gemm1_weights_scale, wb.gemm2_weights, wb.gemm2_weights_scale, 0, 2.5)
    assert torch.equal(a, c)


def test_experts_entry_point_fp32_and_bf16():
    """kf_moe_experts on pre-routed rows with -1 and non-local ids (expert-parallel receive side)."""
    T, offset, E = 700, 64, 64
    g = torch.Generator().manual_seed(21)
    idx = torch.stack([torch.randperm(256, generator=g)[:8] for _ in range(T)]).to(torch.int32)
    idx[torch.rand(T, 8, generator=g) < 0.2] = -1
    w = torch.rand(T, 8, generator=g)
    ti = to_cuda(S.token_inputs(T, seed=22))
    wb = gpu_bank(E, offset, seed=7)
    out32 = B.experts(idx.cuda(), w.cuda(), ti.hidden_states, ti.hidden_states_scale, wb.gemm1_weights,
                      wb.gemm1_weights_scale, wb.gemm2_weights, wb.gemm2_weights_scale, offset,
                      out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert B.read_status() == 0
    ref = O.moe_experts(idx.cuda(), w.cuda(), ti.hidden_states, ti.hidden_states_scale, wb.gemm1_weights,
                        wb.gemm1_weights_scale, wb.gemm2_weights, wb.gemm2_weights_scale, offset)
    res = O.check_tolerance(out32.to(torch.bfloat16), ref.to(torch.bfloat16))
    assert res["ok"], res
    out16 = B.experts(idx.cuda(), w.cuda(), ti.hidden_states, ti.hidden_states_scale, wb.gemm1_weights,
                      wb.gemm1_weights_scale, wb.gemm2_weights, wb.gemm2_weights_scale, offset)
    assert torch.equal(out16, out32.to(torch.bfloat16))


def test_device_error_raises_on_the_next_call_and_on_check():
    """An expert id outside [0, 256) is skipped by the kernels' bounds checks, which set a status
    bit; the binding raises RuntimeError for it at the next call on the stream (and check() raises
    at once)."""
    T = 40
    ti = to_cuda(S.token_inputs(T, seed=23))
    wb = gpu_bank(32, 0, seed=9)
    idx, w = B.route(ti.routing_logits, ti.routing_bias, 2.5)
    bad = idx.clone()
    bad[3, 2] = 300
    B.experts(bad, w, ti.hidden_states, ti.hidden_states_scale, wb.gemm1_weights, wb.gemm1_weights_scale,
              wb.gemm2_weights, wb.gemm2_weights_scale, 0)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="expert id"):
        B.experts(idx, w, ti.hidden_states, ti.hidden_states_scale, wb.gemm1_weights, wb.gemm1_weights_scale,
                  wb.gemm2_weights, wb.gemm2_weights_scale, 0)
    B.experts(bad, w, ti.hidden_states, ti.hidden_states_scale, wb.gemm1_weights, wb.gemm1_weights_scale,
              wb.gemm2_weights, wb.gemm2_weights_scale, 0)
    with pytest.raises(RuntimeError, match="expert id"):
        B.check()
    B.check()           # read and cleared: a later clean call does not raise
    _run(ti, wb, 0, 2.5)
