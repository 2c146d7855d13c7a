"""The CPU oracle against the reference's own outputs (golden fixtures)."""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from tests.golden_cases import layer_cases, layer_inputs, routing_cases, routing_inputs

LAYER = layer_cases()
ROUTING = routing_cases()


@pytest.mark.parametrize("name", sorted(LAYER))
def test_oracle_layer_matches_reference(name):
    case = LAYER[name]
    ti, wb, offset, rsf = layer_inputs(case)
    out, idx, w = O.moe_layer(ti.routing_logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale,
                              wb.gemm1_weights, wb.gemm1_weights_scale, wb.gemm2_weights,
                              wb.gemm2_weights_scale, offset, rsf, return_routing=True)
    ids_sorted, _ = idx.sort(dim=1)
    assert np.array_equal(ids_sorted.numpy(), case["topk_sorted"].astype(np.int64))
    assert np.array_equal(torch.gather(w, 1, ids_sorted).numpy(), case["topk_weights"])
    # the restatement performs the same fp32 operations in the same order: bit-exact
    assert np.array_equal(out.view(torch.int16).numpy(), case["out_bf16"])


@pytest.mark.parametrize("name", sorted(ROUTING))
def test_oracle_routing_matches_reference(name):
    case = ROUTING[name]
    ti = routing_inputs(case)
    idx, w = O.route(ti.routing_logits, ti.routing_bias, 2.5)
    ids_sorted, _ = idx.sort(dim=1)
    assert np.array_equal(ids_sorted.numpy(), case["topk_sorted"].astype(np.int64))
    assert np.array_equal(torch.gather(w, 1, ids_sorted).numpy(), case["topk_weights"])


def test_oracle_sort_tokens_is_stable_by_expert():
    idx = torch.tensor([[3, 1, 40, 2, 0, 5, 6, 7], [1, 3, 9, 10, 11, 12, 13, 33]])
    sid, sle, starts, counts = O.sort_tokens(idx, 0, 32)
    assert sle.tolist() == sorted(sle.tolist())
    # token order inside each expert is ascending (stable argsort of the flat pairs)
    for e in range(32):
        seg = sid[int(starts[e]): int(starts[e] + counts[e])].tolist()
        assert seg == sorted(seg)
    assert int(counts.sum()) == 14


def test_tolerance_checker_rejects_single_fp8_requant_scale_error():
    ref = torch.linspace(-3, 3, 10000).to(torch.bfloat16)
    bad = (ref.float() * 1.05).to(torch.bfloat16)
    assert not O.check_tolerance(bad, ref)["ok"]
    assert O.check_tolerance(ref, ref)["ok"]


def _quant_golden():
    import os
    d = np.load(os.path.join(os.path.dirname(__file__), "golden", "quant_golden.npz"))
    x = torch.from_numpy(d["x_bits"].view(np.int16)).view(torch.bfloat16)
    return x, torch.from_numpy(d["q_bits"]), torch.from_numpy(d["scale"])


def test_oracle_quantizer_matches_reference_bit_exact():
    """``quantize_rows_per_128`` against the reference ``_quantize_fp8_block_rows`` outputs (kernel.py:126-141)."""
    x, q_ref, s_ref = _quant_golden()
    q, s = O.quantize_rows_per_128(x)
    assert torch.equal(q.view(torch.uint8), q_ref)
    assert torch.equal(s, s_ref)
    assert torch.equal(s[:, 6], torch.ones(56))       # all-zero row: scale 1, codes 0
    assert int(q[6].view(torch.uint8).max()) == 0


def test_oracle_agrees_with_the_flashinfer_trace_reference():
    """Cross-check against a second, independent statement of the same definition: flashinfer's
    DS-routing FP8 block-scale MoE trace reference (flashinfer-python 0.6.11.post2,
    ``flashinfer/trace/templates/moe.py``, ``_trtllm_fp8_block_scale_moe_ds_routing_reference``),
    run on 4 local experts placed where the most tokens route (it dequantises every local expert)."""
    fi = pytest.importorskip("flashinfer.trace.templates.moe")
    from kernelforge_b200 import synthetic as S
    T, E, rsf = 64, 4, 2.5
    ti = S.token_inputs(T, seed=11)
    idx, _ = O.route(ti.routing_logits, ti.routing_bias, rsf)
    hist = torch.bincount(idx.flatten().long(), minlength=256)
    offset = int(torch.stack([hist[o:o + E].sum() for o in range(256 - E + 1)]).argmax())
    assert int(hist[offset:offset + E].sum()) >= 8            # enough pairs reach the local experts
    wb = S.expert_bank(E, offset, seed=3)
    ours = O.moe_layer(ti.routing_logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale,
                       wb.gemm1_weights, wb.gemm1_weights_scale, wb.gemm2_weights, wb.gemm2_weights_scale,
                       offset, rsf)
    ref = fi._trtllm_fp8_block_scale_moe_ds_routing_reference(
        ti.routing_logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale, wb.gemm1_weights,
        wb.gemm1_weights_scale, wb.gemm2_weights, wb.gemm2_weights_scale, 8, 8, 4, offset, rsf)
    assert ref.abs().max() > 0
    assert O.check_tolerance(ours, ref)["ok"]
    # both are fp32 restatements (different op order): far tighter than the layer's tolerance
    d = (ours.float() - ref.float()).abs().max()
    assert d <= 2e-3 * ref.float().abs().max(), float(d)


@pytest.mark.parametrize("mistake", ["gate_up_swapped", "w2_scale_grid_misread"])
def test_goldens_reject_a_wrong_weight_layout(mistake):
    """Negative controls for the layout conventions: W13 rows are [up (X1); gate (X2)] (reference
    ``kernel.py:1940-1943``) and the W2 scale grid is [E, H/128, I/128] (``kernel.py:118-123``).  The
    same layer computed with either convention broken misses the reference's golden output by far
    more than the tolerance, so the golden match above pins both conventions."""
    case = LAYER["t16_off0"]
    ti, wb, offset, rsf = layer_inputs(case)
    w13, w13s, w2, w2s = wb.gemm1_weights, wb.gemm1_weights_scale, wb.gemm2_weights, wb.gemm2_weights_scale
    if mistake == "gate_up_swapped":
        w13 = torch.cat([w13[:, 2048:], w13[:, :2048]], dim=1)
        w13s = torch.cat([w13s[:, 16:], w13s[:, :16]], dim=1)
    else:   # the same 896 numbers per expert read as an [I/128, H/128] grid, then transposed into place
        w2s = w2s.reshape(w2s.shape[0], 16, 56).transpose(1, 2).contiguous()
    out = O.moe_layer(ti.routing_logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale,
                      w13, w13s, w2, w2s, offset, rsf)
    ref = torch.from_numpy(case["out_bf16"]).view(torch.bfloat16)
    assert not O.check_tolerance(out, ref)["ok"]
