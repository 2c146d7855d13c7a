"""Expert-parallel CUDA kernels on one GPU (ranks emulated): dispatch packing,
the packed-row experts entry point and the combine, each bit-exact against the
tensor-op restatement in tests/ep_reference.py."""
import pytest
import torch

from kernelforge_b200 import binding as B
from kernelforge_b200 import ep
from kernelforge_b200 import synthetic as S
from tests import ep_reference as R
from tests.helpers import gpu_available, gpu_bank, to_cuda

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not gpu_available(), reason="needs a B200")]


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("T", [5, 300])
def test_dispatch_matches_restatement(world, T):
    ti = to_cuda(S.token_inputs(T, seed=70 + T))
    idx, w = B.route(ti.routing_logits, ti.routing_bias, 2.5)
    send, counts, pos = B.ep_dispatch(idx, w, ti.hidden_states, ti.hidden_states_scale, world)
    plan = R.dispatch_plan(idx, w, world)
    ref_rows = R.pack_rows(ti.hidden_states, ti.hidden_states_scale, plan)
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
    hid, sc, ids, ww = R.unpack_rows(rows)
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
    ref = R.combine(back, pos.long())
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


# ---------------------------------------------------------------- peer exchange --
# The peer-to-peer kernels with the ranks emulated on one GPU: every "peer"
# pointer points at another local buffer, and the ranks' kernels run one after
# the other on one stream (their stream order stands in for the barriers).


def _ptrs(ts):
    return torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device="cuda")


def _emulated_ranks_from(world, T, fp8_rows):
    """As _emulated_ranks, with each rank's hidden rows replaced by the given (e4m3, scales)."""
    return _emulated_ranks(world, T, fp8_rows=fp8_rows)


def _emulated_ranks(world, T, bf16_rows=None, fp8_rows=None):
    lib = B.library()
    ranks = []
    for r in range(world):
        ti = to_cuda(S.token_inputs(T, seed=200 + r))
        if bf16_rows is not None:       # pack bf16 rows, quantised on the way out
            ti = S.TokenInputs(ti.routing_logits, ti.routing_bias, bf16_rows[r], None)
        if fp8_rows is not None:
            ti = S.TokenInputs(ti.routing_logits, ti.routing_bias, fp8_rows[r][0], fp8_rows[r][1])
        idx, w = B.route(ti.routing_logits, ti.routing_bias, 2.5)
        ranks.append({"ti": ti, "idx": idx, "w": w,
                      "counts": torch.zeros(world * world, dtype=torch.int32, device="cuda"),
                      "recv": torch.zeros((T * world, ep.ROW_BYTES), dtype=torch.uint8, device="cuda"),
                      "back": torch.zeros((int(lib.kf_ep_max_send_rows(T, world)), B.H), dtype=torch.bfloat16,
                                          device="cuda"),
                      "ws": torch.zeros(max(int(lib.kf_ep_workspace_bytes(T, world)), 256), dtype=torch.uint8,
                                        device="cuda"),
                      "pos": torch.empty((T, world), dtype=torch.int32, device="cuda"),
                      "status": torch.zeros(1, dtype=torch.int32, device="cuda")})
    stream = torch.cuda.current_stream().cuda_stream
    peer_counts = _ptrs([x["counts"] for x in ranks])
    peer_recv = _ptrs([x["recv"] for x in ranks])
    for r, x in enumerate(ranks):
        rc = lib.kf_ep_plan_p2p(B._ptr(x["idx"]), T, world, r, peer_counts.data_ptr(), B._ptr(x["ws"]),
                                x["ws"].numel(), stream)
        assert rc == 0
    for r, x in enumerate(ranks):
        rc = lib.kf_ep_pack_p2p(B._ptr(x["idx"]), B._ptr(x["w"]), B._ptr(x["ti"].hidden_states),
                                B._ptr(x["ti"].hidden_states_scale), T, world, r, x["counts"].data_ptr(),
                                peer_recv.data_ptr(), T * world, B._ptr(x["pos"]), x["status"].data_ptr(),
                                B._ptr(x["ws"]), x["ws"].numel(), stream)
        assert rc == 0
    torch.cuda.synchronize()
    return ranks


@pytest.mark.parametrize("world", [2, 4])
def test_peer_pack_matches_dispatch(world):
    """Every rank's receive area = the sources' dispatch rows for it, in source order; counts and pos as dispatch."""
    T = 300
    ranks = _emulated_ranks(world, T)
    sends = [B.ep_dispatch(x["idx"], x["w"], x["ti"].hidden_states, x["ti"].hidden_states_scale, world)
             for x in ranks]
    torch.cuda.synchronize()
    counts = torch.stack([c.cpu() for _, c, _ in sends]).to(torch.int32)        # [source, dest]
    for r, x in enumerate(ranks):
        assert torch.equal(x["counts"].cpu().view(world, world), counts)          # every rank holds the full matrix
        assert torch.equal(x["pos"], sends[r][2])
        assert int(x["status"].item()) == 0
    for d, x in enumerate(ranks):
        parts = []
        for s in range(world):
            off = int(counts[s, :d].sum())
            parts.append(sends[s][0][off:off + int(counts[s, d])])
        expect = torch.cat(parts)
        assert torch.equal(x["recv"][:expect.shape[0]], expect)


def test_peer_pack_quantises_bf16_rows_like_the_quantiser():
    """bf16 rows packed with the quantisation fused in = the rows kf_quantize_hidden makes, packed as e4m3."""
    world, T = 4, 300
    g = torch.Generator().manual_seed(9)
    rows = [(torch.randn(T, B.H, generator=g) * 3).to(torch.bfloat16).cuda() for _ in range(world)]
    fused = _emulated_ranks(world, T, bf16_rows=rows)
    plain = []
    for r in range(world):           # the same routing inputs, rows quantised first
        q, s = B.quantize_hidden(rows[r])
        plain.append((q, s))
    ref = _emulated_ranks_from(world, T, plain)
    for d, (a, b) in enumerate(zip(fused, ref)):
        assert torch.equal(a["counts"], b["counts"])
        n = int(a["counts"].view(world, world)[:, d].sum())
        assert n > 0 and torch.equal(a["recv"][:n], b["recv"][:n])
        assert torch.equal(a["pos"], b["pos"])


def test_peer_return_fused_into_reduce():
    """experts_packed_p2p stores each partial at its source's send position: the same rows experts_packed returns."""
    world, T = 2, 300
    E = 256 // world
    ranks = _emulated_ranks(world, T)
    counts = ranks[0]["counts"].cpu().view(world, world)
    banks = [gpu_bank(E, d * E, seed=5) for d in range(world)]
    peer_back = _ptrs([x["back"] for x in ranks])
    partials = []
    for d, x in enumerate(ranks):
        R = int(counts[:, d].sum())
        rows = x["recv"][:R]
        wb = banks[d]
        partials.append(B.experts_packed(rows, wb.gemm1_weights, wb.gemm1_weights_scale, wb.gemm2_weights,
                                         wb.gemm2_weights_scale, d * E))
        B.experts_packed_p2p(rows, wb.gemm1_weights, wb.gemm1_weights_scale, wb.gemm2_weights,
                             wb.gemm2_weights_scale, d * E, x["counts"], d, world, peer_back)
    torch.cuda.synchronize()
    for s, x in enumerate(ranks):
        expect = torch.cat([partials[d][int(counts[:s, d].sum()):int(counts[:s + 1, d].sum())] for d in range(world)])
        assert torch.equal(x["back"][:expect.shape[0]], expect)


@pytest.mark.parametrize("fused", [True, False])
def test_peer_return_stores_nothing_past_the_received_rows(fused):
    """A call with more rows than the count matrix gives this rank: the extra rows
    (no local pair) reach no source's return buffer, fused into the reduce or not."""
    world, T, d = 2, 300, 0
    E = 256 // world
    lib = B.library()
    ranks = _emulated_ranks(world, T)
    counts = ranks[0]["counts"].cpu().view(world, world)
    R = int(counts[:, d].sum())
    extra = min(16, T * world - R)
    assert extra > 0
    x = ranks[d]
    ids = x["recv"][R:R + extra, B.H + 56 * 4:B.H + 56 * 4 + 32]
    ids.fill_(0xFF)                       # expert ids -1: rows without a local pair
    rows = x["recv"][:R + extra]
    wb = gpu_bank(E, d * E, seed=5)
    part = B.experts_packed(rows[:R], wb.gemm1_weights, wb.gemm1_weights_scale, wb.gemm2_weights,
                            wb.gemm2_weights_scale, d * E)
    for y in ranks:
        y["back"].fill_(7.0)
    peer_back = _ptrs([y["back"] for y in ranks])
    if fused:
        B.experts_packed_p2p(rows, wb.gemm1_weights, wb.gemm1_weights_scale, wb.gemm2_weights,
                             wb.gemm2_weights_scale, d * E, x["counts"], d, world, peer_back)
    else:
        part_x = B.experts_packed(rows, wb.gemm1_weights, wb.gemm1_weights_scale, wb.gemm2_weights,
                                  wb.gemm2_weights_scale, d * E)
        rc = lib.kf_ep_return_p2p(B._ptr(part_x), R + extra, world, d, x["counts"].data_ptr(), peer_back.data_ptr(),
                                  torch.cuda.current_stream().cuda_stream)
        assert rc == 0
    torch.cuda.synchronize()
    assert B.read_status() == 0
    for s, y in enumerate(ranks):
        n, so = int(counts[s, d]), int(counts[s, :d].sum())
        off = int(counts[:s, d].sum())
        assert torch.equal(y["back"][so:so + n], part[off:off + n])
        assert bool((y["back"][:so] == 7.0).all()) and bool((y["back"][so + n:] == 7.0).all())


def test_peer_barrier_times_out_instead_of_hanging():
    """A rank that never arrives: the barrier gives up after its bounded wait and reports it (no trap, no hang)."""
    lib = B.library()
    flags = [torch.zeros(2, dtype=torch.int32, device="cuda") for _ in range(2)]
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    peer_flags = _ptrs(flags)
    rc = lib.kf_ep_barrier(peer_flags.data_ptr(), flags[0].data_ptr(), 0, 2, 1, status.data_ptr(),
                           torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) & 0x20            # KF_STATUS_TIMEOUT_PEER
    assert flags[0].tolist() == [1, 0] and flags[1].tolist() == [1, 0]   # its own arrival reached both ranks
