"""Expert-parallel data flow on CPU gloo ranks (world size 2): dispatch dedup/masking,
all-to-all exchange, reverse exchange and fixed-order combine; failure cases on the host."""
import multiprocessing as mp
import os
import socket

import pytest
import torch

from kernelforge_b200 import ep
from tests import ep_reference as R
from tests.ep_workers import oracle_route, tokens_for, worker


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(world, T_per_rank, combine="f32", mode="normal", tmp_path=None, timeout=120):
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=worker, args=(r, world, port, T_per_rank, combine, mode, str(tmp_path)))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish")
    return [torch.load(os.path.join(tmp_path, f"r{r}.pt")) for r in range(world)]


def test_dispatch_plan_dedups_and_masks():
    ti = tokens_for(0, 64)
    idx, w = oracle_route(ti.routing_logits, ti.routing_bias, 2.5)
    for world in (2, 4, 8):
        plan = R.dispatch_plan(idx, w, world)
        per = 256 // world
        dest = idx.long() // per
        for t in range(64):
            ranks = sorted(set(dest[t].tolist()))
            assert [d for d in range(world) if plan.pos[t, d] >= 0] == ranks
            for d in ranks:
                row = int(plan.pos[t, d])
                assert int(plan.send_token[row]) == t
                ids = plan.send_ids[row].tolist()
                assert sorted(i for i in ids if i >= 0) == sorted(i for i in idx[t].tolist() if i // per == d)
        assert int(plan.send_counts.sum()) == int((plan.pos >= 0).sum())
        if world == 8:   # one routing group per rank: at most topk_group = 4 destinations
            assert int((plan.pos >= 0).sum(dim=1).max()) <= 4


def test_pack_unpack_roundtrip():
    ti = tokens_for(1, 10)
    idx, w = oracle_route(ti.routing_logits, ti.routing_bias, 2.5)
    plan = R.dispatch_plan(idx, w, 4)
    rows = R.pack_rows(ti.hidden_states, ti.hidden_states_scale, plan)
    assert rows.shape == (plan.send_token.numel(), ep.ROW_BYTES) and ep.ROW_BYTES % 16 == 0
    hid, sc, ids, ww = R.unpack_rows(rows)
    assert torch.equal(hid.view(torch.uint8), ti.hidden_states.index_select(0, plan.send_token).view(torch.uint8))
    assert torch.equal(sc, ti.hidden_states_scale[:, plan.send_token])
    assert torch.equal(ids, plan.send_ids) and torch.equal(ww, plan.send_w)


@pytest.mark.parametrize("combine", ["f32", "bf16"])
def test_ep_two_ranks_matches_single_process(tmp_path, combine):
    res = _run(2, [37, 53], combine=combine, tmp_path=tmp_path)
    for r in res:
        assert "error" not in r, r.get("trace")
        out, ref = r["out"].float(), r["ref"]
        if combine == "f32":
            assert torch.allclose(out, ref.to(torch.bfloat16).float(), rtol=1e-2, atol=1e-2)
            assert (out - ref).abs().max() <= 1e-2 * ref.abs().max()
        else:
            d = (out - ref).abs()
            assert d.max() <= 1e-2 * ref.abs().max()
            assert ((d <= 1e-2 + 2e-2 * ref.abs()).float().mean()) >= 0.999


def test_ep_zero_token_rank(tmp_path):
    res = _run(2, [41, 0], tmp_path=tmp_path)
    assert "error" not in res[0], res[0].get("trace")
    assert "error" not in res[1], res[1].get("trace")
    assert res[1]["out"].shape == (0, 7168)
    assert (res[0]["out"].float() - res[0]["ref"]).abs().max() <= 1e-2 * res[0]["ref"].abs().max()


def test_ep_dropped_rank_raises_on_survivor(tmp_path):
    """A rank leaves before the first collective: the survivor's collective times out with an error."""
    res = _run(2, [16, 16], mode="drop", tmp_path=tmp_path)
    assert res[1].get("dropped")
    assert "error" in res[0]


def test_peer_capacity_needs():
    """Receive-area need = the largest column sum, return-area need = the largest row sum of the count matrix."""
    from kernelforge_b200.ep import peer_capacity_needs
    counts = torch.tensor([[5, 0, 7], [1, 2, 3], [0, 9, 0]], dtype=torch.int32)   # [source, destination]
    assert peer_capacity_needs(counts) == (11, 12)   # column 1: 0+2+9, row 0: 5+0+7
    assert peer_capacity_needs(torch.zeros(2, 2, dtype=torch.int32)) == (0, 0)


def test_peer_status_errors_are_decoded_and_sticky():
    """A non-zero status word of the peer exchange raises on check(), naming its cause, every time."""
    from types import SimpleNamespace
    assert ep.peer_status_error(0) is None
    assert "barrier" in ep.peer_status_error(ep.STATUS_TIMEOUT_PEER)
    assert "overflowed" in ep.peer_status_error(ep.STATUS_SLOT_OVERFLOW)
    m = object.__new__(ep.ExpertParallelMoE)
    m.exchange = "p2p"
    m._peer = None
    m.check()                                           # before the first step: nothing to check
    m._peer = SimpleNamespace(status=torch.zeros(1, dtype=torch.int32))
    m.check()
    m._peer.status[0] = ep.STATUS_TIMEOUT_PEER
    for _ in range(2):
        with pytest.raises(RuntimeError, match="0x20"):
            m.check()
    m.exchange = "nccl"
    m.check()                                           # NCCL exchange: its collectives raise instead
