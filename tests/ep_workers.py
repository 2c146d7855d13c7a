"""Worker functions for the CPU (gloo) expert-parallel tests; run in spawned processes."""
import datetime
import os
import sys
import traceback

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from kernelforge_b200 import synthetic as S  # noqa: E402
from oracle import moe_oracle as O  # noqa: E402
from tests import ep_reference as R  # noqa: E402


def oracle_route(logits, bias, rsf):
    idx, w = O.route(logits, bias, rsf)
    return idx.to(torch.int32), torch.gather(w, 1, idx)


def linear_experts(ids, w, hid, sc, w13, w13s, w2, w2s, offset, out_dtype=torch.bfloat16):
    """Stand-in for the expert kernels with the same skip semantics: expert g maps x to
    x * (g + 1) / 256, so the layer output is x * sum_k w_k (g_k + 1) / 256 over local experts."""
    E = w13.shape[0]
    x = (hid.to(torch.float32).view(-1, 56, 128) * sc.t().unsqueeze(-1)).view(-1, 7168)
    ids = ids.to(torch.int64)
    loc = ids - int(offset)
    valid = (ids >= 0) & (loc >= 0) & (loc < E)
    coef = ((ids + 1).to(torch.float32) * w * valid).sum(dim=1)
    return (x * coef.unsqueeze(1) / 256.0).to(out_dtype)


def tokens_for(rank, T):
    return S.token_inputs(T, seed=40 + rank)


def dummy_bank(E):
    z = torch.zeros(E, 1)
    return S.ExpertWeights(z, z, z, z)


def worker(rank, world, port, T_per_rank, combine, mode, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(1)
    res = {"rank": rank}
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
        E = 256 // world
        T = T_per_rank[rank]
        ti = tokens_for(rank, T)
        layer = R.TorchExchangeMoE(dummy_bank(E), rank * E, E, route_fn=oracle_route, experts_fn=linear_experts,
                                   combine_dtype=torch.float32 if combine == "f32" else torch.bfloat16)
        if mode == "drop" and rank == world - 1:
            res["dropped"] = True      # leaves before its first collective
            torch.save(res, os.path.join(result_dir, f"r{rank}.pt"))
            os._exit(0)
        out = layer.forward(ti.routing_logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale, 2.5)
        idx, w = oracle_route(ti.routing_logits, ti.routing_bias, 2.5)
        ref = linear_experts(idx, w, ti.hidden_states, ti.hidden_states_scale, torch.zeros(256, 1), None, None,
                             None, 0, out_dtype=torch.float32)
        res["out"] = out
        res["ref"] = ref
        res["sent"] = R.dispatch_plan(idx, w, world).send_counts
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # reported to the test, which decides whether it was expected
        res["error"] = f"{type(exc).__name__}: {exc}"
        res["trace"] = traceback.format_exc()
    torch.save(res, os.path.join(result_dir, f"r{rank}.pt"))
