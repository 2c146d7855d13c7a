"""Worker for the multi-GPU expert-parallel test (NCCL, one process per GPU)."""
import datetime
import os
import sys
import traceback

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def worker(rank, world, port, T, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    res = {"rank": rank}
    try:
        from kernelforge_b200 import binding as B
        from kernelforge_b200 import ep
        from kernelforge_b200 import synthetic as S
        from oracle import moe_oracle as O
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        E = 256 // world
        ti = S.token_inputs(T, seed=60 + rank, device=dev)
        shard = S.expert_bank(E, rank * E, seed=3, device=dev)
        layer = ep.ExpertParallelMoE(shard, rank * E, E, combine_dtype=torch.float32, exchange="nccl")
        out = layer.forward(ti.routing_logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale, 2.5)
        torch.cuda.synchronize(dev)
        res["status"] = B.read_status(dev)
        # single-GPU reference on this rank's tokens: all 256 experts resident here
        full = S.expert_bank(256, 0, seed=3, device=dev)
        single = B.kernel(ti.routing_logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale,
                          full.gemm1_weights, full.gemm1_weights_scale, full.gemm2_weights,
                          full.gemm2_weights_scale, 0, 2.5)
        idx, w = B.route(ti.routing_logits, ti.routing_bias, 2.5)
        ref = O.moe_experts(idx, w, ti.hidden_states, ti.hidden_states_scale, full.gemm1_weights,
                            full.gemm1_weights_scale, full.gemm2_weights, full.gemm2_weights_scale, 0)
        res["ep_vs_ref"] = O.check_tolerance(out, ref.to(torch.bfloat16))
        res["single_vs_ref"] = O.check_tolerance(single, ref.to(torch.bfloat16))
        res["ep_vs_single_maxdiff"] = float((out.float() - single.float()).abs().max())
        # the peer-to-peer exchange against the NCCL one (same kernels and combine order: bit-identical),
        # over two steps in a row (the barrier epochs advance and the buffers are reused)
        nccl = ep.ExpertParallelMoE(shard, rank * E, E, exchange="nccl")
        p2p = ep.ExpertParallelMoE(shard, rank * E, E, exchange="p2p")
        args = (ti.routing_logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale, 2.5)
        o_nccl = nccl.forward(*args)
        o_p2p = [p2p.forward(*args) for _ in range(2)]
        torch.cuda.synchronize(dev)
        res["p2p_equal_nccl"] = [bool(torch.equal(o, o_nccl)) for o in o_p2p]
        res["p2p_vs_ref"] = O.check_tolerance(o_p2p[1], ref.to(torch.bfloat16))
        res["p2p_pairs"] = p2p.local_pairs()
        p2p.check()                                        # no barrier gave up, no receive area overflowed
        res["p2p_status"] = p2p.status()
        res["nccl_pairs"] = nccl.local_pairs()
        # uneven token counts (one rank empty in the second step): the receive and return areas are
        # sized from the count matrix every rank holds, and grow together when a step needs more
        uneven = ep.ExpertParallelMoE(shard, rank * E, E, exchange="p2p")
        res["uneven"] = []
        for step, Ts in enumerate(([64, 32], [700, 0])):
            tu = S.token_inputs(Ts[rank], seed=90 + 10 * step + rank, device=dev)
            ou = uneven.forward(tu.routing_logits, tu.routing_bias, tu.hidden_states, tu.hidden_states_scale, 2.5)
            torch.cuda.synchronize(dev)
            if Ts[rank] == 0:
                res["uneven"].append({"ok": tuple(ou.shape) == (0, 7168)})
                continue
            iu, wu = B.route(tu.routing_logits, tu.routing_bias, 2.5)
            ru = O.moe_experts(iu, wu, tu.hidden_states, tu.hidden_states_scale, full.gemm1_weights,
                               full.gemm1_weights_scale, full.gemm2_weights, full.gemm2_weights_scale, 0)
            res["uneven"].append(O.check_tolerance(ou, ru.to(torch.bfloat16)))
        res["uneven_caps"] = (uneven._peer.recv_cap, uneven._peer.send_cap)
        res["uneven_status"] = uneven.status()
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:
        res["error"] = f"{type(exc).__name__}: {exc}"
        res["trace"] = traceback.format_exc()
    torch.save(res, os.path.join(result_dir, f"g{rank}.pt"))
