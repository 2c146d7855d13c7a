"""Expert-parallel layer on 2 GPUs (NCCL and the peer-to-peer exchange) vs the single-GPU layer and the fp32 reference."""
import multiprocessing as mp
import os
import socket

import pytest
import torch

from tests.helpers import gpu_available

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not gpu_available() or torch.cuda.device_count() < 2, reason="needs 2 B200s")]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_ep_two_gpus(tmp_path):
    from tests.ep_gpu_worker import worker
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=worker, args=(r, 2, port, 1024, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(600)
        if p.is_alive():
            p.kill()
            pytest.fail("EP rank did not finish")
    for r in range(2):
        res = torch.load(os.path.join(tmp_path, f"g{r}.pt"))
        assert "error" not in res, res.get("trace")
        assert res["status"] == 0
        assert res["ep_vs_ref"]["ok"], res
        assert res["single_vs_ref"]["ok"], res
        assert res["p2p_equal_nccl"] == [True, True], res
        assert res["p2p_vs_ref"]["ok"], res
        assert res["p2p_pairs"] == res["nccl_pairs"], res
        assert all(u["ok"] for u in res["uneven"]), res["uneven"]
        assert res["p2p_status"] == 0 and res["uneven_status"] == 0, res
