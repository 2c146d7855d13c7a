"""Both GEMM implementations -- single-CTA (default) and CTA-pair (cta_group::2,
KF_MOE_GEMM=pair) -- against the fp32 reference, each in a fresh process (the
path is chosen once per process)."""
import os
import subprocess
import sys

import pytest

from tests.helpers import gpu_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not gpu_available(), reason="needs a B200")]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = r"""
import sys, torch
sys.path.insert(0, %r)
from kernelforge_b200 import binding as B, synthetic as S
from oracle import moe_oracle as O
from tests.helpers import gpu_bank, to_cuda
bad = []
for T, E, off, seed in [(1, 32, 0, 1), (40, 32, 0, 2), (300, 32, 96, 3), (1000, 32, 0, 4), (700, 256, 0, 5)]:
    ti = to_cuda(S.token_inputs(T, seed=seed))
    wb = gpu_bank(E, off, seed=seed)
    out = B.kernel(ti.routing_logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale,
                   wb.gemm1_weights, wb.gemm1_weights_scale, wb.gemm2_weights, wb.gemm2_weights_scale, off, 2.5)
    torch.cuda.synchronize()
    st = B.read_status()
    idx, w = B.route(ti.routing_logits, ti.routing_bias, 2.5)
    ref = O.moe_experts(idx, w, ti.hidden_states, ti.hidden_states_scale, wb.gemm1_weights, wb.gemm1_weights_scale,
                        wb.gemm2_weights, wb.gemm2_weights_scale, off).to(torch.bfloat16)
    res = O.check_tolerance(out, ref)
    if st or not res["ok"]:
        bad.append((T, E, off, st, res))
print("BAD", bad) if bad else print("OK")
sys.exit(1 if bad else 0)
""" % ROOT


@pytest.mark.parametrize("path", ["1sm", "pair"])
def test_gemm_path_parity(path):
    env = dict(os.environ)
    if path == "pair":
        env["KF_MOE_GEMM"] = "pair"
    else:
        env.pop("KF_MOE_GEMM", None)
    r = subprocess.run([sys.executable, "-c", SCRIPT], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
