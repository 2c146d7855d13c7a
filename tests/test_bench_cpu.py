"""The bench's reference arm (the reference algorithm's CPU path): its JSON line at N = 1, and one line
from rank 0 alone under torchrun with 2 ranks.  No GPU needed."""
import json
import os
import socket
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _json_lines(out: str):
    return [json.loads(l) for l in out.splitlines() if l.startswith("{")]


def _check_reference_line(d, n_gpus):
    assert d["impl"] == "reference" and d["n_gpus"] == n_gpus
    assert d["unit"] == "tokens/s" and d["higher_is_better"] is True and d["value"] > 0
    assert d["metric"].startswith("MoE layer tokens/s")
    assert d["config"]["workload"] == "ep_layer_T8192_per_gpu_256_experts"
    assert d["config"]["local_experts_per_gpu"] == 256 // n_gpus
    # measured, not extrapolated: the steps' time is the measured slices' time
    assert abs(d["ms_per_step"] * d["steps"] / 1e3 - d["tokens_per_step"] * d["steps"] / d["value"]) < 1e-6 * d["ms_per_step"]
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["value"] == d["value"] and cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_single_process():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0"],
                       cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _json_lines(r.stdout)
    assert len(lines) == 1
    _check_reference_line(lines[0], 1)


def test_reference_arm_under_torchrun_prints_once():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), "bench.py", "--impl", "reference",
           "--gpus", "2", "--steps", "1", "--warmup", "0"]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _json_lines(r.stdout)
    assert len(lines) == 1
    _check_reference_line(lines[0], 2)


# ------------------------------------------------------------------ clock sampling --
def _bench():
    import importlib
    sys.path.insert(0, ROOT)
    return importlib.import_module("bench")


def _row(idx, uuid, bus, mhz, reasons=("Not Active",) * 4):
    return [str(idx), uuid, f"00000000:{bus:02X}:00.0", str(mhz), "1965", "900.0", *reasons]


def _samples():
    """nvidia-smi rows of an 8-GPU box every 25 ms for 1 s; GPU 5 (bus 0x9A) runs the bench from t = 0.4 s."""
    out = []
    for k in range(40):
        t = k * 0.025
        for g in range(8):
            busy = g == 5 and 0.4 <= t <= 0.8
            reasons = ("Not Active", "Not Active", "Not Active", "Active" if busy else "Not Active")
            out.append((t, _row(g, f"GPU-0000000{g}-aaaa-bbbb-cccc-dddddddddddd", 0x18 + 0x10 * g,
                                1300 if busy else 1965, reasons)))
    return out


def test_clock_rows_are_this_gpus_by_uuid_then_pci_then_index():
    b = _bench()
    s = _samples()
    rows, how = b.select_gpu_rows(s, {"uuid": b._hex("00000005-aaaa-bbbb-cccc-dddddddddddd"), "pci": None, "index": 0})
    assert how == "uuid" and {f[0] for _, f in rows} == {"5"}
    rows, how = b.select_gpu_rows(s, {"uuid": "ffff", "pci": (0, 0x18 + 0x50, 0), "index": 0})
    assert how == "pci" and {f[0] for _, f in rows} == {"5"}
    rows, how = b.select_gpu_rows(s, {"uuid": "", "pci": None, "index": 5})
    assert how == "index" and {f[0] for _, f in rows} == {"5"}
    assert b._pci_of("00000000:9A:00.0") == (0, 0x9A, 0) and b._pci_of("n/a") is None


def test_clock_summary_uses_only_the_timed_window():
    b = _bench()
    rows, _ = b.select_gpu_rows(_samples(), {"uuid": b._hex("GPU-00000005-aaaa-bbbb-cccc-dddddddddddd"),
                                             "pci": None, "index": 0})
    c = b.summarize_clocks(rows, [(0.45, 0.75, "timed steps")])
    assert c["sm_mhz"] == 1300 and c["sm_max_mhz"] == 1965 and c["reasons"] == ["sw_power_cap"]
    assert c["samples"] >= 3 and c["window"] == "timed steps"
    # too few samples in the timed window: the wider window is used, never the idle samples outside it
    c = b.summarize_clocks(rows, [(0.45, 0.47, "timed steps"), (0.45, 0.75, "timed + profiled")])
    assert c["window"] == "timed + profiled" and c["sm_mhz"] == 1300
    c = b.summarize_clocks(rows, [(5.0, 6.0, "timed steps")])
    assert c["reasons"] == ["unsampled"] and c["samples"] == 0


def test_gpu_identity_follows_cuda_visible_devices(monkeypatch):
    b = _bench()
    props = type("P", (), {"uuid": "00000005-aaaa-bbbb-cccc-dddddddddddd", "pci_domain_id": 0, "pci_bus_id": 0x68,
                           "pci_device_id": 0})()
    monkeypatch.setattr(b.torch.cuda, "get_device_properties", lambda i: props)
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "5,6")
    ident = b.gpu_identity(0)
    assert ident["index"] == 5 and ident["pci"] == (0, 0x68, 0)
    assert ident["uuid"] == b._hex("GPU-00000005-aaaa-bbbb-cccc-dddddddddddd")


def test_clock_sampler_retries_slower_when_the_fast_interval_is_refused(tmp_path):
    """A stand-in nvidia-smi that refuses -lms 25 and samples at 200 ms: the sampler ends up with samples."""
    import time
    b = _bench()
    fake = tmp_path / "fake-smi"
    fake.write_text("#!" + sys.executable + "\n"
                    "import sys, time\n"
                    "if sys.argv[sys.argv.index('-lms') + 1] == '25':\n"
                    "    sys.exit(2)\n"
                    "for _ in range(200):\n"
                    "    print('0, GPU-00000000-aaaa-bbbb-cccc-dddddddddddd, 00000000:18:00.0, 1300, 1965, 900.0, "
                    "Not Active, Not Active, Not Active, Active', flush=True)\n"
                    "    time.sleep(0.02)\n")
    fake.chmod(0o755)
    cs = b.ClockSampler(ident={"uuid": b._hex("00000000-aaaa-bbbb-cccc-dddddddddddd"), "pci": None, "index": 0},
                        exe=str(fake))
    t0 = time.time()
    cs.start()
    deadline = time.time() + 20
    while len(cs.samples) < 5 and time.time() < deadline:
        time.sleep(0.05)
    t1 = time.time()
    cs.stop()
    c = cs.summary([(t0, t1, "timed steps")])
    assert c["samples"] >= 5 and c["sm_mhz"] == 1300 and c["reasons"] == ["sw_power_cap"]
    assert c["gpu_matched_by"] == "uuid"


def test_clock_sampler_without_nvidia_smi_reports_unsampled():
    b = _bench()
    cs = b.ClockSampler(ident={"uuid": "", "pci": None, "index": 0}, exe="/nonexistent/nvidia-smi")
    cs.start()
    cs.stop()
    assert cs.summary([(0.0, 1e12, "timed steps")])["reasons"] == ["unsampled"]


def test_cpu_baseline_object_of_the_bench_line():
    """The main arm's cpu_baseline on a decode-sized workload (16 tokens, 32 local experts): the whole
    layer timed as its slices, and the error report when the layer cannot be built."""
    b = _bench()
    c = b.measure_cpu_baseline(16, 32, 0, parts=4)
    assert c["kind"] == "port" and c["value"] > 0 and c["cores"] >= 1 and "active" in c["sample"]
    for args in ((16, 32, 300), (-1, 32, 0)):   # experts past 256 / no inputs: reported, not raised
        err = b.measure_cpu_baseline(*args, parts=4)
        assert err["value"] is None and err["error"]


def test_cpu_slices_partition_the_layer():
    """The reference arm's slices cover every token's routing, every output row and every active
    expert exactly once per round of `parts` slices."""
    b = _bench()
    lay = b.CpuReferenceLayer(40, 32, 0, parts=4, pool=1)
    seen_experts = []
    for j in range(4):
        seen_experts += list(range(j, 32, 4))
        lay.run_part(j)
    assert sorted(seen_experts) == list(range(32))
    rows = [range(j * 40 // 4, (j + 1) * 40 // 4) for j in range(4)]
    assert sorted(r for rr in rows for r in rr) == list(range(40))


def test_reference_and_own_arm_share_the_config():
    import argparse
    b = _bench()
    for world in (1, 2, 8):
        args = argparse.Namespace(workload="ep", tokens=None, ep_exchange="p2p", graph=False, zipf=False)
        T, E, name = b.workload_shape(args, world)
        assert b.line_config(name, T, E, world, args)["local_experts_per_gpu"] == 256 // world
