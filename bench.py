#!/usr/bin/env python
"""Benchmark of the fused DeepSeek-V3 FP8 block-scale MoE layer on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl kernelforge|reference]
                    [--workload ep|prefill|decode] [--tokens T] [--zipf] [--graph]
                    [--ep-exchange p2p|nccl] [--no-cpu-baseline]

Default workload ("ep", the layer of config 3 of the headline metric): 8192
tokens per GPU, all 256 experts sharded 256/N per GPU (N=1: all 256 on one GPU),
hidden 7168 / intermediate 2048 FP8 block-scaled weights; tokens are routed over
all experts.  With N > 1 the layer runs expert-parallel (one process per GPU,
launched by torchrun): dispatch rows and returned partials travel by stores into
the ranks' symmetric buffers (--ep-exchange p2p, the default) or by NCCL
all-to-all (--ep-exchange nccl).  A "step" is one forward of the layer over the
GPU's 8192 tokens; per-GPU work is fixed as N grows (weak scaling).

Prints ONE JSON line (rank 0).  Metric: tokens/s of the whole job (all GPUs).
Inputs are synthetic (seeded N(0,1) logits / activations, N(0,0.02) weights,
generated on the GPU); the weights (11.3 GB) are far larger than L2, so every
step streams them from HBM (no L2 flush needed).

--impl reference times the reference algorithm's CPU path (the oracle port of
solution/triton/kernel.py::kernel's PyTorch loop) on this host's cores: per step,
all tokens routed and the expert loop run on 8 of the active experts, scaled to
all of them (CpuOracleSample).
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, I, E_GLOBAL = 7168, 2048, 256
FLOP_PER_PAIR = 2 * (2 * I * H + H * I)            # 88,080,384
GEMM1_FLOP_PER_PAIR = 2 * 2 * I * H                # 58,720,256
W13_BYTES_PER_EXPERT = 2 * I * H                   # 29,360,128 (e4m3)
W2_BYTES_PER_EXPERT = H * I                        # 14,680,064
W13_SCALE_BYTES = (2 * I // 128) * (H // 128) * 4
W2_SCALE_BYTES = (H // 128) * (I // 128) * 4
METRIC = "MoE layer tokens/s (FP8 block-scale DeepSeek-V3 layer, T=8192 tokens per GPU, 256 experts EP-sharded)"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="kernelforge", choices=["kernelforge", "reference"])
    p.add_argument("--workload", default="ep", choices=["ep", "prefill", "decode"])
    p.add_argument("--tokens", type=int, default=None)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--graph", action="store_true", help="replay the layer as a CUDA graph (1 GPU)")
    p.add_argument("--zipf", action="store_true",
                   help="config 4: routing bias skewing expert popularity to Zipf(1.2) over a seeded permutation")
    p.add_argument("--ep-exchange", default="p2p", choices=["p2p", "nccl"],
                   help="N > 1: peer-to-peer stores into symmetric buffers, or NCCL all-to-all")
    return p.parse_args()


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16": d["bf16_tflops"], "bf16_sustained": d["bf16_tflops_sustained"],
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


CLOCK_FIELDS = ("index,uuid,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                "clocks_event_reasons.sw_power_cap")
REASON_NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


def _hex(s) -> str:
    return re.sub(r"[^0-9a-f]", "", str(s).lower())


def gpu_identity(dev_index: int) -> dict:
    """How to find this CUDA device among nvidia-smi's rows: its UUID, PCI address and, as a last resort,
    the physical index CUDA_VISIBLE_DEVICES maps it to."""
    p = torch.cuda.get_device_properties(dev_index)
    vis = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    phys = dev_index
    if dev_index < len(vis) and vis[dev_index].isdigit():
        phys = int(vis[dev_index])
    pci = tuple(getattr(p, k, None) for k in ("pci_domain_id", "pci_bus_id", "pci_device_id"))
    return {"uuid": _hex(getattr(p, "uuid", "")), "pci": pci if None not in pci else None, "index": phys}


def _pci_of(field: str):
    """(domain, bus, device) of an nvidia-smi pci.bus_id such as 00000000:17:00.0, or None."""
    m = re.fullmatch(r"\s*([0-9a-fA-F]+):([0-9a-fA-F]+):([0-9a-fA-F]+)\.[0-9a-fA-F]+\s*", field)
    return tuple(int(x, 16) for x in m.groups()) if m else None


def select_gpu_rows(samples, ident):
    """The samples of this GPU: matched by UUID, else by PCI address, else by physical index.
    Returns (rows, how) with rows = [(time, fields)] and fields = the CLOCK_FIELDS values."""
    if ident.get("uuid"):
        rows = [(t, f) for t, f in samples if _hex(f[1]) == ident["uuid"]]
        if rows:
            return rows, "uuid"
    if ident.get("pci"):
        rows = [(t, f) for t, f in samples if _pci_of(f[2]) == tuple(ident["pci"])]
        if rows:
            return rows, "pci"
    rows = [(t, f) for t, f in samples if f[0].strip() == str(ident.get("index"))]
    return rows, "index"


def summarize_clocks(rows, windows):
    """Median SM clock, max clock and the throttle reasons seen in the first window of `windows` that
    holds at least 3 samples (else the last, widest one).  Samples outside the windows (idle time
    before and after the timed steps) never count."""
    def num(x):
        try:
            return float(x)
        except ValueError:
            return None
    win, label = [], "none"
    for lo, hi, name in windows:
        win = [f for t, f in rows if lo <= t <= hi]
        label = name
        if len(win) >= 3:
            break
    if not win:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0, "window": label}
    mhz = [v for v in (num(f[3]) for f in win) if v is not None]
    mx = [v for v in (num(f[4]) for f in win) if v is not None]
    reasons = sorted({REASON_NAMES[i] for f in win for i in range(4) if f[6 + i].strip().lower() == "active"})
    return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": max(mx) if mx else None,
            "reasons": reasons, "samples": len(win), "window": label}


class ClockSampler:
    """nvidia-smi samples (every 25 ms, all GPUs; this GPU's rows picked by UUID / PCI address) of the
    SM clock and throttle reasons while the timed steps run.  If nvidia-smi ends without a sample (an
    interval it refuses), it is started again at 200 ms."""

    def __init__(self, dev_index=None, ident=None, exe: str = "nvidia-smi"):
        self.ident = ident if ident is not None else gpu_identity(dev_index)
        self.exe = exe
        self.samples = []
        self._lock = threading.Lock()
        self._stopping = False
        self._periods = []
        self._proc = None
        self._threads = []

    def start(self, period_ms: int = 25):
        self._periods = [period_ms] + ([200] if period_ms != 200 else [])
        self._launch()

    def _launch(self):
        with self._lock:
            if self._stopping or not self._periods:
                return
            cmd = [self.exe, f"--query-gpu={CLOCK_FIELDS}", "--format=csv,noheader,nounits", "-lms",
                   str(self._periods.pop(0))]
            try:
                proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            except OSError:
                return
            self._proc = proc
            th = threading.Thread(target=self._read, args=(proc,), daemon=True)
            self._threads.append(th)
            th.start()

    def _read(self, proc):
        got = 0
        for line in proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 10:
                self.samples.append((time.time(), parts))
                got += 1
        proc.wait()
        if got == 0:
            self._launch()

    def stop(self):
        with self._lock:
            self._stopping = True
            proc = self._proc
        if proc is not None and proc.poll() is None:
            proc.terminate()
            try:
                proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                proc.kill()
        for th in list(self._threads):
            th.join(timeout=5)

    def summary(self, windows):
        rows, how = select_gpu_rows(list(self.samples), self.ident)
        out = summarize_clocks(rows, windows)
        out["gpu_matched_by"] = how
        return out


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    return world, rank, local


def workload_shape(args, world):
    if args.workload == "ep":
        T = args.tokens or 8192
        E = E_GLOBAL // world
        return T, E, "ep_layer_T8192_per_gpu_256_experts" if T == 8192 else f"ep_layer_T{T}_per_gpu_256_experts"
    if args.workload == "prefill":
        T = args.tokens or 4096
        return T, 32, f"prefill_T{T}_32_local_experts"
    T = args.tokens or 16
    return T, 32, f"decode_T{T}_32_local_experts"


# ---------------------------------------------------------------- CPU baseline --
class CpuOracleSample:
    """A bounded sample of the workload for the reference algorithm's CPU path, timed so that it
    scales to the whole layer.

    The reference's CPU layer (``solution/triton/kernel.py:1927-1950``, restated in
    ``oracle/moe_oracle.py``) loops over the active local experts independently: each iteration
    dequantises one expert's weights and its rows and runs that expert's two GEMMs, so dequantising
    weights is paid once per expert and amortised over its pairs.  A sample of a few tokens would
    pay it for a handful of pairs and understate the path's throughput by orders of magnitude.
    This sample keeps the workload's amortisation.  It routes all T tokens, then runs the loop for
    k of the active experts (at the midpoints of k quantiles of the per-expert pair counts) with all
    of their pairs, and scales that loop time by active/k.  The per-call fixed work (zeroing the fp32 accumulator, the bf16 cast) is timed as a
    call with no local pair and counted once.  The expert weights are generated once, outside the
    timing.
    """

    def __init__(self, T: int, num_local: int, offset: int = 0, k: int = 8, seed: int = 1000):
        from kernelforge_b200 import synthetic as S
        from oracle import moe_oracle as O
        torch.set_num_threads(os.cpu_count() or 1)
        self.O, self.T = O, T
        self.ti = S.token_inputs(T, seed=seed)
        idx, _ = O.route(self.ti.routing_logits, self.ti.routing_bias, 2.5)
        counts = torch.bincount(idx.flatten().long(), minlength=E_GLOBAL)
        self.active = [e for e in range(offset, offset + num_local) if counts[e] > 0]
        # experts at the midpoints of k equal quantiles of the pair counts: the sample's pairs per
        # expert track the population's, so both the per-expert and the per-pair work scale by active/k
        by_count = sorted(self.active, key=lambda e: (int(counts[e]), e))
        k = min(k, len(self.active))
        self.sample = sorted(by_count[int((i + 0.5) * len(by_count) / k)] for i in range(k))
        self.total_pairs = int(sum(int(counts[e]) for e in self.active))
        # with no local pair the loop is empty and never reads the (placeholder) weights
        banks = [S.expert_weights(g, seed=0) for g in (self.sample or [offset])]
        self.w = [torch.stack([b[i] for b in banks]) for i in range(4)]
        self.lut = torch.full((E_GLOBAL,), -1, dtype=torch.int64)
        if self.sample:
            self.lut[torch.tensor(self.sample)] = torch.arange(len(self.sample))
        self.pairs = int((self.lut[idx] >= 0).sum())

    def time_once(self) -> float:
        """Estimated seconds of the whole layer on this host (one timed sample)."""
        O, ti = self.O, self.ti
        t0 = time.perf_counter()
        idx, w = O.route(ti.routing_logits, ti.routing_bias, 2.5)
        cidx = self.lut[idx]
        wsel = torch.gather(w, 1, idx)
        t1 = time.perf_counter()
        O.moe_experts(cidx, wsel, ti.hidden_states, ti.hidden_states_scale, *self.w, 0).to(torch.bfloat16)
        t2 = time.perf_counter()
        O.moe_experts(torch.full_like(cidx, -1), wsel, ti.hidden_states, ti.hidden_states_scale, *self.w,
                      0).to(torch.bfloat16)
        t3 = time.perf_counter()
        fixed = t3 - t2
        loop = max(0.0, (t2 - t1) - fixed)
        scale = len(self.active) / len(self.sample) if self.sample else 0.0
        return (t1 - t0) + fixed + loop * scale

    def describe(self, est_s: float) -> str:
        return (f"all {self.T} tokens routed; the expert loop timed on {len(self.sample)} of the "
                f"{len(self.active)} active experts ({self.pairs} of {self.total_pairs} pairs) and scaled by "
                f"{len(self.active)}/{max(1, len(self.sample))}; estimated layer {est_s:.1f} s (PyTorch CPU, "
                f"reference algorithm restated in oracle/moe_oracle.py)")


def measure_cpu_baseline(T: int, num_local: int, offset: int, repeats: int = 3) -> dict:
    """The ``cpu_baseline`` object of the bench line: the median of `repeats` CpuOracleSample
    estimates after one warm-up.  A failure is reported inside the object (it must not cost the
    measured line it rides on)."""
    try:
        smp = CpuOracleSample(T, num_local, offset)
        smp.time_once()
        est = statistics.median(smp.time_once() for _ in range(repeats))
        return {"value": T / est, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
                "sample": f"median of {repeats}: " + smp.describe(est)}
    except Exception as exc:  # noqa: BLE001 -- reported in the line, not swallowed
        return {"value": None, "unit": "tokens/s", "error": f"{type(exc).__name__}: {exc}"}


def run_reference(args, world, rank):
    if rank != 0:
        return
    T, E, name = workload_shape(args, 1)
    smp = CpuOracleSample(T, E)
    cores = torch.get_num_threads()
    for _ in range(args.warmup):
        smp.time_once()
    ests = [smp.time_once() for _ in range(args.steps)]
    t_all = sum(ests)
    value = T * args.steps / t_all
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t_all / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": name, "tokens_per_gpu": T, "experts": E_GLOBAL,
                   "sample": "per step: " + smp.describe(statistics.median(ests))},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": smp.describe(statistics.median(ests))},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------- our arm --
def main():
    args = parse()
    if args.impl == "reference":
        # the reference's CPU path runs on rank 0 alone; under torchrun the other ranks exit
        # at once, so this arm needs no process group (and no GPU)
        run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")))
        return
    world, rank, local = dist_setup(args)

    from kernelforge_b200 import binding as B
    from kernelforge_b200 import synthetic as S
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    T, E, name = workload_shape(args, world)
    offset = rank * E if args.workload == "ep" else 0
    peaks = load_peaks()

    bias = S.zipf_bias(seed=0).to(dev) if args.zipf else None
    ti = S.token_inputs(T, seed=17 + rank, device=dev, routing_bias=bias)
    if args.zipf:
        name += "_zipf1.2"
    wb = S.expert_bank(E, offset, seed=0, device=dev)
    torch.cuda.synchronize(dev)

    if world > 1:
        from kernelforge_b200 import ep
        layer = ep.ExpertParallelMoE(wb, offset, E, plumbing="p2p" if args.ep_exchange == "p2p" else "cuda")

        def step(logits, bias, hid, hs):
            return layer.forward(logits, bias, hid, hs, 2.5)
    else:
        def step(logits, bias, hid, hs):
            return B.kernel(logits, bias, hid, hs, wb.gemm1_weights, wb.gemm1_weights_scale, wb.gemm2_weights,
                            wb.gemm2_weights_scale, offset, 2.5)
    profiled_step = step
    if args.graph and world == 1:
        from kernelforge_b200.graph import GraphedMoE
        graphed = GraphedMoE(wb, offset, 2.5, T).capture()
        step = graphed

    # local (token, expert) pairs of this rank's GEMMs (for the FLOP count) and the local
    # experts that receive at least one pair (whose weights a step must read)
    idx, _ = B.route(ti.routing_logits, ti.routing_bias, 2.5)
    pairs = int(((idx >= offset) & (idx < offset + E)).sum().item()) if world == 1 else None
    active = int(torch.unique(idx[(idx >= offset) & (idx < offset + E)]).numel()) if world == 1 else None

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    for _ in range(args.warmup):
        step(ti.routing_logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale)
    torch.cuda.synchronize(dev)

    clocks = ClockSampler(dev.index)
    if rank == 0:           # only rank 0's line reports clocks; one sampler keeps the host quiet
        clocks.start()
    time.sleep(0.5)
    stream = torch.cuda.current_stream(dev)

    def timed(k_steps, profile):
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        sev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(k_steps)]
        barrier()
        torch.cuda.synchronize(dev)
        if profile:
            B.profile_begin()
        ev0.record(stream)
        fn = profiled_step if profile else step
        for k in range(k_steps):
            sev[k][0].record(stream)
            fn(ti.routing_logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale)
            sev[k][1].record(stream)
        ev1.record(stream)
        torch.cuda.synchronize(dev)
        prof_ = B.profile_end() if profile else None
        barrier()
        return ev0.elapsed_time(ev1), sorted(a.elapsed_time(b) for a, b in sev), prof_

    # headline: K steps, nothing but the layer in the timed region
    t_wall0 = time.time()
    ms, step_ms, _ = timed(args.steps, False)
    t_wall1 = time.time()
    # the same K steps again with every library launch bracketed by CUDA events (kernel durations)
    _, _, prof = timed(args.steps, True)
    t_wall2 = time.time()
    clocks.stop()
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
        pairs = layer.local_pairs()   # rank 0's GEMM rows in the last step
    ms_per_step = ms / args.steps
    value = world * T * args.steps / (ms / 1e3)

    # End to end through the public API: every step copies its inputs from pinned
    # host memory and its bf16 result back to pinned host memory.  As in a serving
    # loop, the copies run on their own streams and overlap the neighbouring
    # steps' kernels: step k+1's inputs go up and step k-1's result comes down
    # while step k computes (two device input sets, two host output buffers).
    e2e = None
    h_in = [tuple(t.cpu().pin_memory() for t in (ti.routing_logits, ti.routing_bias, ti.hidden_states,
                                                  ti.hidden_states_scale)) for _ in range(2)]
    h_out = [torch.empty((T, H), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    d_in = [tuple(torch.empty_like(t) for t in (ti.routing_logits, ti.routing_bias, ti.hidden_states,
                                                  ti.hidden_states_scale)) for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in h_in[0])
    d2h = h_out[0].numel() * h_out[0].element_size()
    e2e_steps = max(3, min(args.steps, 20))
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = lambda: torch.cuda.Event(enable_timing=False)
    loaded = [ev() for _ in range(e2e_steps)]
    computed = [ev() for _ in range(e2e_steps)]

    def upload(k):
        b = k % 2
        if k >= 2:
            up.wait_event(computed[k - 2])      # step k-2 has finished reading this input set
        with torch.cuda.stream(up):
            for d, h in zip(d_in[b], h_in[b]):
                d.copy_(h, non_blocking=True)
        loaded[k].record(up)

    barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(up)
    stream.wait_event(e0)
    down.wait_event(e0)
    upload(0)
    for k in range(e2e_steps):
        if k + 1 < e2e_steps:
            upload(k + 1)
        stream.wait_event(loaded[k])
        if args.graph and world == 1:
            stream.wait_stream(down)   # the graph reuses one output buffer: step k-1's copy must be done
        o = step(*d_in[k % 2])
        computed[k].record(stream)
        down.wait_event(computed[k])
        o.record_stream(down)
        with torch.cuda.stream(down):
            h_out[k % 2].copy_(o, non_blocking=True)
    down.wait_stream(stream)
    down.wait_stream(up)
    e1.record(down)
    torch.cuda.synchronize(dev)
    e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e_ms = float(t.item())
    # the copies alone, serialised, for one step (how much the overlap hides)
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    c0.record(stream)
    for d, h in zip(d_in[0], h_in[0]):
        d.copy_(h, non_blocking=True)
    h_out[0].copy_(o, non_blocking=True)
    c1.record(stream)
    torch.cuda.synchronize(dev)
    e2e = {"value": world * T * e2e_steps / (e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
           "d2h_bytes_per_step": d2h, "steps": e2e_steps, "copy_ms_per_step_serial": c0.elapsed_time(c1),
           "overlap": "each step's host copies run on side streams beside the neighbouring steps' kernels"}
    if world > 1:
        # a barrier of the peer exchange that gave up in the last step invalidates the numbers; every
        # rank reads its own status word and all of them raise together
        st = torch.tensor([layer.status()], dtype=torch.int64, device=dev)
        torch.distributed.all_reduce(st, op=torch.distributed.ReduceOp.MAX)
        err = ep.peer_status_error(int(st.item()))
        if err:
            raise RuntimeError(err)

    # roofline of the dominant kernel (GEMM1: 2/3 of the layer's FLOPs)
    g1_ms, g1_n = prof["gemm1_swiglu"]
    g2_ms, g2_n = prof["gemm2_weighted"]
    total_launches = sum(n for _, n in prof.values())   # launches in K profiled steps = launches in K timed steps
    roofline = None
    if g1_n and pairs is not None and args.workload == "decode":
        # decode is weight-streaming bound: GEMM1 reads the W13 tiles (and scales) of every active expert
        g1_avg = g1_ms / g1_n
        g1_bytes = active * (W13_BYTES_PER_EXPERT + W13_SCALE_BYTES) + pairs * (H + H // 128 * 4)
        achieved = g1_bytes / (g1_avg / 1e3) / 1e9
        roofline = {"bound": "hbm", "kernel": "gemm1_swiglu", "achieved": achieved, "peak": peaks["hbm_gbs"],
                    "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"], "traffic": None,
                    "peak_note": f"{peaks['source']} HBM copy bandwidth", "avg_launch_ms": g1_avg,
                    "active_experts": active}
    elif g1_n and pairs is not None:
        g1_avg = g1_ms / g1_n
        achieved = GEMM1_FLOP_PER_PAIR * pairs / (g1_avg / 1e3) / 1e12
        peak = 2.0 * peaks["bf16_sustained"]
        # DRAM bytes of one GEMM1 launch from an ncu capture of this exact workload (N = 1, 256 local
        # experts, T = 8192): profiles/launches_ep_layer_T8192.md.  Other workloads: not captured.
        traffic = 12.01e9 if (args.workload == "ep" and world == 1 and T == 8192) else None
        roofline = {"bound": "tensor", "kernel": "gemm1_swiglu", "achieved": achieved, "peak": peak,
                    "unit": "TFLOP/s", "frac": achieved / peak, "traffic": traffic,
                    "traffic_note": "DRAM bytes per launch (ncu dram__bytes_read+write); algorithmic 8.26e9"
                                    if traffic else None,
                    "peak_note": f"FP8 dense = 2 x {peaks['source']} sustained cuBLAS bf16 "
                                 f"({peaks['bf16_sustained']} TFLOP/s)",
                    "avg_launch_ms": g1_avg}
    kernels = {k: {"ms_per_launch": (v[0] / v[1]) if v[1] else None, "launches": v[1],
                   "share": (v[0] / sum(x[0] for x in prof.values())) if v[1] else 0.0}
               for k, v in prof.items()}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = measure_cpu_baseline(T, E, offset)
    try:
        clock_summary = clocks.summary([(t_wall0, t_wall1, "timed steps"),
                                        (t_wall0, t_wall2, "timed steps + the same steps profiled")])
    except Exception as exc:  # noqa: BLE001
        clock_summary = {"sm_mhz": None, "reasons": ["unsampled"], "error": f"{type(exc).__name__}: {exc}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp8_e4m3 (fp32 accumulate)", "data": "synthetic",
            "config": {"workload": name, "tokens_per_gpu": T, "local_experts_per_gpu": E,
                       "global_experts": E_GLOBAL, "hidden": H, "intermediate": I, "top_k": 8,
                       "parallelism": f"ep{world}", "ep_exchange": args.ep_exchange if world > 1 else None,
                       "l2": "inputs larger than L2 (weights stream from HBM)",
                       "pairs_rank0": pairs, "cuda_graph": bool(args.graph and world == 1)},
            "p50_step_ms": step_ms[len(step_ms) // 2], "p90_step_ms": step_ms[int(len(step_ms) * 0.9)],
            "tflops_per_gpu": (FLOP_PER_PAIR * pairs / (ms_per_step / 1e3) / 1e12) if pairs else None,
            "layer_hbm_gbs": (active * (W13_BYTES_PER_EXPERT + W2_BYTES_PER_EXPERT + W13_SCALE_BYTES + W2_SCALE_BYTES)
                              / (ms_per_step / 1e3) / 1e9) if active else None,
            "active_local_experts": active,
            "roofline": roofline, "kernels": kernels, "gpu_launches": total_launches,
            "e2e": e2e, "cpu_baseline": cpu,
            "clocks": clock_summary,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
