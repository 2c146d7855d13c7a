#!/usr/bin/env python
"""Benchmark of the fused DeepSeek-V3 FP8 block-scale MoE layer on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl kernelforge|reference]
                    [--workload ep|prefill|decode] [--tokens T] [--zipf] [--graph]
                    [--ep-exchange p2p|nccl] [--no-cpu-baseline] [--no-extra]

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
step streams them from HBM (no L2 flush needed).  After the timed steps the line
also carries a sampled parity check of the step's output against the fp32
reference ("parity"), and at N = 1 the single-GPU configurations of the metric:
the decode sweep (config 1: p50 microseconds and HBM fraction, L2 flushed before
every call), prefill (config 2: FP8 fraction of GEMM1) and the Zipf-skewed layer
(config 4) ("single_gpu_configs").

--impl reference times the reference algorithm's CPU path (the oracle port of
solution/triton/kernel.py::kernel's PyTorch loop) on this host's cores.  The
layer is cut into 32 equal slices -- slice j routes tokens [jT/32, (j+1)T/32),
runs the expert loop for the local experts e = j (mod 32) with all of their
pairs, and zeroes and casts its share of the output rows -- so 32 consecutive
slices do exactly the work of one layer call.  Each step times one slice (the
next in turn); value = tokens of layer work per measured second.
"""
from __future__ import annotations

import argparse
import hashlib
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
EXPERT_BYTES = W13_BYTES_PER_EXPERT + W2_BYTES_PER_EXPERT + W13_SCALE_BYTES + W2_SCALE_BYTES
TOKEN_IN_BYTES = H + (H // 128) * 4 + E_GLOBAL * 4    # fp8 row, its scales, its routing logits
TOKEN_OUT_BYTES = H * 2                               # bf16 output row
METRIC = "MoE layer tokens/s (FP8 block-scale DeepSeek-V3 layer, T=8192 tokens per GPU, 256 experts EP-sharded)"
CPU_PARTS = 32


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="kernelforge", choices=["kernelforge", "reference"])
    p.add_argument("--workload", default="ep", choices=["ep", "prefill", "decode"])
    p.add_argument("--tokens", type=int, default=None)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-extra", action="store_true", help="skip the single-GPU configurations (N = 1)")
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


def fp8_peak(peaks) -> dict:
    """FP8 dense peak for a kernel timed in short steps: 2 x the burst bf16 cuBLAS figure.  The pool
    measures no FP8 GEMM; the factor 2 is the nominal fp8/bf16 ratio (4.5 / 2.25 PFLOP/s), assumed."""
    return {"peak": 2.0 * peaks["bf16"],
            "peak_note": f"FP8 dense taken as 2 x the {peaks['source']} burst cuBLAS bf16 figure "
                         f"({peaks['bf16']} TFLOP/s); the factor 2 is assumed (no FP8 GEMM is measured)"}


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
class CpuReferenceLayer:
    """The reference algorithm's CPU layer on the bench's workload, cut into equal timed slices.

    The reference's CPU path (``solution/triton/kernel.py:1842-1950``: routing, ``_sort_tokens``,
    then a loop over the active local experts that dequantises each expert's weights and rows and
    runs its two GEMMs and the weighted ``index_add_``), restated in ``oracle/moe_oracle.py``, is
    cut into ``parts`` slices: slice j routes tokens ``[jT/parts, (j+1)T/parts)``, zeroes and
    casts to bf16 that share of the output rows, and runs the expert loop for the local experts
    e = j (mod parts) with all of their pairs (their pair lists taken from the routing of every
    token, made once outside the timing).  The ``parts`` slices together do exactly the work of
    one layer call; every slice is timed on its own.  The expert weights come from a pool of
    ``pool`` generated experts (expert e uses pool entry e mod pool): their values do not change
    the cost of the dense fp32 arithmetic, and generating all 256 would take minutes.  The slices
    time the work; their accumulated output is not the layer's (each slice casts its rows before
    later slices add into them).
    """

    def __init__(self, T: int, num_local: int, offset: int = 0, parts: int = CPU_PARTS, pool: int = 8,
                 seed: int = 1000, routing_bias=None):
        from kernelforge_b200 import synthetic as S
        from oracle import moe_oracle as O
        if T <= 0 or num_local < 1 or offset < 0 or offset + num_local > E_GLOBAL:
            raise ValueError(f"no CPU layer for T={T}, experts [{offset}, {offset + num_local})")
        torch.set_num_threads(os.cpu_count() or 1)
        self.O, self.T, self.E, self.offset, self.parts = O, T, num_local, offset, parts
        self.ti = S.token_inputs(T, seed=seed, routing_bias=routing_bias)
        self.idx, self.w = O.route(self.ti.routing_logits, self.ti.routing_bias, 2.5)
        self.loc = self.idx - offset
        self.pool = [S.expert_weights(offset + e, seed=0) for e in range(min(pool, num_local))]
        self.acc = torch.zeros(T, H, dtype=torch.float32)
        self.out = torch.empty(T, H, dtype=torch.bfloat16)
        self.active = int(torch.unique(self.loc[(self.loc >= 0) & (self.loc < num_local)]).numel())

    def run_part(self, j: int) -> float:
        """Seconds of slice j."""
        O, ti = self.O, self.ti
        t0 = j * self.T // self.parts
        t1 = (j + 1) * self.T // self.parts
        s = time.perf_counter()
        O.route(ti.routing_logits[t0:t1], ti.routing_bias, 2.5)
        self.acc[t0:t1].zero_()
        for e in range(j, self.E, self.parts):
            tok = torch.nonzero((self.loc == e).any(dim=1)).flatten()      # token order (stable)
            if tok.numel() == 0:
                continue
            rows = O.dequant_hidden_rows(ti.hidden_states, ti.hidden_states_scale, tok)
            y = O.expert_forward(rows, *self.pool[e % len(self.pool)])
            rw = self.w[tok, self.offset + e]
            self.acc.index_add_(0, tok, y * rw.unsqueeze(1))
        self.out[t0:t1] = self.acc[t0:t1].to(torch.bfloat16)
        return time.perf_counter() - s

    def describe(self) -> str:
        return (f"reference CPU layer (oracle/moe_oracle.py restatement of kernel.py:1842-1950, PyTorch fp32, "
                f"{torch.get_num_threads()} threads) on T={self.T} tokens and {self.E} local experts "
                f"({self.active} active), cut into {self.parts} slices that together do one layer's work: "
                f"slice j routes 1/{self.parts} of the tokens, casts 1/{self.parts} of the output rows and runs "
                f"the expert loop of the experts e = j (mod {self.parts}); weights from a pool of "
                f"{len(self.pool)} generated experts")


def zipf_cpu_bias():
    from kernelforge_b200 import synthetic as S
    return S.zipf_bias(seed=0)


def measure_cpu_baseline(T: int, num_local: int, offset: int, parts: int = CPU_PARTS, routing_bias=None) -> dict:
    """The ``cpu_baseline`` object of the bench line: the whole layer once, every slice timed (about
    10-30 s of CPU work at the bench's workload).  A failure is reported inside the object (it must
    not cost the measured line it rides on)."""
    try:
        lay = CpuReferenceLayer(T, num_local, offset, parts=parts, routing_bias=routing_bias)
        lay.run_part(0)                                 # warm-up (allocator, thread pool)
        total = sum(lay.run_part(j) for j in range(parts))
        return {"value": T / total, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
                "sample": f"the whole layer once ({parts} slices, {total:.1f} s measured): " + lay.describe()}
    except Exception as exc:  # noqa: BLE001 -- reported in the line, not swallowed
        return {"value": None, "unit": "tokens/s", "error": f"{type(exc).__name__}: {exc}"}


def line_config(name, T, E, world, args, pairs=None):
    """The ``config`` object, the same in both arms."""
    return {"workload": name, "tokens_per_gpu": T, "local_experts_per_gpu": E, "global_experts": E_GLOBAL,
            "hidden": H, "intermediate": I, "top_k": 8, "parallelism": f"ep{world}",
            "ep_exchange": args.ep_exchange if world > 1 else None,
            "l2": "inputs larger than L2 (weights stream from HBM)", "cuda_graph": bool(args.graph and world == 1)}


def run_reference(args, world, rank):
    if rank != 0:
        return
    # the same per-GPU workload and config as this N's own arm; the CPU layer routes the GPU's T
    # tokens over all the experts they reach (all 256 for the expert-parallel layer: the per-token
    # work of the whole job)
    T, E, name = workload_shape(args, args.gpus)
    if args.zipf:
        name += "_zipf1.2"
    lay = CpuReferenceLayer(T, E_GLOBAL if args.workload == "ep" else E,
                            routing_bias=zipf_cpu_bias() if args.zipf else None)
    cores = torch.get_num_threads()
    part = 0
    for _ in range(args.warmup):
        lay.run_part(part % lay.parts)
        part += 1
    times = []
    for _ in range(args.steps):
        times.append(lay.run_part(part % lay.parts))
        part += 1
    total = sum(times)
    value = (T / lay.parts) * args.steps / total
    sample = (f"each step is one slice (1/{lay.parts} of the layer's work, the next slice in turn), timed: "
              + lay.describe())
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": line_config(name, T, E, args.gpus, args),
        "tokens_per_step": T / lay.parts,
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------- parity --
def sampled_parity(out, ti, idx, w, bank_fn, expert_range, n_sample: int = 256, seed: int = 5) -> dict:
    """The step's output on a seeded sample of tokens against the fp32 reference (the oracle's
    expert math on this GPU, ``oracle/moe_oracle.py``), with the layer's acceptance test.

    ``idx``/``w``: the step's routing of these tokens (int32 ids, weights [T, 8]), checked for
    every token against the oracle's routing on the CPU.  ``expert_range`` = (lo, hi): the global
    experts the output covers (the local experts at N = 1, all 256 after the expert-parallel
    exchange); other ids contribute nothing, as in the layer.  ``bank_fn(global_ids)`` returns
    the weights of those experts stacked in the given (ascending) order."""
    from oracle import moe_oracle as O
    T = int(out.shape[0])
    ref_idx, _ = O.route(ti.routing_logits.float().cpu(), ti.routing_bias.cpu(), 2.5)
    routing_exact = bool(torch.equal(idx.long().cpu().sort(dim=1).values, ref_idx.sort(dim=1).values))
    g = torch.Generator().manual_seed(seed)
    sel = torch.randperm(T, generator=g)[:min(T, n_sample)].sort().values.to(out.device)
    sidx = idx[sel].long()
    lo, hi = expert_range
    experts = sorted(e for e in set(sidx.flatten().tolist()) if lo <= e < hi)
    if experts:
        wb = bank_fn(experts)
        remap = torch.full((E_GLOBAL,), -1, dtype=torch.long, device=out.device)
        remap[torch.tensor(experts, device=out.device)] = torch.arange(len(experts), device=out.device)
        ref = O.moe_experts(remap[sidx].to(torch.int32), w[sel], ti.hidden_states[sel],
                            ti.hidden_states_scale[:, sel], *wb, 0).to(torch.bfloat16)
    else:   # no sampled token reaches an expert the output covers: zero rows
        ref = torch.zeros((sel.numel(), H), dtype=torch.bfloat16, device=out.device)
    res = O.check_tolerance(out[sel], ref)
    return {"ok": bool(res["ok"] and routing_exact), "routing_exact_all_tokens": routing_exact,
            "tokens_checked": int(sel.numel()), "experts_checked": len(experts),
            "max_abs_err": res["max_abs_err"], "max_abs_ref": res["max_abs_ref"], "frac_within": res["frac_within"],
            "tolerance": "max|err| <= 1e-2 max|ref|, >= 99.9% within 1e-2 + 2e-2 |ref|; routing sets exact"}


# ------------------------------------------------- single-GPU configurations --
def time_calls(fn, n: int, warmup: int, flush=None):
    """Per-call device milliseconds (CUDA events on the current stream), sorted; with ``flush`` (a
    buffer larger than L2) it is rewritten before every call, outside the timed events."""
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        fn()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    for a, b in evs:
        if flush is not None:
            flush.add_(1)
        a.record(stream)
        fn()
        b.record(stream)
    torch.cuda.synchronize()
    return sorted(a.elapsed_time(b) for a, b in evs)


def single_gpu_configs(B, S, dev, peaks, bank256) -> dict:
    """Configs 1, 2 and 4 of the headline metric on this GPU, each timed and with its roofline."""
    fp8 = fp8_peak(peaks)
    res = {"peaks": {"hbm_gbs": peaks["hbm_gbs"], "fp8_tflops": fp8["peak"], "note": fp8["peak_note"]}}
    wb32 = S.expert_bank(32, 0, seed=0, device=dev)
    flush = torch.zeros(256 << 20, dtype=torch.uint8, device=dev)     # 256 MB > L2 (126 MB)

    def layer(ti, wb):
        return lambda: B.kernel(ti.routing_logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale,
                                wb.gemm1_weights, wb.gemm1_weights_scale, wb.gemm2_weights, wb.gemm2_weights_scale,
                                0, 2.5)

    def counts(ti, E):
        idx, _ = B.route(ti.routing_logits, ti.routing_bias, 2.5)
        loc = idx[(idx >= 0) & (idx < E)]
        return int(loc.numel()), int(torch.unique(loc).numel())

    def kernel_ms(fn, reps=10):
        B.profile_begin()
        for _ in range(reps):
            fn()
        torch.cuda.synchronize()
        prof = B.profile_end()
        return {k: v[0] / v[1] for k, v in prof.items() if v[1]}

    # config 1: decode sweep, 32 local experts, weight-streaming bound
    dec = {}
    for T in (1, 2, 4, 8, 16, 32, 64):
        ti = S.token_inputs(T, seed=300 + T, device=dev)
        fn = layer(ti, wb32)
        ms = time_calls(fn, 200, 10, flush=flush)
        pairs, active = counts(ti, 32)
        nbytes = active * EXPERT_BYTES + T * (TOKEN_IN_BYTES + TOKEN_OUT_BYTES) + 512
        p50 = ms[len(ms) // 2]
        km = kernel_ms(fn)
        g1 = km.get("gemm1_swiglu")
        g1_bytes = active * (W13_BYTES_PER_EXPERT + W13_SCALE_BYTES) + pairs * (H + (H // 128) * 4)
        dec[f"T{T}"] = {"p50_us": 1e3 * p50, "p90_us": 1e3 * ms[int(len(ms) * 0.9)], "active_experts": active,
                        "pairs": pairs, "layer_bytes": nbytes, "layer_hbm_gbs": nbytes / (p50 / 1e3) / 1e9,
                        "layer_hbm_frac": nbytes / (p50 / 1e3) / 1e9 / peaks["hbm_gbs"],
                        "gemm1_hbm_frac": (g1_bytes / (g1 / 1e3) / 1e9 / peaks["hbm_gbs"]) if g1 else None,
                        "kernel_us": {k: 1e3 * v for k, v in km.items()}}
    res["config1_decode"] = {"local_experts": 32, "l2": "256 MB buffer rewritten before every timed call",
                             "calls": 200, "bytes": "active experts' W13+W2+scales + token rows in and out",
                             "sweep": dec}

    # config 2: prefill, 32 local experts, uniform routing
    pre = {}
    for T in (4096, 16384):
        ti = S.token_inputs(T, seed=400 + T, device=dev)
        fn = layer(ti, wb32)
        ms = time_calls(fn, 20, 3)
        pairs, active = counts(ti, 32)
        p50 = ms[len(ms) // 2]
        km = kernel_ms(fn, 5)
        g1 = km["gemm1_swiglu"]
        pre[f"T{T}"] = {"p50_ms": p50, "tokens_per_s": T / (p50 / 1e3), "pairs": pairs,
                        "layer_tflops": FLOP_PER_PAIR * pairs / (p50 / 1e3) / 1e12,
                        "layer_fp8_frac": FLOP_PER_PAIR * pairs / (p50 / 1e3) / 1e12 / fp8["peak"],
                        "gemm1_tflops": GEMM1_FLOP_PER_PAIR * pairs / (g1 / 1e3) / 1e12,
                        "gemm1_fp8_frac": GEMM1_FLOP_PER_PAIR * pairs / (g1 / 1e3) / 1e12 / fp8["peak"],
                        "kernel_ms": km}
    res["config2_prefill"] = {"local_experts": 32, "sweep": pre}

    # config 4: Zipf(1.2)-skewed routing over all 256 experts on this GPU
    if bank256 is not None:
        zb = S.zipf_bias(seed=0).to(dev)
        zz = {}
        for T in (128, 1024, 4096, 16384):
            ti = S.token_inputs(T, seed=500 + T, device=dev, routing_bias=zb)
            fn = layer(ti, bank256)
            ms = time_calls(fn, 10 if T >= 4096 else 30, 3)
            pairs, active = counts(ti, 256)
            p50 = ms[len(ms) // 2]
            km = kernel_ms(fn, 3)
            g1 = km["gemm1_swiglu"]
            zz[f"T{T}"] = {"p50_ms": p50, "tokens_per_s": T / (p50 / 1e3), "pairs": pairs, "active_experts": active,
                           "layer_hbm_frac": (active * EXPERT_BYTES / (p50 / 1e3) / 1e9) / peaks["hbm_gbs"],
                           "gemm1_fp8_frac": GEMM1_FLOP_PER_PAIR * pairs / (g1 / 1e3) / 1e12 / fp8["peak"],
                           "kernel_ms": km}
        res["config4_zipf_256_experts"] = {"sweep": zz}
    del wb32, flush
    return res


# DRAM bytes per GEMM1 launch from ncu captures (dram__bytes_read.sum + dram__bytes_write.sum), valid
# only for the kernel source they were captured on: the line reports null once the source changes.
TRAFFIC = {
    "ep_layer_T8192_per_gpu_256_experts": {
        "bytes": 8 * (1_223_874_560 + 32_855_040), "source_sha16": "8099a11cbb49f7bd",
        "note": "ncu dram__bytes_read.sum + dram__bytes_write.sum of gemm1_swiglu_kernel on a 1/8 replica "
                "(8192 tokens, 32 local experts: the same pairs per expert), scaled by 8 experts' worth"},
}


GEMM_SOURCES = ("kf_grouped_gemm.cu", "kf_internal.cuh", "kf_ptx.cuh", "kf_fp8.cuh")
GEMM2_MARK = b"// A GEMM2 work unit as the promotion warps see it"


def gemm_source_sha16() -> str:
    """Hash of the source GEMM1 is compiled from: its file up to the end of the GEMM1 kernel (the
    GEMM2 kernel and the launchers follow) and the headers it includes."""
    h = hashlib.sha256()
    for name in GEMM_SOURCES:
        with open(os.path.join(ROOT, "kernelforge_b200", "csrc", name), "rb") as f:
            text = f.read()
        if name == "kf_grouped_gemm.cu":
            text = text[:text.index(GEMM2_MARK)]
        h.update(text)
    return h.hexdigest()[:16]


def gemm1_traffic(name: str):
    rec = TRAFFIC.get(name)
    if rec is None:
        return None, "no ncu capture of this workload"
    if gemm_source_sha16() != rec["source_sha16"]:
        return None, "the GEMM kernels changed since the ncu capture"
    return rec["bytes"], rec["note"]


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

    layer = None
    if world > 1:
        from kernelforge_b200 import ep
        layer = ep.ExpertParallelMoE(wb, offset, E, exchange=args.ep_exchange)

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

    # At N > 1, rank 0 first times its own shard on one GPU at the same pair load an expert-parallel
    # rank carries (N x T tokens routed over all experts give each shard of 256/N experts about
    # 8 x T pairs): the baseline of the scaling efficiency at equal per-GPU work.
    equal_load = None
    if world > 1 and args.workload == "ep":
        if rank == 0:
            t_ref = world * T
            tr_in = S.token_inputs(t_ref, seed=99, device=dev)
            ref_call = lambda: B.kernel(tr_in.routing_logits, tr_in.routing_bias, tr_in.hidden_states,
                                        tr_in.hidden_states_scale, wb.gemm1_weights, wb.gemm1_weights_scale,
                                        wb.gemm2_weights, wb.gemm2_weights_scale, offset, 2.5)
            ms_ref = time_calls(ref_call, 5, 3)
            ridx, _ = B.route(tr_in.routing_logits, tr_in.routing_bias, 2.5)
            ref_pairs = int(((ridx >= offset) & (ridx < offset + E)).sum().item())
            equal_load = {"tokens": t_ref, "local_experts": E, "pairs": ref_pairs, "p50_ms": ms_ref[len(ms_ref) // 2]}
            del tr_in
            B.release_workspaces()
            torch.cuda.empty_cache()
        barrier()

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

    # End to end through the public API: every step copies its inputs from pinned host
    # memory and its bf16 result back to pinned host memory.  As in a serving
    # loop, the copies run on their own streams and overlap the neighbouring
    # steps' kernels: step k+1's inputs go up and step k-1's result comes down
    # while step k computes (two device input sets, two host output buffers).
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
    else:
        B.check(dev)        # device status of the timed calls (raises on a set bit)

    # parity of one more step (all ranks run it: the exchange is collective), checked on rank 0
    out = profiled_step(ti.routing_logits, ti.routing_bias, ti.hidden_states, ti.hidden_states_scale)
    torch.cuda.synchronize(dev)
    parity = None
    if rank == 0:
        ridx, rw = B.route(ti.routing_logits, ti.routing_bias, 2.5)
        if world == 1:
            def bank_fn(experts):
                sel = torch.tensor(experts, device=dev) - offset
                return (wb.gemm1_weights[sel], wb.gemm1_weights_scale[sel], wb.gemm2_weights[sel],
                        wb.gemm2_weights_scale[sel])
        else:
            def bank_fn(experts):           # every rank's experts, generated here by global id
                ws = [S.expert_weights(g, seed=0, device=dev) for g in experts]
                return tuple(torch.stack([x[i] for x in ws]) for i in range(4))
        try:
            parity = sampled_parity(out, ti, ridx, rw, bank_fn, (offset, offset + E) if world == 1 else (0, E_GLOBAL))
        except Exception as exc:  # noqa: BLE001 -- reported in the line
            parity = {"ok": False, "error": f"{type(exc).__name__}: {exc}"}
        if world > 1:
            parity["note"] = (f"rank 0's tokens after the exchange over {world} ranks, against all the experts "
                              f"they reach (weights regenerated on rank 0 by global expert id)")
    barrier()

    # roofline of the dominant kernel (GEMM1: 2/3 of the layer's FLOPs)
    g1_ms, g1_n = prof["gemm1_swiglu"]
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
        fp8 = fp8_peak(peaks)
        traffic, tnote = gemm1_traffic(name) if world == 1 else (None, "captured at N = 1 only")
        roofline = {"bound": "tensor", "kernel": "gemm1_swiglu", "achieved": achieved, "peak": fp8["peak"],
                    "unit": "TFLOP/s", "frac": achieved / fp8["peak"], "traffic": traffic, "traffic_note": tnote,
                    "algorithmic_bytes": (active or 0) * (W13_BYTES_PER_EXPERT + W13_SCALE_BYTES)
                                         + pairs * (H + (H // 128) * 4 + 2 * I + (I // 128) * 4),
                    "peak_note": fp8["peak_note"], "avg_launch_ms": g1_avg,
                    "frac_of_2x_sustained_bf16": achieved / (2.0 * peaks["bf16_sustained"])}
    kernels = {k: {"ms_per_launch": (v[0] / v[1]) if v[1] else None, "launches": v[1],
                   "share": (v[0] / sum(x[0] for x in prof.values())) if v[1] else 0.0}
               for k, v in prof.items()}

    extra = None
    if rank == 0 and world == 1 and not args.no_extra:
        try:
            extra = single_gpu_configs(B, S, dev, peaks, wb if E == E_GLOBAL else None)
        except Exception as exc:  # noqa: BLE001 -- reported in the line
            extra = {"error": f"{type(exc).__name__}: {exc}"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = measure_cpu_baseline(T, E, offset, routing_bias=zipf_cpu_bias() if args.zipf else None)
    try:
        clock_summary = clocks.summary([(t_wall0, t_wall1, "timed steps"),
                                        (t_wall0, t_wall2, "timed steps + the same steps profiled")])
    except Exception as exc:  # noqa: BLE001
        clock_summary = {"sm_mhz": None, "reasons": ["unsampled"], "error": f"{type(exc).__name__}: {exc}"}

    if equal_load is not None:
        equal_load["efficiency_vs_ep_step"] = equal_load["p50_ms"] / ms_per_step
        equal_load["ep_pairs_rank0"] = pairs
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp8_e4m3 (fp32 accumulate)", "data": "synthetic",
            "config": line_config(name, T, E, world, args),
            "pairs_rank0": pairs,
            "p50_step_ms": step_ms[len(step_ms) // 2], "p90_step_ms": step_ms[int(len(step_ms) * 0.9)],
            "tflops_per_gpu": (FLOP_PER_PAIR * pairs / (ms_per_step / 1e3) / 1e12) if pairs else None,
            "layer_hbm_gbs": (active * EXPERT_BYTES / (ms_per_step / 1e3) / 1e9) if active else None,
            "active_local_experts": active,
            "roofline": roofline, "kernels": kernels, "gpu_launches": total_launches,
            "e2e": e2e, "cpu_baseline": cpu, "parity": parity, "equal_load_1gpu": equal_load,
            "single_gpu_configs": extra,
            "clocks": clock_summary,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
