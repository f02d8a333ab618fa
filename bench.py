#!/usr/bin/env python
"""Benchmark of the dyn-quant fused split GEMV on B200.

Metric: microseconds per GEMV and achieved HBM GB/s (fraction of the measured
B200 copy bandwidth) at Llama-2 7B/70B dimensions, INT4 group 128, k = 3.0.
A "step" is one batch-1 pass through the GEMVs of one workload:

  llama2_70b_mlp (default) gate 8192->28672, up 8192->28672, down 28672->8192, 3 % outliers
  llama2_70b_q   q_proj 8192->8192, 3 % outliers
  llama2_7b_mlp  gate 4096->11008, up 4096->11008, down 11008->4096, 1 % outliers
  llama2_7b_q    q_proj 4096->4096, 2 % outliers
  sweep_8192     one 8192x8192 GEMV (--batch, --frac, --k, --dist: the outlier / batch sweep)
  mixtral_moe    Mixtral-8x7B FFN decode step: 8 experts, 16 tokens, top-2

value = whole-job algorithmic bytes / time (GB/s; inputs resident in HBM; the
K timed steps are one CUDA graph of back-to-back launches; weights rotate over
enough copies that every step reads them from HBM, not L2).  Algorithmic bytes
per GEMV = d_out*d_in/2 (INT4) + 4*d_out*d_in/128 (FP16 scale + zero)
+ 2*d_out*n_o (FP16 outlier columns, n_o = detected outliers; for a batch the
union of the vectors' masks) + 2*m*d_in (x) + 2*m*d_out (y).

Weights and activations are seeded synthetic tensors (dyn_quant/synth.py):
weight matrix i of a workload is synth.weights(d_out, d_in, seed=100 + i) in
both arms; the GPU arm's extra rotating copies are row rotations of it.

One process per GPU.  Under torchrun (N > 1) the 70B workloads are
row-sharded, as a 70B model is deployed: each rank holds whole 16-row blocks
of the weights, runs the split GEMV on its slice with the same x, and the
output slices are gathered inside every GEMV kernel over NVLink peer memory
(--gather nccl: an NCCL all-gather after every GEMV instead) ("scaling":
"strong": the total work is the workload's, whatever N).  The 7B and sweep workloads fit one GPU
and run as N independent replicas ("scaling": "weak"); --shard overrides
either choice.  The time is the max over ranks.  At N = 1 the line also
carries extra blocks (7B MLP, 7B q_proj, the Mixtral MoE step and one point
of the outlier / batch sweep), each with its own per-GEMV numbers.

--impl reference times the reference's split GEMV restated on the CPU (the
reference has no CPU GEMV of its own; this is the oracle port, OpenMP over
rows) on the host cores, same workload, config and metric; under torchrun
only rank 0 runs it (one host) and it loads no GPU library.
"""
from __future__ import annotations

import argparse
import ctypes as C
import importlib.util
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "dyn-quant_b200")
for _p in (ROOT, PKG_DIR):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

METRIC = "µs per GEMV and achieved HBM GB/s (% of B200 peak) at Llama-2 7B/70B dims"
L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0
K_OUTLIER = 3.0

# name -> list of (gemv name, d_out, d_in, outlier fraction, activation key)
WORKLOADS = {
    "llama2_7b_mlp": [("gate", 11008, 4096, 0.01, "h"), ("up", 11008, 4096, 0.01, "h"),
                      ("down", 4096, 11008, 0.01, "ff")],
    "llama2_7b_q": [("q", 4096, 4096, 0.02, "h")],
    "llama2_70b_mlp": [("gate", 28672, 8192, 0.03, "h"), ("up", 28672, 8192, 0.03, "h"),
                       ("down", 8192, 28672, 0.03, "ff")],
    "llama2_70b_q": [("q", 8192, 8192, 0.03, "h")],
    # the outlier / batch sweep: one 8192 x 8192 GEMV (--batch, --frac, --k, --dist)
    "sweep_8192": [("w", 8192, 8192, 0.01, "h")],
}

# Mixtral-8x7B-shaped MoE FFN decode step: E experts (w1/w3 D->F, w2 F->D),
# T tokens with top-K experts drawn uniformly from a seed.
MOE_WORKLOADS = {
    "mixtral_moe": dict(E=8, D=4096, F=14336, T=16, K=2, frac=0.02),
}

# Extra blocks of the default N = 1 line: (workload, batch, outlier fraction or None, k, dist).
EXTRAS = [("llama2_7b_mlp", 1, None, K_OUTLIER, "normal"), ("llama2_7b_q", 1, None, K_OUTLIER, "normal"),
          ("sweep_8192", 16, 0.05, K_OUTLIER, "normal"), ("mixtral_moe", 1, None, K_OUTLIER, "normal")]


class WL:
    """One measured workload: its name and the sweep parameters."""

    def __init__(self, name: str, batch: int = 1, frac: float | None = None, k: float = K_OUTLIER,
                 dist: str = "normal") -> None:
        self.name, self.batch, self.frac, self.k, self.dist = name, batch, frac, k, dist

    @classmethod
    def from_args(cls, args) -> "WL":
        return cls(args.workload, args.batch, args.frac, args.k, args.dist)


def gemv_bytes(d_out: int, d_in: int, n_o: int, m: int = 1) -> int:
    """Algorithmic bytes of one (batched) split GEMV: INT4 codes, FP16 scale and
    zero, the FP16 columns of the n_o outlier channels (for m > 1 the union of
    the vectors' masks), m activation vectors and m outputs."""
    return d_out * d_in // 2 + 4 * d_out * (d_in // 128) + 2 * d_out * n_o + 2 * m * (d_in + d_out)


def shard_mode(wl: WL, shard: str) -> str:
    """How N > 1 ranks split a GEMV workload (see --shard)."""
    if shard != "auto":
        return shard
    return "rows" if wl.name.startswith("llama2_70b") else "replicas"


def workload_spec(wl: WL):
    """The workload's GEMVs, with the fraction override applied."""
    spec = WORKLOADS[wl.name]
    if wl.frac is not None:
        spec = [(n, o, i, wl.frac, key) for n, o, i, _, key in spec]
    return spec


_SYNTH = None


def synth():
    """dyn_quant/synth.py loaded by file path: the CPU legs use the seeded
    generators without importing the dyn_quant package (and its GPU library)."""
    global _SYNTH
    if _SYNTH is None:
        spec = importlib.util.spec_from_file_location("dq_bench_synth", os.path.join(PKG_DIR, "dyn_quant", "synth.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        _SYNTH = mod
    return _SYNTH


def weights_np(d_out: int, d_in: int, gi: int) -> np.ndarray:
    """Weight matrix gi of a workload (both arms)."""
    return synth().weights(d_out, d_in, seed=100 + gi)


def activations(wl: WL, seed_base: int = 0):
    """Seeded activations per key (numpy f16): [d_in], or [batch, d_in] with
    vector t drawn from seed + t."""
    S = synth()
    acts = {}
    for name, d_out, d_in, frac, key in workload_spec(wl):
        if key not in acts:
            seed = seed_base + (1 if key == "h" else 2)
            if wl.batch == 1:
                acts[key] = S.activation(d_in, frac, seed=seed, dist=wl.dist)
            else:
                acts[key] = S.activations(wl.batch, d_in, frac, seed=seed, dist=wl.dist)
    return acts


def workload_config(wl: WL, world: int, shard: str, gather: str) -> dict:
    """The line's `config`: the workload and how it is run at this N (the
    same dict in both arms)."""
    spec = workload_spec(wl)
    sharded = world > 1 and shard_mode(wl, shard) == "rows"
    if sharded:
        par = (f"row-sharded over {world} GPUs, the output slices gathered "
               + ("by each GEMV kernel over NVLink peer memory" if gather == "peer" else
                  "by an NCCL all-gather after every GEMV"))
    elif world > 1:
        par = f"{world} independent replicas (data parallel, no collective)"
    else:
        par = "1 GPU"
    return {"workload": wl.name, "gemvs": [[n, o, i] for n, o, i, *_ in spec], "batch": wl.batch, "group": 128,
            "outlier_k": wl.k, "outlier_frac": spec[0][3], "dist": wl.dist,
            "weights": "synth.weights(d_out, d_in, seed=100 + i), FP16 N(0, 1/d_in)",
            "l2": "inputs larger than L2: the GPU arm's steps rotate over weight copies totalling >= 3x L2",
            "parallelism": par}


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self._t:
            self._t.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [v.strip() for v in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def measured_peak_gbs():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "of measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "of fallback"


def ncu_traffic(workload: str, batch: int):
    """DRAM bytes (read + write) per algorithmic byte of the workload's split
    GEMV launches, from the committed ncu summary profiles/ncu_traffic.json
    (one capture on one GPU), and the summary it comes from."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(p) as f:
            entry = json.load(f).get(f"{workload}/m{batch}")
    except (OSError, ValueError):
        return None, None
    if not entry:
        return None, None
    return entry["dram_bytes_per_launch"] / entry["algorithmic_bytes_per_launch"], entry.get("source")


# ---------------------------------------------------------------------------
# CPU legs (oracle port of the reference's split GEMV)
# ---------------------------------------------------------------------------
def cpu_prepare(wl: WL):
    import oracle as O
    acts = activations(wl)
    mats = []
    for i, (name, d_out, d_in, frac, key) in enumerate(workload_spec(wl)):
        w = weights_np(d_out, d_in, i)
        mats.append((name, w, *O.quantize(w), acts[key]))
    return mats


def cpu_step(mats, k: float):
    """One step on the host: every GEMV, each activation vector separately
    (the reference computes one vector per call)."""
    import oracle as O
    total = 0
    for name, w, packed, scales, zeros, x in mats:
        xs = x.reshape(-1, w.shape[1])
        union = np.zeros(w.shape[1], bool)
        for row in xs:
            _, _, mask = O.split_gemv(packed, scales, zeros, w, row, k)
            union |= mask.astype(bool)
        total += gemv_bytes(w.shape[0], w.shape[1], int(union.sum()), xs.shape[0])
    return total


def cpu_baseline(wl: WL, budget_s: float = 10.0) -> dict:
    import oracle as O
    cores = os.cpu_count() or 1
    O.set_num_threads(cores)
    mats = cpu_prepare(wl)
    cpu_step(mats, wl.k)  # warm
    t0 = time.perf_counter()
    nbytes, n = 0, 0
    while True:
        nbytes += cpu_step(mats, wl.k)
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    gb_s = nbytes / dt / 1e9
    return {"value": round(gb_s, 3), "unit": "GB/s", "cores": O.num_threads(), "kind": "port",
            "sample": f"{n} full {wl.name} steps (split GEMV incl. detection, same weights and activations as the "
                      f"GPU arm's first weight copy) in {dt:.1f} s, OpenMP over rows, oracle/dq_oracle.c -O3",
            "us_per_gemv": round(dt / (n * len(mats)) * 1e6, 1)}


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    import oracle as O
    wl = WL.from_args(args)
    if wl.name in MOE_WORKLOADS:
        return run_moe_reference(args, rank, world)
    cores = os.cpu_count() or 1
    O.set_num_threads(cores)
    mats = cpu_prepare(wl)
    for _ in range(args.warmup):
        cpu_step(mats, wl.k)
    t0 = time.perf_counter()
    nbytes = 0
    for _ in range(args.steps):
        nbytes += cpu_step(mats, wl.k)
    dt = time.perf_counter() - t0
    value = nbytes / dt / 1e9
    ngemv = len(mats)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "fixed (one host)", "vs_baseline": None, "dtype": "w4a16 (fp32 accumulate)",
        "data": "synthetic (seeded N(0,1/d_in) weights, N(0,1) activations with U[10,100] outliers)",
        "config": workload_config(wl, world, args.shard, args.gather),
        "execution": f"rank 0 only, on its host's {O.num_threads()} cores (the other ranks exit without work)",
        "us_per_gemv": round(dt / (args.steps * ngemv) * 1e6, 2),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": O.num_threads(), "kind": "port",
                         "sample": f"{args.steps} full {wl.name} steps on the host cores (the reference ships no "
                                   f"CPU split GEMV; this is its kernel restated in C, OpenMP over rows)"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU legs
# ---------------------------------------------------------------------------
def init_nccl(dev) -> None:
    """The process group (nccl) with its communicator created eagerly, while
    file descriptor 1 points at stderr: NCCL's own start-up lines then stay
    out of stdout, which carries rank 0's one JSON line."""
    import datetime
    import torch.distributed as dist
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    try:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        dist.barrier()
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)


def graph_time_us(stream, g, n: int) -> float:
    """Mean µs per launch of a graph of n launches (one warm replay first)."""
    import torch
    with torch.cuda.stream(stream):
        g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        g.replay()
        e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) * 1e3 / n


def gemv_block(args, wl: WL, rank: int, world: int, dev, main: bool) -> dict:
    """Measure one GEMV workload; returns the fields of its JSON line (rank 0)
    or of its extra block."""
    import torch
    import torch.distributed as dist

    import dyn_quant
    from dyn_quant import _lib
    from dyn_quant.sharded import shard_rows

    L = _lib.lib()
    spec = workload_spec(wl)
    M = wl.batch
    sharded = world > 1 and shard_mode(wl, args.shard) == "rows"
    peer = sharded and args.gather == "peer"  # the gather fused into the GEMV kernel
    acts_np = activations(wl, 0 if sharded else 1000 * rank)
    acts = {k: torch.from_numpy(v).to(dev) for k, v in acts_np.items()}
    rows = [shard_rows(o, world, rank) if sharded else (0, o, o) for _, o, _, _, _ in spec]

    # detected outliers per activation (the mask the kernel applies; for a
    # batch, the union of the vectors' masks, whose FP16 columns are read)
    n_o = {}
    for key, x in acts.items():
        masks = [dyn_quant.detect_outliers(r, wl.k)[0] for r in x.reshape(-1, x.shape[-1])]
        n_o[key] = int(torch.stack(masks).any(0).sum().item())
    step_bytes = sum(gemv_bytes(o, i, n_o[key], M) for _, o, i, _, key in spec)
    job_step_bytes = step_bytes  # the whole job's: replicas add theirs
    if world > 1 and not sharded:
        t = torch.tensor([step_bytes], dtype=torch.float64, device=dev)
        dist.all_reduce(t)
        job_step_bytes = int(t.item())
    local_bytes = [gemv_bytes(max(r1 - r0, 0), i, n_o[key], M)
                   for (_, _, i, _, key), (r0, r1, _) in zip(spec, rows)]
    n_gemv = len(spec)
    kernels_per_gemv = 1 if M == 1 else 3  # batched: plan, INT4 part, FP16 part

    # weight copies, rotated so each step reads its weights from HBM: copy 0 is
    # the seeded matrix (this rank's rows), the others row rotations of it
    n_sets = max(2, math.ceil(3 * L2_BYTES / max(sum(local_bytes), 1)))
    if args.max_sets:
        n_sets = min(n_sets, args.max_sets)  # profiling runs: ncu flushes caches itself
    sets = [[] for _ in range(n_sets)]
    for gi, (name, d_out, d_in, frac, key) in enumerate(spec):
        r0, r1, per = rows[gi]
        if r1 <= r0:
            raise SystemExit(f"{name}: {d_out} rows do not give every one of {world} ranks a row block")
        w0 = torch.from_numpy(weights_np(d_out, d_in, gi)[r0:r1]).to(dev)
        n_rows = r1 - r0
        if peer and n_rows < per:  # every rank runs the same shape: zero rows pad the last slices
            w0 = torch.cat([w0, torch.zeros(per - n_rows, d_in, dtype=w0.dtype, device=dev)])
            n_rows = per
        for s in range(n_sets):
            w = w0 if s == 0 else torch.roll(w0, shifts=s * 97, dims=0).contiguous()
            lin = dyn_quant.DynQuantLinear(d_in, n_rows, wl.k)
            lin.load_weight(w)
            del w
            sets[s].append(lin)
        del w0
    torch.cuda.synchronize()

    outs = [torch.zeros(M * per, dtype=torch.float16, device=dev) for (_, _, per) in rows]
    fulls = [torch.empty(world * M * per, dtype=torch.float16, device=dev) for (_, _, per) in rows]
    ws_bytes = max(L.dq_workspace_bytes(r1 - r0, i) if M == 1 else L.dq_workspace_bytes_batched(r1 - r0, i, M)
                   for (_, _, i, _, _), (r0, r1, _) in zip(spec, rows))
    wspace = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)  # zero-filled once
    structs = [[_lib.weights(lin.packed.data_ptr(), lin.scales.data_ptr(), lin.zeros.data_ptr(), None,
                             lin.fp16_w.data_ptr(), lin.d_out, lin.d_in, lin._native.data_ptr()) for lin in mods]
               for mods in sets]

    gathers = None
    if peer:
        from dyn_quant.sharded import PeerGather
        if M != 1:
            raise SystemExit("--gather peer runs batch 1")
        gathers = [PeerGather(per, o, None, dev) for (_, o, _, _, _), (_, _, per) in zip(spec, rows)]

    def launch_gemv(s: int, gi: int, stream, gather: bool = True, x=None, split: bool = True):
        key = spec[gi][4]
        xs = acts[key] if x is None else x
        if not split:
            st = L.dq_int4_gemv(C.byref(structs[s][gi]), C.c_void_p(xs.data_ptr()), C.c_void_p(outs[gi].data_ptr()),
                                C.c_void_p(wspace.data_ptr()), ws_bytes, C.c_void_p(stream.cuda_stream))
        elif peer:  # one kernel: this rank's rows, then every rank's rows into the full y
            st = L.dq_split_gemv_gather(C.byref(structs[s][gi]), C.c_void_p(xs.data_ptr()),
                                        C.c_void_p(fulls[gi].data_ptr()), wl.k, C.c_void_p(wspace.data_ptr()),
                                        ws_bytes, C.byref(gathers[gi].desc), C.c_void_p(stream.cuda_stream))
        elif M == 1:
            st = L.dq_split_gemv(C.byref(structs[s][gi]), C.c_void_p(xs.data_ptr()),
                                 C.c_void_p(outs[gi].data_ptr()), wl.k, C.c_void_p(wspace.data_ptr()),
                                 ws_bytes, C.c_void_p(stream.cuda_stream))
        else:
            st = L.dq_split_gemv_batched(C.byref(structs[s][gi]), C.c_void_p(xs.data_ptr()),
                                         C.c_void_p(outs[gi].data_ptr()), M, wl.k, C.c_void_p(wspace.data_ptr()),
                                         ws_bytes, C.c_void_p(stream.cuda_stream))
        if st != 0:
            raise RuntimeError(f"GEMV: {_lib.status_string(st)}")
        if split and sharded and not peer and gather:
            dist.all_gather_into_tensor(fulls[gi], outs[gi])

    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for gi in range(n_gemv):  # first calls: kernel attributes, module load
            launch_gemv(0, gi, stream)
            if M == 1 and world == 1:
                launch_gemv(0, gi, stream, split=False)
    stream.synchronize()

    # Graphs of back-to-back launches (no events between kernels, so each launch
    # overlaps its predecessor's tail as it would in a decode step).
    def capture(launches, gather: bool = True, split: bool = True):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            cur = torch.cuda.current_stream()
            for s, gi in launches:
                launch_gemv(s, gi, cur, gather, split=split)
        return g

    def steps(first: int, count: int):
        return [((first + i) % n_sets, gi) for i in range(count) for gi in range(n_gemv)]

    warm_graph = capture(steps(0, max(args.warmup, n_sets)))
    timed_graph = capture(steps(0, args.steps))
    # per-GEMV graphs: one shape at a time, outside the timed region (with the
    # gather fused, the kernel with its gather; with NCCL, the kernel alone)
    per_gemv_graphs = [capture([(i % n_sets, gi) for i in range(args.steps)], gather=False) for gi in range(n_gemv)]
    # For context, the INT4-only GEMV (the reference's int4_gemv: no detection,
    # no FP16 columns) on the same weights, timed the same way (batch 1, one GPU).
    int4_graphs = ([capture([(i % n_sets, gi) for i in range(args.steps)], gather=False, split=False)
                    for gi in range(n_gemv)] if (M == 1 and world == 1) else [])
    torch.cuda.synchronize()

    with torch.cuda.stream(stream):
        warm_graph.replay()  # >= W untimed warm-up steps
    stream.synchronize()

    sampler = ClockSampler(dev.index) if (main and not args.no_clocks) else None
    if sampler:
        sampler.start()

    def soak(seconds: float):
        t_end = time.perf_counter() + seconds
        with torch.cuda.stream(stream):
            while time.perf_counter() < t_end:
                for _ in range(10):
                    warm_graph.replay()
                stream.synchronize()

    soak(args.soak if main else 0.1)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        t_start.record(stream)
        timed_graph.replay()
        t_end.record(stream)
    stream.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    soak(args.soak if main else 0.0)
    clocks = sampler.stop() if sampler else None

    elapsed_ms = t_start.elapsed_time(t_end)
    if world > 1:
        t = torch.tensor([elapsed_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())

    per_gemv_us = [graph_time_us(stream, g, args.steps) for g in per_gemv_graphs]
    int4_us = [graph_time_us(stream, g, args.steps) for g in int4_graphs]

    # The split GEMV kernel is the dominant (on one GPU the only) kernel: its
    # average launch duration is the timed region over the launches, and
    # achieved = algorithmic bytes per launch / that duration.  Sharded runs
    # time the kernel alone in the per-GEMV graphs (the timed region also
    # holds the gathers).
    peak, peak_note = measured_peak_gbs()
    if sharded:
        achieved = sum(local_bytes) / (sum(per_gemv_us) * 1e-6) / 1e9
    else:
        achieved = sum(local_bytes) * args.steps / (elapsed_ms * 1e-3) / 1e9
    value = job_step_bytes * args.steps / (elapsed_ms * 1e-3) / 1e9
    us_per_gemv = elapsed_ms * 1e3 / (args.steps * n_gemv)

    e2e = None
    if main:
        e2e = run_e2e(args, wl, spec, sets, acts_np, dev, job_step_bytes, world, rows, sharded,
                      launch_gemv if peer else None, fulls)

    # accuracy of this rank's rows (weight copy 0) against an FP32 dense GEMV
    # on the original FP16 weights and activations
    rel_l2 = []
    for gi, (name, d_out, d_in, frac, key) in enumerate(spec):
        lin = sets[0][gi]
        x = acts[key].reshape(-1, d_in)
        y = lin(x.squeeze(0) if M == 1 else x).float().reshape(M, -1)
        y32 = x.float() @ lin.fp16_w.float().t()
        rel_l2.append(float((torch.linalg.vector_norm(y - y32) / torch.linalg.vector_norm(y32)).item()))

    out = None
    if rank == 0:
        per_name = {}
        for j, (name, d_out, d_in, _, key) in enumerate(spec):
            us = per_gemv_us[j]
            per_name[name] = {"shape": [d_out, d_in], "n_outliers": n_o[key], "bytes": local_bytes[j],
                              "us": round(us, 3), "gb_s": round(local_bytes[j] / (us * 1e-6) / 1e9, 1),
                              "frac": round(local_bytes[j] / (us * 1e-6) / 1e9 / peak, 4),
                              "rel_l2_vs_fp32": float(f"{rel_l2[j]:.3e}")}
            if sharded:
                per_name[name]["rows"] = [rows[j][0], rows[j][1]]
            if int4_us:
                b4 = gemv_bytes(d_out, d_in, 0, 1)
                per_name[name]["int4_only"] = {"us": round(int4_us[j], 3),
                                               "gb_s": round(b4 / (int4_us[j] * 1e-6) / 1e9, 1)}
        per_launch = sum(local_bytes) / n_gemv
        ratio, source = ncu_traffic(wl.name, M)
        traffic = round(ratio * per_launch) if ratio else None
        out = {
            "value": round(value, 2), "ms_per_step": round(elapsed_ms / args.steps, 5),
            "scaling": "strong" if sharded else "weak",
            "config": workload_config(wl, world, args.shard, args.gather),
            "us_per_gemv": round(us_per_gemv, 3),
            "gemvs": per_name,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_note": peak_note,
                         "kernel": ("split GEMV kernel (native unit layout, staged outlier columns)" if M == 1 else
                                    "batched split GEMV (plan, INT4 part, FP16 part)"),
                         "algorithmic_bytes_per_launch": round(per_launch),
                         "traffic": traffic,
                         "traffic_note": (f"ncu dram__bytes_read.sum + dram__bytes_write.sum per algorithmic byte of "
                                          f"one 1-GPU capture ({source}) times this rank's algorithmic bytes per "
                                          f"launch" if ratio else "no ncu capture of this workload")},
            "gpu_launches": args.steps * n_gemv * kernels_per_gemv,
            "e2e": e2e,
            "clocks": clocks,
        }
    del warm_graph, timed_graph, per_gemv_graphs, int4_graphs
    if gathers:
        for g in gathers:
            g.close()
    return out


def run_e2e(args, wl, spec, sets, acts_np, dev, job_step_bytes, world, rows, sharded, fused=None, fulls=None):
    """The same steps through DynQuantLinear.forward from pinned host buffers.

    Row-sharded runs gather each GEMV's output slices with
    dyn_quant.sharded.gather_rows (or, given `fused`, through the kernel with
    the gather fused, which writes `fulls`), so every rank copies the full y
    back; replicas (world > 1, not sharded) each run the whole workload and
    the value counts the bytes of all of them over the max-over-ranks time."""
    import torch
    import torch.distributed as dist
    from dyn_quant.sharded import gather_rows
    M = wl.batch
    # The step's inputs sit in one pinned buffer (each 16-byte aligned) and go
    # to the device in one copy; the outputs come back after the last GEMV, so
    # the GEMV launches follow one another on the stream.
    keys = list(acts_np)
    segs = [(v.size + 7) // 8 * 8 for v in acts_np.values()]
    offs = np.cumsum([0] + segs)
    xh_all = torch.zeros(int(offs[-1]), dtype=torch.float16).pin_memory()
    for i, k in enumerate(keys):
        xh_all[int(offs[i]):int(offs[i]) + acts_np[k].size].copy_(torch.from_numpy(acts_np[k].reshape(-1)))
    xd_all = torch.empty(int(offs[-1]), dtype=torch.float16, device=dev)
    xd = {k: xd_all[int(offs[i]):int(offs[i]) + acts_np[k].size].view(acts_np[k].shape) for i, k in enumerate(keys)}
    yh = [torch.empty(M * (world * per if sharded else o), dtype=torch.float16).pin_memory()
          for (_, o, _, _, _), (_, _, per) in zip(spec, rows)]
    gbuf = [torch.empty(world * per, dtype=torch.float16, device=dev) for (_, _, per) in rows]
    ypad = [torch.zeros(M, per, dtype=torch.float16, device=dev) for (_, _, per) in rows]
    gbig = [torch.empty(world * M * per, dtype=torch.float16, device=dev) for (_, _, per) in rows]
    # Unsharded at batch 1: the outputs land in slices of one device buffer (forward's
    # out=) and come back in one copy.
    one_out = not sharded and fused is None and M == 1
    if one_out:
        ysegs = [(M * o + 7) // 8 * 8 for (_, o, _, _, _) in spec]
        yoffs = np.cumsum([0] + ysegs)
        yd_all = torch.empty(int(yoffs[-1]), dtype=torch.float16, device=dev)
        yh_all = torch.empty(int(yoffs[-1]), dtype=torch.float16).pin_memory()
        yd = [yd_all[int(yoffs[gi]):int(yoffs[gi]) + o] for gi, (_, o, _, _, _) in enumerate(spec)]
    h2d = xh_all.numel() * 2
    d2h = yh_all.numel() * 2 if one_out else sum(v.numel() * 2 for v in yh)
    stream = torch.cuda.current_stream(dev)
    times = []

    def step(s):
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        xd_all.copy_(xh_all, non_blocking=True)
        if one_out:
            for gi, (name, d_out, d_in, frac, key) in enumerate(spec):
                sets[s][gi](xd[key], out=yd[gi])
            yh_all.copy_(yd_all, non_blocking=True)
            end.record(stream)
            end.synchronize()
            return start.elapsed_time(end)
        ys = []
        for gi, (name, d_out, d_in, frac, key) in enumerate(spec):
            if fused is not None:
                fused(s, gi, stream, True, xd[key])
                ys.append(fulls[gi])
                continue
            y = sets[s][gi](xd[key])
            if sharded and M == 1:
                y = gather_rows(y, d_out, rows[gi][2], None, gbuf[gi])
            elif sharded:  # [M, rows] slices, gathered rank-major
                ypad[gi][:, :y.shape[-1]].copy_(y)
                dist.all_gather_into_tensor(gbig[gi], ypad[gi].reshape(-1))
                y = gbig[gi]
            ys.append(y)
        for gi, y in enumerate(ys):
            yh[gi].copy_(y.reshape(-1), non_blocking=True)
        end.record(stream)
        end.synchronize()
        return start.elapsed_time(end)

    n_sets = len(sets)
    for i in range(max(3, args.warmup)):
        step(i % n_sets)
    for i in range(args.steps):
        times.append(step(i % n_sets))
    ms = max(statistics.mean(times), 1e-9)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    if world == 1:
        api = ("DynQuantLinear.forward, pinned host buffers (one H2D of the step's inputs, the GEMVs writing "
               "into one output buffer, one D2H of it), synchronised every step")
    elif sharded:
        api = ("DynQuantLinear.forward on each rank's rows + the gather, pinned host buffers on "
               "every rank (bytes per rank), synchronised every step")
    else:
        api = (f"DynQuantLinear.forward on {world} replicas, pinned host buffers on every rank (bytes per "
               "rank), synchronised every step; value: all replicas' bytes over the max-over-ranks time")
    return {"value": round(job_step_bytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(ms, 4), "api": api}


# ---------------------------------------------------------------------------
# MoE FFN step (expert-per-GPU under torchrun)
# ---------------------------------------------------------------------------
def moe_routing_np(cfg: dict, seed: int = 0):
    """Top-K experts per token (uniform without replacement) and weights
    (uniform, normalised per token), from one seed."""
    rng = np.random.default_rng(seed)
    ex = np.stack([rng.choice(cfg["E"], cfg["K"], replace=False) for _ in range(cfg["T"])])
    w = rng.random((cfg["T"], cfg["K"])).astype(np.float32)
    return ex, w / w.sum(1, keepdims=True)


def moe_config(wl: WL, world: int) -> dict:
    cfg = dict(MOE_WORKLOADS[wl.name], k=wl.k)
    if wl.frac is not None:
        cfg["frac"] = wl.frac
    return {"workload": wl.name, "experts": cfg["E"], "d_model": cfg["D"], "d_ff": cfg["F"], "tokens": cfg["T"],
            "top_k": cfg["K"], "outlier_frac": cfg["frac"], "outlier_k": wl.k, "dist": wl.dist,
            "l2": "inputs larger than L2: the GPU arm's steps rotate over weight copies totalling >= 3x L2",
            "parallelism": (f"expert-parallel over {world} GPUs (expert e on rank e % {world}), NCCL all-reduce "
                            "of the FP32 combined outputs") if world > 1 else "1 GPU, all experts"}


def moe_step_bytes(cfg: dict, routing, x, layer, experts) -> int:
    """Algorithmic bytes of the experts' GEMVs in one step: per expert and
    matrix, the weights once, the FP16 columns of the union of the routed
    tokens' outliers (for w2, of the gated activations' outliers), the
    tokens' inputs and outputs."""
    import torch
    import dyn_quant
    from dyn_quant.moe import silu_mul_pairs
    D, F = cfg["D"], cfg["F"]
    total = 0
    for e in experts:
        rows = routing.tokens64.get(e)
        if rows is None:
            continue
        xe = x.index_select(0, rows)
        m = xe.shape[0]

        def union(v):
            return int(torch.stack([dyn_quant.detect_outliers(r, cfg.get("k", 3.0))[0] for r in v]).any(0).sum())
        n_x = union(xe)
        n_h = union(silu_mul_pairs(layer.gate_up(e, xe)))
        total += gemv_bytes(2 * F, D, n_x, m) + gemv_bytes(D, F, n_h, m)
    return total


def moe_block(args, wl: WL, rank: int, world: int, dev, main: bool) -> dict | None:
    import torch
    import torch.distributed as dist
    from dyn_quant.moe import MoEFFN, MoERouting

    cfg = dict(MOE_WORKLOADS[wl.name], k=wl.k)
    if wl.frac is not None:
        cfg["frac"] = wl.frac
    E, D, F, T = cfg["E"], cfg["D"], cfg["F"], cfg["T"]
    local = [e for e in range(E) if e % world == rank]
    ex, w = moe_routing_np(cfg)
    routing = MoERouting(torch.from_numpy(ex), torch.from_numpy(w), E, device=dev)
    x = torch.from_numpy(synth().activations(T, D, cfg["frac"], seed=1, dist=wl.dist)).to(dev)
    # this rank's experts; several copies when they would fit in L2, so that
    # every step streams its weights from HBM
    per_copy = sum((2 * F * D + D * F) // 2 for _ in local)
    n_sets = max(1, math.ceil(3 * L2_BYTES / max(per_copy, 1)))
    if args.max_sets:
        n_sets = min(n_sets, args.max_sets)
    gen = torch.Generator(device=dev)
    layers = []
    for s_ in range(n_sets):
        layer = MoEFFN(E, D, F, wl.k, experts=local)
        for e in local:
            ws = []
            for j, (o, i) in enumerate(((F, D), (F, D), (D, F))):
                gen.manual_seed(100_000 * s_ + 100 * e + j)
                ws.append((torch.randn(o, i, generator=gen, device=dev, dtype=torch.float32) / math.sqrt(i)).half())
            layer.load_expert(e, *ws)
            del ws
        layers.append(layer)
    torch.cuda.synchronize()
    local_bytes = moe_step_bytes(cfg, routing, x, layers[0], local)
    tot = torch.tensor([local_bytes], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tot)
    step_bytes = int(tot.item())
    outs = [torch.zeros(T, D, dtype=torch.float32, device=dev) for _ in range(n_sets)]
    group = None

    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for s_ in range(n_sets):
            layers[s_](x, routing, group, outs[s_])  # first calls: workspaces, kernel attributes
    stream.synchronize()

    def capture(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(n):
                layers[i % n_sets](x, routing, group, outs[i % n_sets])
        return g

    warm = capture(max(args.warmup, n_sets))
    timed = capture(args.steps)
    with torch.cuda.stream(stream):
        warm.replay()
    stream.synchronize()
    sampler = ClockSampler(dev.index) if (main and not args.no_clocks) else None
    if sampler:
        sampler.start()
    t_end = time.perf_counter() + (args.soak if main else 0.1)
    with torch.cuda.stream(stream):
        while time.perf_counter() < t_end:
            warm.replay()
            stream.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        timed.replay()
        e1.record(stream)
    stream.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop() if sampler else None
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = step_bytes * args.steps / (ms * 1e-3) / 1e9
    achieved = local_bytes * args.steps / (ms * 1e-3) / 1e9
    peak, peak_note = measured_peak_gbs()

    # end to end: pinned host tokens in, combined output back, every step
    xh = x.cpu().pin_memory()
    yh = torch.empty(T, D, dtype=torch.float16).pin_memory()
    xd = torch.empty_like(x)
    cur = torch.cuda.current_stream(dev)
    times = []
    for i in range(max(3, args.warmup) + args.steps):
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(cur)
        xd.copy_(xh, non_blocking=True)
        yh.copy_(layers[i % n_sets](xd, routing, group, outs[i % n_sets]), non_blocking=True)
        a1.record(cur)
        a1.synchronize()
        if i >= max(3, args.warmup):
            times.append(a0.elapsed_time(a1))
    e2e_ms = max(statistics.mean(times), 1e-9)
    if world > 1:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    del warm, timed
    if rank != 0:
        return None
    n_tok = {e: routing.count(e) for e in range(E)}
    active = [e for e in local if routing.count(e)]
    grouped = len(active) <= 16 and all(routing.count(e) <= 16 for e in active)
    # per step: grouped, two calls of three kernels, the gated activation and
    # one combine per expert; else per expert two calls, activation, combine
    launches = (7 + len(active)) if (grouped and active) else 8 * len(active)
    return {
        "value": round(value, 2), "ms_per_step": round(ms / args.steps, 5),
        "scaling": "strong" if world > 1 else "weak",
        "config": moe_config(wl, world), "tokens_per_expert": n_tok, "step_bytes": step_bytes,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_note": peak_note,
                     "kernel": "one MoE step on rank 0: the grouped batched split GEMV (plan, INT4 part, FP16 part) "
                               "on every local expert's stacked [w1; w3], dq_silu_mul_pairs, the same on every w2, "
                               "dq_moe_combine per expert",
                     "algorithmic_bytes_per_step": local_bytes, "traffic": None,
                     "traffic_note": "no ncu capture of this workload"},
        "gpu_launches": args.steps * launches,
        "e2e": {"value": round(step_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": T * D * 2, "d2h_bytes_per_step": T * D * 2, "ms_per_step": round(e2e_ms, 4),
                "api": "MoEFFN.forward, pinned host buffers, synchronised every step"},
        "clocks": clocks,
    }


def moe_cpu_sample(cfg: dict, n_pairs: int, seed: int = 0):
    """The first n_pairs (token, expert) pairs of the routing, with each
    expert's matrices quantized by the oracle (seeded: a CPU sample of the
    same shapes)."""
    import oracle as O
    S = synth()
    ex, w = moe_routing_np(cfg, seed)
    x = S.activations(cfg["T"], cfg["D"], cfg["frac"], seed=1)
    pairs = [(t, int(ex[t, j])) for t in range(cfg["T"]) for j in range(cfg["K"])][:n_pairs]
    mats = {}
    for _, e in pairs:
        if e not in mats:
            mats[e] = [(m, *O.quantize(m)) for m in (S.weights(cfg["F"], cfg["D"], seed=10 + e),
                                                     S.weights(cfg["F"], cfg["D"], seed=20 + e),
                                                     S.weights(cfg["D"], cfg["F"], seed=30 + e))]
    return x, pairs, mats


def moe_cpu_pairs(cfg: dict, x, pairs, mats, k: float) -> int:
    """The reference's computation of the pairs on the host; returns their algorithmic bytes."""
    import oracle as O
    total = 0
    for t, e in pairs:
        (w1, p1, s1, z1), (w3, p3, s3, z3), (w2, p2, s2, z2) = mats[e]
        a, _, m1 = O.split_gemv(p1, s1, z1, w1, x[t], k)
        b, _, m3 = O.split_gemv(p3, s3, z3, w3, x[t], k)
        af, bf = a.astype(np.float32), b.astype(np.float32)
        h = (af / (np.float32(1) + np.exp(-af)) * bf).astype(np.float16)
        _, _, m2 = O.split_gemv(p2, s2, z2, w2, h, k)
        total += (gemv_bytes(cfg["F"], cfg["D"], int(m1.sum())) + gemv_bytes(cfg["F"], cfg["D"], int(m3.sum()))
                  + gemv_bytes(cfg["D"], cfg["F"], int(m2.sum())))
    return total


def moe_cpu_baseline(wl: WL, budget_s: float) -> dict:
    import oracle as O
    cfg = dict(MOE_WORKLOADS[wl.name], k=wl.k)
    O.set_num_threads(os.cpu_count() or 1)
    x, pairs, mats = moe_cpu_sample(cfg, 4)
    moe_cpu_pairs(cfg, x, pairs[:1], mats, wl.k)  # warm
    t0 = time.perf_counter()
    nbytes, n = 0, 0
    while True:
        nbytes += moe_cpu_pairs(cfg, x, pairs, mats, wl.k)
        n += len(pairs)
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": round(nbytes / dt / 1e9, 3), "unit": "GB/s", "cores": O.num_threads(), "kind": "port",
            "sample": f"{n} (token, expert) FFN evaluations (3 split GEMVs each, per token as the reference "
                      f"computes them) in {dt:.1f} s, OpenMP over rows, oracle/dq_oracle.c -O3"}


def run_moe_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    import oracle as O
    wl = WL.from_args(args)
    O.set_num_threads(os.cpu_count() or 1)
    cfg = dict(MOE_WORKLOADS[wl.name], k=wl.k)
    x, pairs, mats = moe_cpu_sample(cfg, 2)
    for _ in range(max(1, args.warmup // 3)):
        moe_cpu_pairs(cfg, x, pairs[:1], mats, wl.k)
    t0 = time.perf_counter()
    nbytes = 0
    for _ in range(args.steps):
        nbytes += moe_cpu_pairs(cfg, x, pairs, mats, wl.k)
    dt = time.perf_counter() - t0
    value = nbytes / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "fixed (one host)", "vs_baseline": None,
        "dtype": "w4a16 (fp32 accumulate)", "data": "synthetic",
        "config": moe_config(wl, world),
        "execution": f"rank 0 only, on its host's {O.num_threads()} cores (the other ranks exit without work)",
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": O.num_threads(), "kind": "port",
                         "sample": f"each step: {len(pairs)} (token, expert) FFN evaluations of the workload on the "
                                   "host cores (the reference computes one split GEMV per token and expert)"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
SWEEP_M = (1, 4, 8, 16)
SWEEP_FRAC = (0.0, 0.01, 0.05, 0.10)
SWEEP_DIST = ("normal", "t3")
SWEEP_K = (2.0, 3.0, 4.0, 6.0)


def run_sweep(args, dev) -> None:
    """The outlier / batch sweep on one 8192 x 8192 GEMV: every point of
    M x outlier fraction x distribution x k, timed as a graph of back-to-back
    split GEMV calls over rotating weight copies (the batch-1 kernel at M = 1,
    the batched kernels above).  One JSON line per point; with --sweep-md the
    table is also written as markdown."""
    import torch

    import dyn_quant
    from dyn_quant import _lib

    L = _lib.lib()
    d_out = d_in = 8192
    n_sets = max(2, math.ceil(3 * L2_BYTES / gemv_bytes(d_out, d_in, 0, 1)))
    w0 = torch.from_numpy(weights_np(d_out, d_in, 0)).to(dev)
    mods = []
    for s in range(n_sets):
        lin = dyn_quant.DynQuantLinear(d_in, d_out, 3.0)
        lin.load_weight(w0 if s == 0 else torch.roll(w0, shifts=s * 97, dims=0).contiguous())
        mods.append(lin)
    w32 = mods[0].fp16_w.float()
    structs = [_lib.weights(m.packed.data_ptr(), m.scales.data_ptr(), m.zeros.data_ptr(), None, m.fp16_w.data_ptr(),
                            d_out, d_in, m._native.data_ptr()) for m in mods]
    ws_bytes = max(L.dq_workspace_bytes(d_out, d_in), L.dq_workspace_bytes_batched(d_out, d_in, max(SWEEP_M)))
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
    y = torch.empty(max(SWEEP_M) * d_out, dtype=torch.float16, device=dev)
    stream = torch.cuda.Stream(device=dev)
    peak, peak_note = measured_peak_gbs()
    n_launch = 20
    rows = []
    for dist_ in SWEEP_DIST:
        for frac in SWEEP_FRAC:
            for M in SWEEP_M:
                S = synth()
                xh = S.activation(d_in, frac, seed=1, dist=dist_) if M == 1 else \
                    S.activations(M, d_in, frac, seed=1, dist=dist_)
                x = torch.from_numpy(np.ascontiguousarray(xh)).to(dev)
                for k in SWEEP_K:
                    def launch(i, st):
                        w = structs[i % n_sets]
                        if M == 1:
                            r = L.dq_split_gemv(C.byref(w), C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()), k,
                                                C.c_void_p(ws.data_ptr()), ws_bytes, C.c_void_p(st.cuda_stream))
                        else:
                            r = L.dq_split_gemv_batched(C.byref(w), C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()),
                                                        M, k, C.c_void_p(ws.data_ptr()), ws_bytes,
                                                        C.c_void_p(st.cuda_stream))
                        if r != 0:
                            raise RuntimeError(f"sweep GEMV: {_lib.status_string(r)}")
                    with torch.cuda.stream(stream):
                        launch(0, stream)
                    stream.synchronize()
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, stream=stream):
                        cur = torch.cuda.current_stream()
                        for i in range(n_launch):
                            launch(i, cur)
                    us = statistics.median(graph_time_us(stream, g, n_launch) for _ in range(3))
                    del g
                    xr = x.reshape(M, d_in)
                    masks = [dyn_quant.detect_outliers(r, k)[0] for r in xr]
                    n_union = int(torch.stack(masks).any(0).sum().item())
                    n_mean = float(torch.stack(masks).sum(1).float().mean().item())
                    mods[0].outlier_k = k  # the sweep point's k for the accuracy check too
                    yk = mods[0](xr.squeeze(0) if M == 1 else xr).float().reshape(M, d_out)
                    y32 = xr.float() @ w32.t()
                    rl2 = float((torch.linalg.vector_norm(yk - y32) / torch.linalg.vector_norm(y32)).item())
                    b = gemv_bytes(d_out, d_in, n_union, M)
                    row = {"M": M, "frac": frac, "dist": dist_, "k": k, "outliers_per_vector": round(n_mean, 1),
                           "outliers_union": n_union, "us": round(us, 2), "gb_s": round(b / (us * 1e-6) / 1e9, 1),
                           "frac_of_peak": round(b / (us * 1e-6) / 1e9 / peak, 3), "rel_l2_vs_fp32": float(f"{rl2:.3e}")}
                    rows.append(row)
                    print(json.dumps(row), flush=True)
    if args.sweep_md:
        with open(args.sweep_md, "w") as f:
            f.write("# Outlier / batch sweep: one 8192 x 8192 split GEMV on one B200\n\n")
            f.write("Command: `python bench.py --sweep --sweep-md " + args.sweep_md + "`\n\n")
            f.write(f"Weights synth.weights(8192, 8192, seed=100) and {n_sets - 1} row rotations (every call reads "
                    "its weights from HBM); activations synth.activation(s) seed 1 (vector t: seed 1 + t); "
                    f"graph of {n_launch} back-to-back calls, median of 3 replays. Batch 1: the batch-1 kernel; "
                    "M > 1: the batched kernels (plan, INT4 part, FP16 part). Bytes: INT4 codes + FP16 scale/zero + "
                    "the FP16 columns of the union of the vectors' outliers + x + y. Peak: "
                    f"{peak:.1f} GB/s ({peak_note}). rel-L2 against an FP32 dense GEMV on the original FP16 weights.\n\n")
            f.write("| dist | frac | M | k | outliers / vector | union | µs | GB/s | of peak | rel-L2 vs FP32 |\n")
            f.write("|---|---|---|---|---|---|---|---|---|---|\n")
            for r in rows:
                f.write(f"| {r['dist']} | {r['frac']:.2f} | {r['M']} | {r['k']:g} | {r['outliers_per_vector']} | "
                        f"{r['outliers_union']} | {r['us']} | {r['gb_s']} | {r['frac_of_peak']} | "
                        f"{r['rel_l2_vs_fp32']:.3e} |\n")


def run_ours(args, rank: int, world: int, local_rank: int) -> None:
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        init_nccl(dev)
    if args.sweep:
        if world > 1:
            raise SystemExit("--sweep runs on one GPU")
        run_sweep(args, dev)
        return
    wl = WL.from_args(args)
    if wl.name in MOE_WORKLOADS:
        main = moe_block(args, wl, rank, world, dev, True)
    else:
        main = gemv_block(args, wl, rank, world, dev, True)
    extras = {}
    if not args.no_extras and args.batch == 1:
        for name, batch, frac, k, dist_ in EXTRAS:
            if name == wl.name:
                continue
            if world > 1 and name not in MOE_WORKLOADS:
                continue  # at N > 1: the main workload, and the MoE step expert-parallel
            ewl = WL(name, batch, frac, k, dist_)
            blk = (moe_block if name in MOE_WORKLOADS else gemv_block)(args, ewl, rank, world, dev, False)
            torch.cuda.empty_cache()
            if rank == 0:
                blk.pop("clocks", None)
                extras[name if batch == 1 else f"{name}/m{batch}/frac{frac}"] = blk
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = moe_cpu_baseline(wl, args.cpu_budget) if wl.name in MOE_WORKLOADS else cpu_baseline(wl, args.cpu_budget)
    if rank == 0:
        line = {"metric": METRIC, "value": main["value"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": main["ms_per_step"], "higher_is_better": True,
                "scaling": main["scaling"], "vs_baseline": None, "dtype": "w4a16 (fp32 accumulate)",
                "data": "synthetic (seeded N(0,1/d_in) weights, N(0,1) activations with U[10,100] outliers)",
                "config": main["config"]}
        for k_ in ("us_per_gemv", "gemvs", "tokens_per_expert", "step_bytes", "roofline", "gpu_launches", "e2e",
                   "clocks"):
            if k_ in main:
                line[k_] = main[k_]
        line["cpu_baseline"] = cpu
        if extras:
            line["extras"] = extras
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + sorted(MOE_WORKLOADS), default="llama2_70b_mlp")
    ap.add_argument("--soak", type=float, default=0.6, help="seconds of replays before/after the timed region")
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="measure the main workload only")
    ap.add_argument("--batch", type=int, default=1, help="activation vectors per GEMV call (1..16 per kernel)")
    ap.add_argument("--frac", type=float, default=None, help="injected outlier fraction (default: the workload's)")
    ap.add_argument("--k", type=float, default=K_OUTLIER, help="outlier threshold in standard deviations")
    ap.add_argument("--dist", choices=["normal", "t3"], default="normal", help="activation distribution")
    ap.add_argument("--gather", choices=["peer", "nccl"], default="peer",
                    help="row-sharded runs: the output slices gathered inside the GEMV kernel over NVLink peer "
                         "memory (the default), or by an NCCL all-gather after each GEMV")
    ap.add_argument("--shard", choices=["auto", "rows", "replicas"], default="auto",
                    help="N > 1: row sharding with a gather, or independent replicas; auto follows the "
                         "deployment of each shape: rows for the 70B workloads, replicas for the 7B and sweep ones")
    ap.add_argument("--sweep", action="store_true",
                    help="the outlier / batch sweep of one 8192x8192 GEMV (M x frac x dist x k), one JSON line per point")
    ap.add_argument("--sweep-md", default=None, help="with --sweep: also write the table as markdown to this path")
    ap.add_argument("--max-sets", type=int, default=0,
                    help="cap on rotating weight copies (profiling runs only; the default rotates through >= 3x L2)")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if not 1 <= args.batch <= 16:
        ap.error("--batch must be in 1..16")
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
