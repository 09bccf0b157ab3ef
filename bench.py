"""Benchmark of the FP8 decode GEMV hot path on B200.

One step = one pass of BASELINE config 1: the FP8-weight GEMV at
(N, K) = (28672, 4096) gate_up, (4096, 14336) down, (6144, 4096) QKV, each at
M = 1, 2, 4, 8 tokens (12 launches), e4m3 weights with fp32 per-channel
scales, fp16 activations, seeded synthetic data.  Two weight sets alternate
between steps (402 MB > 126 MB L2), so every launch streams its weights from
HBM.

  value       whole-job HBM GB/s (algorithmic bytes of all ranks / max-over-
              ranks device time), one CUDA-graph replay per step, inputs
              resident in HBM
  e2e         the same metric through the public torch op, eager, with the
              step's activations copied host->device from pinned memory and
              the outputs read back device->host inside the timed region
  roofline    the GEMV kernel: algorithmic bytes / CUDA-event time of its
              launches vs the measured HBM copy bandwidth
  cpu_baseline  the CPU oracle (torch fp32 dequant-then-matmul, the
              reference tests' oracle) on this host's cores, a bounded sample

`--impl reference` times the reference's CPU path (the oracle port: the
reference's own kernels are Intel-GPU-only and cannot run here) on the same
workload, rank 0 only.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
(N > 1 under torch.distributed.run: one rank per GPU, each rank runs the
same independent GEMV sweep: weak scaling, no collective on the data path.)
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

SHAPES = [("gate_up", 28672, 4096), ("down", 4096, 14336), ("qkv", 6144, 4096)]
MS = [1, 2, 4, 8]
CALLS = [(name, N, K, M) for M in MS for (name, N, K) in SHAPES]
METRIC = "FP8 GEMV HBM GB/s, config 1 sweep (gate_up/down/qkv x M=1,2,4,8)"
FALLBACK_HBM_GBS = 6650.0


def call_bytes(M: int, N: int, K: int) -> int:
    """Algorithmic bytes of one GEMV: weights + activations + fp32 scales + outputs."""
    return N * K + 2 * M * K + 4 * N + 2 * M * N


STEP_BYTES = sum(call_bytes(M, N, K) for (_, N, K, M) in CALLS)


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def profile_traffic() -> float | None:
    """DRAM bytes per config-1 step from the committed ncu summary, if present."""
    f = ROOT / "profiles" / "gemv_fp8_config1.md"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        if line.startswith("dram_bytes_per_step:"):
            return float(line.split(":", 1)[1].strip())
    return None


# ---- clocks sampling ------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.rows: list[list[str]] = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.3)
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        for r in self.rows:
            try:
                sm.append(float(r[0]))
                mx = max(mx, float(r[1]))
                for name, v in zip(self.NAMES, r[3:7]):
                    if v.lower() == "active":
                        reasons.add(name)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "samples": len(sm), "reasons": sorted(reasons)}


# ---- distributed plumbing --------------------------------------------------------------

def dist_init(n_gpus: int):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}; launch with torch.distributed.run")
    if world > 1:
        import torch.distributed as dist
        os.environ.setdefault("NCCL_DEBUG", "WARN")  # keep stdout to the one JSON line
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---- our arm ------------------------------------------------------------------------

def workloads():
    """esimd_learning_b200/workloads.py loaded by path: the seeded input
    builders only, without the package __init__ (which loads the CUDA
    extensions), so the CPU reference arm maps none of this build's .so files."""
    import importlib.util
    mod = sys.modules.get("cek_bench_workloads")
    if mod is None:
        spec = importlib.util.spec_from_file_location("cek_bench_workloads",
                                                      ROOT / "esimd_learning_b200" / "workloads.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        sys.modules["cek_bench_workloads"] = mod
    return mod


def n_sets_for(world: int) -> int:
    """Weight sets rotated between steps so that > 3x L2 (126 MB) of weights
    pass through each GPU before a set is read again."""
    per_rank = sum(N * K for _, N, K in SHAPES) / world
    return 2 if world == 1 else max(2, -(-(3 * 126 * 2**20) // int(per_rank)))


def arm_config(world: int, prefetch: bool) -> dict:
    """The `config` object of the JSON line; both arms print exactly this."""
    if world == 1:
        return {"workload": "BASELINE config 1: batched FP8 GEMV, per-channel fp32 scales",
                "shapes": {n: [N, K] for n, N, K in SHAPES}, "M": MS,
                "l2": "2 weight sets alternating with M: > 126 MB (L2) between two reads of one weight",
                "timing": "CUDA graph of the 12 launches per step, CUDA events",
                "weight_prefetch": prefetch, "parallelism": "single GPU"}
    return {"workload": "BASELINE config 1: batched FP8 GEMV, per-channel fp32 scales",
            "shapes": {n: [N, K] for n, N, K in SHAPES}, "M": MS,
            "l2": f"{n_sets_for(world)} weight sets per rank rotated: > 3x L2 between two reads of one weight",
            "timing": "CUDA graph of the steps (12 launches + 1 barrier each), CUDA events, max over ranks",
            "weight_prefetch": prefetch,
            "parallelism": f"column-parallel x{world}: each rank streams N/{world} rows of every weight and "
                           "pushes its rows into every rank's full output over NVLink in the GEMV epilogue "
                           "(cek_gemv_fp8_allgather), one barrier per step"}


def build_sets(dev, n_sets: int = 2):
    make_fp8_weight = workloads().make_fp8_weight

    gen = torch.Generator().manual_seed(0)
    sets = []
    for s in range(n_sets):
        ws = {}
        for name, N, K in SHAPES:
            wq, sc = make_fp8_weight(N, K, gen)
            ws[name] = (wq.to(dev), sc.to(dev))
        sets.append(ws)
    # all activations of a step in one buffer and all outputs in another, so
    # the end-to-end leg moves each with a single copy
    xkeys = [(name, M) for (name, N, K, M) in CALLS]
    xsizes = [M * K for (name, N, K, M) in CALLS]
    xbuf = torch.randn(sum(xsizes), generator=gen).to(torch.float16).to(dev)
    ysizes = [M * N for (name, N, K, M) in CALLS]
    ybuf = torch.empty(sum(ysizes), dtype=torch.float16, device=dev)
    xs, ys = {}, {}
    xo = yo = 0
    for (name, N, K, M), xn, yn in zip(CALLS, xsizes, ysizes):
        xs[(name, M)] = xbuf[xo:xo + xn].view(M, K)
        ys[(name, M)] = ybuf[yo:yo + yn].view(M, N)
        xo += xn
        yo += yn
    xs["_buf"], ys["_buf"] = xbuf, ybuf
    return sets, xs, ys


def run_ours_tp(args, rank, world, local):
    """N > 1: the same config-1 step, strong-scaled.  Every GEMV is
    column-parallel over the ranks (rows [N r / W, N (r + 1) / W) of each
    weight on rank r) and its all-gather is fused into the epilogue: each
    rank stores its rows into every rank's copy of the full output over
    NVLink peer memory; one barrier ends the step.  value = the step's
    algorithmic bytes (counted once for the whole job) / max-over-ranks time."""
    import esimd_learning_b200 as ops
    from esimd_learning_b200.chain import TPComm, gemv_fp8_allgather, shard_rows

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    W = workloads()
    prefetch = not args.no_prefetch
    nsets = n_sets_for(world)
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    sets = []
    for _ in range(nsets):
        ws = {}
        for name, N, K in SHAPES:
            r0, r1 = shard_rows(N, rank, world)
            ws[name] = W.quantize_per_channel(torch.randn(r1 - r0, K, device=dev, generator=gen) * 0.02) + (r0,)
        sets.append(ws)
    g0 = torch.Generator().manual_seed(0)
    xsz = [M * K for (_, N, K, M) in CALLS]
    xbuf = torch.randn(sum(xsz), generator=g0).to(torch.float16).to(dev)
    xs, o = {}, 0
    for (name, N, K, M), n in zip(CALLS, xsz):
        xs[(name, M)] = xbuf[o:o + n].view(M, K)
        o += n
    ysz = [M * N * 2 for (_, N, K, M) in CALLS]
    yoff = [sum(ysz[:i]) for i in range(len(CALLS))]
    ytotal = (sum(ysz) + 255) // 256 * 256
    comm = TPComm(0, rank, world, dev, data_bytes=2 * ytotal)

    def step(si):
        ws = sets[si % nsets]
        for ci, (name, N, K, M) in enumerate(CALLS):
            w, sc, r0 = ws[name]
            gemv_fp8_allgather(comm, xs[(name, M)], w, sc, r0, N, (si % 2) * ytotal + yoff[ci],
                               early_weights=prefetch)
        comm.barrier()

    graph_steps = nsets if nsets % 2 == 0 else 2 * nsets
    st = torch.cuda.Stream(dev)
    with torch.cuda.stream(st):
        step(0)
        torch.cuda.synchronize()
        barrier(world)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            for si in range(graph_steps):
                step(si)
    torch.cuda.synchronize()
    replays = max(1, -(-args.steps // graph_steps))
    steps = replays * graph_steps
    with torch.cuda.stream(st):
        for _ in range(max(1, -(-args.warmup // graph_steps))):
            graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(st):
            e0.record(st)
            for _ in range(replays):
                graph.replay()
            e1.record(st)
        torch.cuda.synchronize()
    barrier(world)
    ms_step = max_over_ranks(e0.elapsed_time(e1), world) / steps
    value = STEP_BYTES / (ms_step * 1e-3) / 1e9

    # e2e through the public API (chain.gemv_fp8_allgather + barrier), eager:
    # the step's activations copied host->device, the gathered outputs read back
    hx = xbuf.cpu().pin_memory()
    yview = comm.data_tensor(0, (sum(ysz) // 2,))
    hy = torch.empty(yview.shape, dtype=torch.float16).pin_memory()
    e2e_steps = max(3, min(args.steps, 300))
    with torch.cuda.stream(st):
        def e2e_step():
            xbuf.copy_(hx, non_blocking=True)
            step(0)
            hy.copy_(yview, non_blocking=True)
        for _ in range(args.warmup):
            e2e_step()
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(st)
        for _ in range(e2e_steps):
            e2e_step()
        a1.record(st)
        torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(a0.elapsed_time(a1), world) / e2e_steps
    errors = comm.errors()
    peak, peak_kind = peaks()
    per_gpu = STEP_BYTES / world / (ms_step * 1e-3) / 1e9
    out = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "e4m3*fp16->fp32", "data": "synthetic (seeded: x~N(0,1) fp16, W~N(0,0.02) per-row e4m3)",
        "config": arm_config(world, prefetch),
        "roofline": {"bound": "hbm", "achieved": round(per_gpu, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(per_gpu / peak, 4), "peak_source": peak_kind, "traffic": None,
                     "algorithmic_bytes": STEP_BYTES // world,
                     "kernel": "cek::bulk::gemv_bulk_kernel with the all-gather push epilogue (per GPU: "
                               "its share of the step's bytes / step time)"},
        "e2e": {"value": round(STEP_BYTES / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                "h2d_bytes_per_step": hx.numel() * 2, "d2h_bytes_per_step": hy.numel() * 2,
                "ms_per_step": round(e2e_ms, 5),
                "api": "esimd_learning_b200.chain.gemv_fp8_allgather + TPComm.barrier, eager"},
        "gpu_launches": (len(CALLS) + 1) * steps,
        "clocks": clk.summary(),
        "comm_errors": errors,
    }
    del graph
    comm.close()
    torch.cuda.empty_cache()
    if not args.no_chain:
        out["chain"] = measure_chain(dev, rank, world)
    return out


def run_ours(args, rank, world, local):
    import esimd_learning_b200 as ops

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    sets, xs, ys = build_sets(dev)

    def step():
        # the weight set alternates with M, so two uses of one set are always
        # separated by > 126 MB of other weights
        for (name, N, K, M) in CALLS:
            wq, sc = sets[MS.index(M) % 2][name]
            ops.esimd_gemv_fp8_pern(xs[(name, M)], wq, sc, ys[(name, M)], N, K)

    # Static weights: let each GEMV stream its weights while the previous
    # launch drains (programmatic dependent launch; esimd_set_weight_prefetch).
    prefetch = not args.no_prefetch
    ops.esimd_set_weight_prefetch(prefetch)
    st = torch.cuda.Stream(dev)
    with torch.cuda.stream(st):
        step()  # warm (module load) outside capture
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            step()
    torch.cuda.synchronize()

    # --- per-call times: back-to-back launches over rotating weight copies
    # (> 320 MB per shape, so each launch streams its weights from HBM) ---
    per_call = {}
    with torch.cuda.stream(st):
        for (name, N, K) in SHAPES:
            ncopy = max(2, -(-(320 << 20) // (N * K)))
            gen = torch.Generator(device=dev).manual_seed(1)
            copies = [torch.randint(0, 120, (N, K), dtype=torch.uint8, device=dev, generator=gen)
                      .view(torch.float8_e4m3fn) for _ in range(ncopy)]
            sc = sets[0][name][1]
            for M in MS:
                x, y = xs[(name, M)], ys[(name, M)]
                for c in copies:
                    ops.esimd_gemv_fp8_pern(x, c, sc, y, N, K)
                reps = 2 * ncopy
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(st)
                for r in range(reps):
                    ops.esimd_gemv_fp8_pern(x, copies[r % ncopy], sc, y, N, K)
                e1.record(st)
                torch.cuda.synchronize()
                per_call[f"{name}_M{M}"] = e0.elapsed_time(e1) * 1e3 / reps
            del copies
    torch.cuda.empty_cache()

    # --- timed region: graph replays ---
    for i in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(st):
            e0.record(st)
            for i in range(args.steps):
                graph.replay()
            e1.record(st)
        torch.cuda.synchronize()
    barrier(world)
    ms_total = max_over_ranks(e0.elapsed_time(e1), world)
    ms_step = ms_total / args.steps
    value = STEP_BYTES * world / (ms_step * 1e-3) / 1e9

    # --- e2e: public torch op, eager, host buffers, copies inside the timed region ---
    # One pinned host->device copy of the step's 12 activation blocks, the 12
    # op calls, one device->host read of the 12 outputs.
    hx = xs["_buf"].cpu().pin_memory()
    hy = torch.empty(ys["_buf"].shape, dtype=torch.float16).pin_memory()
    h2d = hx.numel() * hx.element_size()
    d2h = hy.numel() * hy.element_size()
    e2e_steps = max(3, min(args.steps, 500))

    def e2e_step():
        xs["_buf"].copy_(hx, non_blocking=True)
        for (name, N, K, M) in CALLS:
            wq, sc = sets[MS.index(M) % 2][name]
            ops.esimd_gemv_fp8_pern(xs[(name, M)], wq, sc, ys[(name, M)], N, K)
        hy.copy_(ys["_buf"], non_blocking=True)

    with torch.cuda.stream(st):
        for i in range(args.warmup):
            e2e_step()
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(st)
        for i in range(e2e_steps):
            e2e_step()
        a1.record(st)
        torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(a0.elapsed_time(a1), world) / e2e_steps
    e2e_value = STEP_BYTES * world / (e2e_ms * 1e-3) / 1e9

    # --- roofline of the GEMV kernel: it is every launch of the timed region,
    # so its achieved bandwidth is the step's algorithmic bytes / device time ---
    peak, peak_kind = peaks()
    achieved = STEP_BYTES / (ms_step * 1e-3) / 1e9
    traffic = profile_traffic()
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                "traffic": traffic,
                "traffic_source": ("the ncu DRAM capture of this workload summarised in profiles/gemv_fp8_config1.md "
                                   "(read from that file, not measured in this run)") if traffic else None,
                "algorithmic_bytes": STEP_BYTES,
                "kernel": "cek::bulk::gemv_bulk_kernel (12 launches per step; traffic = ncu DRAM bytes per step)"}

    out = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "e4m3*fp16->fp32", "data": "synthetic (seed 0: x~N(0,1) fp16, W~N(0,0.02) per-row e4m3)",
        "config": arm_config(world, prefetch),
        "us_per_call": {k: round(v, 3) for k, v in per_call.items()},
        "roofline": roofline,
        "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 5),
                "api": "esimd_learning_b200.esimd_gemv_fp8_pern (torch op), eager"},
        "gpu_launches": len(CALLS) * args.steps,
        "clocks": clk.summary(),
    }
    out["config0"] = measure_config0(dev)
    out["config2"] = measure_config2(dev)
    out["elementwise"] = measure_elementwise(dev)
    if not args.no_gemm:
        out["gemm"] = {f"M{M}": measure_gemm(dev, M) for M in (2048, 8192)}
    if not args.no_chain:
        out["chain"] = measure_chain(dev, rank, world)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline_sample(seconds=args.cpu_seconds)
    if rank == 0 and world == 1 and not args.no_vllm:
        out["vllm"] = vllm_compare_subprocess()
    return out


def vllm_compare_subprocess(timeout_s: int = 240) -> dict:
    """Runs `bench.py --vllm-compare` in a child process (vLLM's import and
    kernels must not be able to take this run down) and returns its JSON."""
    import subprocess
    try:
        r = subprocess.run([sys.executable, str(Path(__file__).resolve()), "--vllm-compare"], capture_output=True,
                           text=True, timeout=timeout_s)
        lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
        if r.returncode != 0 or not lines:
            return {"unavailable": f"exit {r.returncode}: {(r.stderr or r.stdout).strip().splitlines()[-1:]}"}
        return json.loads(lines[-1])
    except Exception as e:  # noqa: BLE001 - a comparison, never fatal
        return {"unavailable": f"{type(e).__name__}: {e}"}


def vllm_compare() -> dict:
    """Config-1 shapes at M = 1 and 8: our W8A16 GEMV (fp16 activations, as
    the reference ops) against vLLM 0.22's CUDA FP8 linear path on the same
    weights, dynamic per-token activation quantisation (scaled_fp8_quant)
    followed by cutlass_scaled_mm (W8A8).  Both timed as CUDA-graph replays
    over rotating weight copies (> 320 MB per shape, cold L2), CUDA events."""
    import esimd_learning_b200 as ops
    from vllm import _custom_ops as vops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    res = {"vllm": __import__("vllm").__version__,
           "path": "scaled_fp8_quant(per-token) + cutlass_scaled_mm, W8A8, fp16 out",
           "ours": "esimd_gemv_fp8_pern, W8A16 (no activation quantisation)"}
    st = torch.cuda.Stream(dev)

    def graph_time(fn, copies, reps):
        with torch.cuda.stream(st):
            for c in copies:
                fn(c)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st):
                for r in range(reps):
                    fn(copies[r % len(copies)])
            g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            g.replay()
            e1.record(st)
            torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / reps

    for name, N, K in SHAPES:
        ncopy = max(2, -(-(320 << 20) // (N * K)))
        gen = torch.Generator(device=dev).manual_seed(7)
        copies = [torch.randint(0, 120, (N, K), dtype=torch.uint8, device=dev, generator=gen)
                  .view(torch.float8_e4m3fn) for _ in range(ncopy)]
        sc = torch.rand(N, device=dev) * 0.01 + 1e-3
        for M in (1, 8):
            x = torch.randn(M, K, device=dev).half()
            y = torch.empty(M, N, device=dev, dtype=torch.float16)
            ours = graph_time(lambda w: ops.esimd_gemv_fp8_pern(x, w, sc, y, N, K), copies, 2 * ncopy)

            def vllm_call(w):
                xq, xs = vops.scaled_fp8_quant(x, use_per_token_if_dynamic=True)
                return vops.cutlass_scaled_mm(xq, w.t(), scale_a=xs, scale_b=sc.view(-1, 1), out_dtype=torch.float16)

            try:
                theirs = graph_time(vllm_call, copies, 2 * ncopy)
            except Exception as e:  # noqa: BLE001
                theirs = f"{type(e).__name__}: {str(e)[:120]}"
            res[f"{name}_M{M}"] = {"ours_us": round(ours, 2),
                                   "vllm_us": round(theirs, 2) if isinstance(theirs, float) else theirs}
        del copies
        torch.cuda.empty_cache()
    return res


def measure_chain(dev, rank: int, world: int, Ms=(1, 8, 16), reps: int = 200) -> dict:
    """the 70B-shaped decode step (esimd_learning_b200.chain)
    tensor-parallel over the `world` ranks of this run.  At TP > 1 the down
    projection's all-reduce runs two ways: fused into the GEMV over NVLink
    peer memory (cek_gemv_fp8_allreduce, "fused") and as GEMV + NCCL
    all-reduce ("nccl").  L layers with distinct weights are captured in one
    CUDA graph so that each replay streams more than 3x L2 of weights per
    rank; time = max over ranks of the CUDA-event time per layer-step."""
    import esimd_learning_b200 as ops
    from esimd_learning_b200.chain import ChainShape, DecodeChain, TPComm, full_weights, shard_weights

    shape = ChainShape()
    per_rank = shape.weight_bytes() // world
    layers = max(1, -(-(3 * 126 * 2**20) // per_rank))
    old = ops.esimd_set_weight_prefetch(True)
    comm = TPComm(max(Ms) * shape.hidden, rank, world, dev) if world > 1 else None
    modes = ["fused", "nccl"] if world > 1 else ["local"]
    shards = []
    for l in range(layers):
        full = full_weights(shape, seed=100 + l, device=dev)
        shards.append(shard_weights(full, shape, rank, world))
        del full
        torch.cuda.empty_cache()
    res = {"tp": world, "layers_per_replay": layers, "weight_bytes_per_rank_per_step": per_rank}
    peak, _ = peaks()
    for mode in modes:
        for M in Ms:
            chains = [DecodeChain(sh, shape, M, dev, world=world, comm=comm if mode == "fused" else None)
                      for sh in shards]
            g = torch.Generator(device=dev).manual_seed(7)
            h = torch.randn(M, shape.hidden, device=dev, generator=g).half()
            r = torch.randn(M, shape.hidden, device=dev, generator=g).half()
            a = torch.randn(M, shape.hidden, device=dev, generator=g).half()
            pos = torch.randint(0, shape.max_position, (M,), device=dev, generator=g)
            st = torch.cuda.Stream(dev)
            with torch.cuda.stream(st):
                for c in chains:
                    c.step(h, r, a, pos)  # warm-up outside capture (NCCL, modules)
                torch.cuda.synchronize()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=st):
                    for c in chains:
                        c.step(h, r, a, pos)
                for _ in range(5):
                    graph.replay()
                torch.cuda.synchronize()
                barrier(world)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(st)
                for _ in range(reps):
                    graph.replay()
                e1.record(st)
                torch.cuda.synchronize()
            barrier(world)
            us = max_over_ranks(e0.elapsed_time(e1) * 1e3 / (reps * layers), world)
            gbs = per_rank / (us * 1e-6) / 1e9
            key = f"M{M}" if mode in ("fused", "local") else f"M{M}_nccl"
            res[key] = {"us_per_step": round(us, 2), "weight_gbs_per_gpu": round(gbs, 1),
                        "frac_of_hbm": round(gbs / peak, 4),
                        "all_reduce": {"fused": "GEMV push over NVLink peer memory + reduce kernel",
                                       "nccl": "NCCL all_reduce", "local": "none (TP=1)"}[mode]}
            del graph, chains
    if comm is not None:
        res["comm_errors"] = comm.errors()
        comm.close()
    ops.esimd_set_weight_prefetch(old)
    torch.cuda.empty_cache()
    return res


def fp8_peak_tflops() -> tuple[float, str]:
    """Dense FP8 denominator: 2x the measured cuBLAS bf16 burst rate (the
    tensor cores run e4m3 at twice the bf16 rate); fallback 2 x 1590."""
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return 2.0 * float(json.loads(p.read_text())["bf16_tflops"]), "2x measured bf16 burst"
    except Exception:
        return 2.0 * 1590.0, "2x fallback bf16"


def measure_config0(dev, reps: int = 240) -> dict:
    """one GEMV, M = 1, N = K = 4096 (16.8 MB of weights),
    per-channel fp32 scales.  A CUDA graph of `reps` back-to-back calls over
    32 rotating weight copies (537 MB, > 4x L2), so every call streams its
    weights from HBM; CUDA events; the per-call mean."""
    import esimd_learning_b200 as ops
    from esimd_learning_b200.workloads import gemv_case

    N = K = 4096
    x, wq, sc = gemv_case(1, N, K, seed=0, device=dev)
    gen = torch.Generator(device=dev).manual_seed(3)
    copies = [wq] + [torch.randint(0, 120, (N, K), dtype=torch.uint8, device=dev, generator=gen)
                     .view(torch.float8_e4m3fn) for _ in range(31)]
    y = torch.empty(1, N, dtype=torch.float16, device=dev)
    st = torch.cuda.Stream(dev)
    with torch.cuda.stream(st):
        for c in copies:
            ops.esimd_gemv_fp8_pern(x, c, sc, y, N, K)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            for r in range(reps):
                ops.esimd_gemv_fp8_pern(x, copies[r % len(copies)], sc, y, N, K)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        g.replay()
        e1.record(st)
        torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / reps
    b = call_bytes(1, N, K)
    peak, src = peaks()
    del copies
    torch.cuda.empty_cache()
    return {"us_per_call": round(us, 3), "gbs": round(b / (us * 1e-6) / 1e9, 1),
            "frac": round(b / (us * 1e-6) / 1e9 / peak, 4), "peak_gbs": peak, "peak_source": src,
            "algorithmic_bytes": b, "timing": "CUDA graph of back-to-back calls, 32 rotating weight copies"}


def measure_config2(dev, reps_per_copy: int = 4) -> dict:
    """fused residual add + RMSNorm -> QKV GEMV [6144, 4096]
    (esimd_fused_add_rms_norm_batched_fp8) at M = 1, 2, 4, 8, against the
    plain GEMV on the same weights.  CUDA graph of back-to-back calls over
    rotating weight copies (> 4x L2); CUDA events; per-call mean.  Bytes:
    N K + 4 N (scales) + 6 M K (read h, r; write r) + 2 K (gamma) + 2 M N."""
    import esimd_learning_b200 as ops
    N, K = 6144, 4096
    gen = torch.Generator(device=dev).manual_seed(5)
    ncopy = -(-(512 << 20) // (N * K))
    copies = [torch.randint(0, 120, (N, K), dtype=torch.uint8, device=dev, generator=gen)
              .view(torch.float8_e4m3fn) for _ in range(ncopy)]
    sc = torch.rand(N, device=dev, generator=gen) * 0.01 + 1e-3
    gamma = (1 + 0.1 * torch.randn(K, device=dev, generator=gen)).half()
    st = torch.cuda.Stream(dev)
    peak, src = peaks()

    def graph_us(fn, reps):
        with torch.cuda.stream(st):
            fn(0)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st):
                for r in range(reps):
                    fn(r)
            g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            g.replay()
            e1.record(st)
            torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / reps

    res = {"shape": [N, K], "timing": "CUDA graph of back-to-back calls, rotating weight copies", "peak_gbs": peak,
           "peak_source": src}
    for M in (1, 2, 4, 8):
        h = torch.randn(M, K, device=dev, generator=gen).half()
        r = torch.randn(M, K, device=dev, generator=gen).half()
        y = torch.empty(M, N, device=dev, dtype=torch.float16)
        fused = graph_us(lambda i: ops.esimd_fused_add_rms_norm_batched_fp8(h, r, gamma, 1e-6, copies[i % ncopy], sc, y),
                         reps_per_copy * ncopy)
        plain = graph_us(lambda i: ops.esimd_gemv_fp8_pern(h, copies[i % ncopy], sc, y, N, K), reps_per_copy * ncopy)
        b = N * K + 4 * N + 6 * M * K + 2 * K + 2 * M * N
        res[f"M{M}"] = {"fused_us": round(fused, 3), "plain_gemv_us": round(plain, 3),
                        "gbs": round(b / (fused * 1e-6) / 1e9, 1), "frac": round(b / (fused * 1e-6) / 1e9 / peak, 4)}
    del copies
    torch.cuda.empty_cache()
    return res


def measure_elementwise(dev, reps: int = 400) -> dict:
    """The decode-chain helpers at config-4 shapes (TP = 1): GeLU(tanh)-and-mul
    on [M, 2 x 28672] and q/k-norm + RoPE on [M, 80 heads x 128] (64 q, 8 k
    heads normed and rotated), M = 1, 8, 16.  CUDA graph of `reps`
    back-to-back calls, CUDA events, per-call mean.  The tensors are small
    enough to stay in L2, so these are launch- and latency-bound; the
    fraction is reported against the HBM copy peak for reference only."""
    import esimd_learning_b200 as ops
    from oracle import oracle as O  # the cos/sin cache builder only
    st = torch.cuda.Stream(dev)
    peak, _ = peaks()

    def graph_us(fn):
        with torch.cuda.stream(st):
            fn()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st):
                for _ in range(reps):
                    fn()
            g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            g.replay()
            e1.record(st)
            torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / reps

    res = {"timing": "CUDA graph of back-to-back calls (L2-resident inputs)"}
    d, hq, hkv, D = 28672, 64, 8, 128
    cs = O.rope_cos_sin_cache(8192, D, 500000.0).to(dev)
    qw = torch.ones(D, dtype=torch.float16, device=dev)
    for M in (1, 8, 16):
        x = torch.randn(M, 2 * d, device=dev).half()
        o = torch.empty(M, d, device=dev, dtype=torch.float16)
        us = graph_us(lambda: ops.esimd_gelu_and_mul(x, o))
        b = 6 * M * d
        res[f"gelu_and_mul_M{M}"] = {"us": round(us, 3), "bytes": b, "gbs": round(b / (us * 1e-6) / 1e9, 1)}
        qkv = torch.randn(M, (hq + 2 * hkv) * D, device=dev).half()
        pos = torch.randint(0, 8192, (M,), device=dev)
        us = graph_us(lambda: ops.esimd_qkv_norm_rope(qkv, pos, qw, qw, cs, hq, hkv, D, 1e-6, True))
        b = 2 * 2 * M * (hq + hkv) * D + 4 * M * D
        res[f"qkv_norm_rope_M{M}"] = {"us": round(us, 3), "bytes": b, "gbs": round(b / (us * 1e-6) / 1e9, 1)}
    return res


def measure_gemm(dev, M: int, reps: int = 20) -> dict:
    """per-token quantisation of A [M, 4096] fp16 and the
    tcgen05 FP8 GEMM against B [14336, 4096] e4m3 (per-channel scales).  Each
    timed launch follows an L2 flush (256 MB write, then read back so
    no dirty line is left for the timed launch to write back); CUDA events on the
    launching stream; median over `reps`.  torch._scaled_mm (cuBLASLt FP8,
    row-wise scales) on the same operands is reported beside it."""
    import esimd_learning_b200 as ops
    from esimd_learning_b200.workloads import prefill_case
    N, K = 14336, 4096
    a, bq, bs = prefill_case(M, N=N, K=K, seed=0, device=dev)
    aq = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=dev)
    as_ = torch.empty(M, dtype=torch.float32, device=dev)
    y = torch.empty(M, N, dtype=torch.float16, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    flush_sum = torch.empty((), dtype=torch.int64, device=dev)
    st = torch.cuda.current_stream(dev)

    def timed(fn):
        ts = []
        for r in range(reps + 3):
            # write 256 MB (evicts the operands), then read it back: the read
            # writes the dirty lines back, so the timed launch starts on a clean
            # L2 and does not pay for the flush's write-backs
            flush.zero_()
            torch.sum(flush, dim=0, dtype=torch.int64, out=flush_sum)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            fn()
            e1.record(st)
            torch.cuda.synchronize()
            if r >= 3:
                ts.append(e0.elapsed_time(e1) * 1e3)
        return statistics.median(ts)

    quant_one_us = timed(lambda: ops.esimd_quant_fp8_per_token(a, aq, as_))
    # steady state: a CUDA graph of back-to-back calls over rotating copies of
    # A (together > 2x L2), so every call reads its input from HBM
    ncopy = max(2, -(-(256 << 20) // (2 * M * K)))
    a_copies = [a.clone() for _ in range(ncopy)]
    q_copies = [torch.empty_like(aq) for _ in range(ncopy)]
    s_copies = [torch.empty_like(as_) for _ in range(ncopy)]
    qs = torch.cuda.Stream(dev)
    with torch.cuda.stream(qs):
        for i in range(ncopy):
            ops.esimd_quant_fp8_per_token(a_copies[i], q_copies[i], s_copies[i])
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=qs):
            for i in range(ncopy):
                ops.esimd_quant_fp8_per_token(a_copies[i], q_copies[i], s_copies[i])
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        q0, q1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        q0.record(qs)
        for _ in range(5):
            g.replay()
        q1.record(qs)
        torch.cuda.synchronize()
    quant_us = q0.elapsed_time(q1) * 1e3 / (5 * ncopy)
    del g, a_copies, q_copies, s_copies
    gemm_us = timed(lambda: ops.esimd_gemm_fp8_pertoken_pern(aq, as_, bq, bs, y))
    flops = 2.0 * M * N * K
    peak, src = fp8_peak_tflops()
    tf = flops / (gemm_us * 1e-6) / 1e12
    res = {"gemm_us": round(gemm_us, 2), "tflops": round(tf, 1), "peak_tflops": peak, "peak_source": src,
           "frac": round(tf / peak, 4), "quant_us": round(quant_us, 2),
           "quant_gbs": round((2 * M * K + M * K + 4 * M) / (quant_us * 1e-6) / 1e9, 1),
           "quant_timing": "CUDA graph of back-to-back calls over rotating input copies (> 2x L2); "
                           "quant_single_launch_us: one launch after the L2 flush",
           "quant_single_launch_us": round(quant_one_us, 2),
           "shape": [M, N, K], "out": "fp16"}
    try:
        sa, sb = as_.reshape(M, 1), bs.reshape(1, N)
        lib_us = timed(lambda: torch._scaled_mm(aq, bq.t(), scale_a=sa, scale_b=sb, out_dtype=torch.float16))
        res["cublaslt_scaled_mm_us"] = round(lib_us, 2)
        res["cublaslt_tflops"] = round(flops / (lib_us * 1e-6) / 1e12, 1)
    except Exception as e:  # library path unavailable: report why
        res["cublaslt_scaled_mm"] = f"unavailable: {type(e).__name__}"
    del flush
    return res


# ---- CPU legs (oracle port of the reference's path) -----------------------------------------

def _cpu_setup():
    torch.set_num_threads(os.cpu_count() or 1)
    make_fp8_weight = workloads().make_fp8_weight
    gen = torch.Generator().manual_seed(0)
    ws = {name: make_fp8_weight(N, K, gen) for name, N, K in SHAPES}
    xs = {(name, M): torch.randn(M, K, generator=gen).to(torch.float16)
          for name, N, K in SHAPES for M in MS}
    return ws, xs


def _cpu_step(O, ws, xs, frac: float) -> int:
    """Run the oracle on the first `frac` of the rows of each of the 12 GEMVs;
    returns the algorithmic bytes processed."""
    b = 0
    for (name, N, K, M) in CALLS:
        n = max(1, int(round(N * frac)))
        wq, sc = ws[name]
        O.gemv_fp8(xs[(name, M)], wq[:n], sc[:n])
        b += call_bytes(M, n, K)
    return b


def cpu_baseline_sample(seconds: float = 15.0) -> dict:
    from oracle import oracle as O
    ws, xs = _cpu_setup()
    _cpu_step(O, ws, xs, 1 / 64)  # warm
    t0 = time.perf_counter()
    b = _cpu_step(O, ws, xs, 1 / 16)
    dt = time.perf_counter() - t0
    frac = min(1.0, (1 / 16) * seconds / max(dt, 1e-3) / 2)
    t0 = time.perf_counter()
    b = _cpu_step(O, ws, xs, frac)
    dt = time.perf_counter() - t0
    # the two halves of the oracle separately, on the same sample: FP8 -> fp32
    # dequantisation of the weights, then the fp32 matmul
    t_deq = t_mm = 0.0
    for (name, N, K, M) in CALLS:
        n = max(1, int(round(N * frac)))
        wq, sc = ws[name]
        t0 = time.perf_counter()
        wf = O.fp8_decode(wq[:n], O.fp8_format_of(wq))
        t1 = time.perf_counter()
        _ = (xs[(name, M)].float() @ wf.T) * sc[:n]
        t2 = time.perf_counter()
        t_deq += t1 - t0
        t_mm += t2 - t1
    return {"value": round(b / dt / 1e9, 3), "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port", "seconds": round(dt, 2),
            "dequant_seconds": round(t_deq, 3), "matmul_seconds": round(t_mm, 3),
            "sample": f"first {frac:.3f} of the rows of each of the 12 config-1 GEMVs, torch fp32 "
                      "dequant-then-matmul (the reference tests' oracle); dequant and matmul also "
                      "timed apart on the same sample"}


def run_reference(args, rank, world):
    if rank != 0:
        return None
    from oracle import oracle as O
    ws, xs = _cpu_setup()
    budget = 150.0
    _cpu_step(O, ws, xs, 1 / 256)
    t0 = time.perf_counter()
    _cpu_step(O, ws, xs, 1 / 64)
    full = (time.perf_counter() - t0) * 64
    frac = max(1 / 2048, min(1.0, budget / max(1, args.steps + args.warmup) / full))
    for _ in range(args.warmup):
        _cpu_step(O, ws, xs, frac)
    t0 = time.perf_counter()
    b = 0
    for _ in range(args.steps):
        b += _cpu_step(O, ws, xs, frac)
    dt = time.perf_counter() - t0
    value = b / dt / 1e9
    sample = (f"each step: first {frac:.4f} of the rows of each of the 12 config-1 GEMVs "
              "(torch fp32 dequant-then-matmul on the host cores)")
    cores = torch.get_num_threads()
    return {"metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "e4m3*fp16->fp32",
            "data": "synthetic (seed 0)", "impl": "reference",
            "config": arm_config(world, not args.no_prefetch),
            "reference_path": "oracle port of the reference tests' torch CPU oracle "
                              "(the reference kernels are Intel-XPU ESIMD only)",
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores,
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def profile_steps():
    """Two eager steps of the config-1 sweep on one weight set (201 MB of
    weights, > L2): 24 launches of the GEMV kernel, nothing else in between."""
    import esimd_learning_b200 as ops
    dev = torch.device("cuda", 0)
    sets, xs, ys = build_sets(dev, n_sets=1)
    torch.cuda.synchronize()
    for _ in range(2):
        for (name, N, K, M) in CALLS:
            wq, sc = sets[0][name]
            ops.esimd_gemv_fp8_pern(xs[(name, M)], wq, sc, ys[(name, M)], N, K)
    torch.cuda.synchronize()
    print("profile steps done")


def _claim_stdout():
    """Route everything libraries print (NCCL banners, warnings) to stderr and
    return a file on the real stdout for the one JSON result line."""
    sys.stdout.flush()
    real = os.dup(1)
    os.dup2(2, 1)
    return os.fdopen(real, "w")


def profile_chain(M: int):
    """Two eager steps of the TP=1 decode chain of BASELINE config 4 (7 kernels
    each, 788 MB of weights)."""
    from esimd_learning_b200.chain import ChainShape, DecodeChain, full_weights, shard_weights
    dev = torch.device("cuda", 0)
    shape = ChainShape()
    chain = DecodeChain(shard_weights(full_weights(shape, seed=0, device=dev), shape, 0, 1), shape, M, dev)
    torch.cuda.empty_cache()
    h, r, a = (torch.randn(M, shape.hidden, device=dev).half() for _ in range(3))
    pos = torch.randint(0, shape.max_position, (M,), device=dev)
    for _ in range(2):
        chain.step(h, r, a, pos)
    torch.cuda.synchronize()
    print("profile chain done")


def profile_config2(M: int):
    """Two calls of the fused add+RMSNorm -> QKV GEMV of BASELINE config 2 at
    this M ([6144, 4096] e4m3 weight, fp32 per-channel scales)."""
    import esimd_learning_b200 as ops
    dev = torch.device("cuda", 0)
    h, r, g, wq, sc = (t.to(dev) for t in workloads().fused_norm_case(M))
    y = torch.empty(M, 6144, dtype=torch.float16, device=dev)
    for _ in range(2):
        ops.esimd_fused_add_rms_norm_batched_fp8(h, r, g, 1e-6, wq, sc, y)
    torch.cuda.synchronize()
    print("profile config2 done")


def profile_gemm(M: int):
    """Two launches each of the per-token quantisation and the tcgen05 GEMM of
    BASELINE config 3 at this M (A [M, 4096], B [14336, 4096])."""
    import esimd_learning_b200 as ops
    from esimd_learning_b200.workloads import prefill_case
    dev = torch.device("cuda", 0)
    a, bq, bs = prefill_case(M, device=dev)
    aq = torch.empty(M, 4096, dtype=torch.float8_e4m3fn, device=dev)
    as_ = torch.empty(M, dtype=torch.float32, device=dev)
    y = torch.empty(M, 14336, dtype=torch.float16, device=dev)
    for _ in range(2):
        ops.esimd_quant_fp8_per_token(a, aq, as_)
        ops.esimd_gemm_fp8_pertoken_pern(aq, as_, bq, bs, y)
    torch.cuda.synchronize()
    print("profile gemm done")


def main():
    out_file = _claim_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gemm", action="store_true", help="skip the config-3 GEMM measurement")
    ap.add_argument("--no-chain", action="store_true", help="skip the config-4 decode-chain measurement")
    ap.add_argument("--no-prefetch", action="store_true", help="GEMVs wait for the previous kernel before any load")
    ap.add_argument("--no-vllm", action="store_true", help="skip the vLLM FP8 linear comparison")
    ap.add_argument("--vllm-compare", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--profile-chain", type=int, default=0, metavar="M",
                    help="run two eager TP=1 decode-chain steps (config 4) at this M and exit; for ncu")
    ap.add_argument("--profile-config2", type=int, default=0, metavar="M",
                    help="run the fused add+RMSNorm -> QKV GEMV of config 2 at this M twice and exit; for ncu")
    ap.add_argument("--profile-gemm", type=int, default=0, metavar="M",
                    help="run quant + tcgen05 GEMM of config 3 at this M twice and exit; for ncu")
    ap.add_argument("--profile", action="store_true",
                    help="run two eager config-1 steps (24 GEMV launches) and exit; for ncu captures")
    args = ap.parse_args()
    if args.vllm_compare:
        print(json.dumps(vllm_compare()), file=out_file, flush=True)
        return
    if args.profile:
        profile_steps()
        return
    if args.profile_config2:
        profile_config2(args.profile_config2)
        return
    if args.profile_gemm:
        profile_gemm(args.profile_gemm)
        return
    if args.profile_chain:
        profile_chain(args.profile_chain)
        return
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        out = run_reference(args, rank, int(os.environ.get("WORLD_SIZE", "1")))
        if out is not None:
            print(json.dumps(out), file=out_file, flush=True)
        return
    rank, world, local = dist_init(args.gpus)
    out = run_ours(args, rank, world, local) if world == 1 else run_ours_tp(args, rank, world, local)
    if rank == 0:
        print(json.dumps(out), file=out_file, flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
