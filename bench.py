"""Benchmark: one Muon optimizer step (``tx.update``) on the Llama-3-8B-shaped
parameter set with rollfast_b200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

A step is ``updates, state = tx.update(grads, state, params)`` for the whole
tree: 224 Muon matrix leaves (32 layers x q,k,v,o,gate,up,down, bf16) and the
AdamW fallback leaves (65 RMSNorm vectors, 128256x4096 embed and unembed).
Gradients are N(0,1) bf16 (two seeded sets, alternated so consecutive steps
differ); inputs (16 GB) are far larger than L2, so no flush is needed.

Printed JSON (rank 0): ``value`` = ms per step (max over ranks, CUDA events),
``e2e`` = the same through host buffers (pinned gradients H2D + updates D2H
inside the timed region), ``roofline`` = the Newton-Schulz tcgen05 GEMM
kernel's algorithmic TFLOP/s (live per-launch CUDA events) against the
measured bf16 peak, ``cpu_baseline`` = the NumPy restatement in ``oracle/``
timed on this host's cores on one 4096x4096 leaf and extrapolated by FLOPs.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Llama-3-8B Muon step ms at 1/2/4/8 B200; NS bf16 TFLOP/s vs peak"
FALLBACK_PEAKS = {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0}
# ncu: 2-matrix capture, 15 stage launches of a 5-iteration NS = 6738 MB -> 449 MB per launch; x 48/2.
TRAFFIC_PER_LAUNCH = round(6738e6 / 15 * 24)


# ---------------------------------------------------------------------------
# Workload
# ---------------------------------------------------------------------------

def llama3_8b_shapes(layers: int = 32, vocab: int = 128256):
    layer = {"q": (4096, 4096), "k": (4096, 1024), "v": (4096, 1024), "o": (4096, 4096),
             "gate": (4096, 14336), "up": (4096, 14336), "down": (14336, 4096),
             "attn_norm": (4096,), "mlp_norm": (4096,)}
    return {"layers": [dict(layer) for _ in range(layers)], "final_norm": (4096,),
            "embed": (vocab, 4096), "unembed": (vocab, 4096)}


def muon_specs(shapes, rf):
    """2-D weight matrices -> Muon; vectors, embed and unembed -> AdamW."""
    def spec(path_leaf_name, s):
        if len(s) == 2 and path_leaf_name not in ("embed", "unembed"):
            return rf.MatrixDimensionNumbers()
        return None
    return {
        "layers": [{k: spec(k, s) for k, s in layer.items()} for layer in shapes["layers"]],
        "final_norm": None, "embed": None, "unembed": None,
    }


def map_shapes(shapes, fn):
    if isinstance(shapes, dict):
        return {k: map_shapes(v, fn) for k, v in shapes.items()}
    if isinstance(shapes, list):
        return [map_shapes(v, fn) for v in shapes]
    return fn(shapes)


def leaves_of(tree):
    if isinstance(tree, dict):
        out = []
        for v in tree.values():
            out += leaves_of(v)
        return out
    if isinstance(tree, list):
        out = []
        for v in tree:
            out += leaves_of(v)
        return out
    return [tree]


def ns_alg_flops(shapes, steps=5):
    tot = 0
    for s in leaves_of(muon_matrix_shapes(shapes)):
        m, n = min(s), max(s)
        tot += (4 * m * m * n + 2 * m ** 3) * steps
    return tot


def muon_matrix_shapes(shapes):
    return [s for layer in shapes["layers"] for k, s in layer.items() if len(s) == 2]


# ---------------------------------------------------------------------------
# Clock sampling (nvidia-smi, during the timed region)
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int, interval_ms: int = 50):
        self.index = index
        self.interval_ms = interval_ms
        self.proc = None
        self.lines = []
        self.skip = 0

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms",
                 str(self.interval_ms), "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            # nvidia-smi takes a moment to start: wait for its first sample
            # (taken before the timed region, so it is not counted) so that
            # even a sub-second timed region is sampled.
            t0 = time.monotonic()
            while not self.lines and self.proc.poll() is None and time.monotonic() - t0 < 10.0:
                time.sleep(0.01)
            self.skip = len(self.lines)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines[self.skip:]:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for nm, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU baseline: the oracle (NumPy float32 restatement) on this host's cores.
# ---------------------------------------------------------------------------

def cpu_sample_ms(reps: int = 1):
    """Time one full Muon step of a single 4096x4096 leaf on the oracle."""
    import oracle as O

    rng = np.random.default_rng(0)
    p = {"q": (rng.standard_normal((4096, 4096)) * 0.02).astype(np.float32)}
    g = {"q": rng.standard_normal((4096, 4096)).astype(np.float32)}
    ora = O.OracleMuon(learning_rate=0.02, weight_decay=0.01)
    st = ora.init(p)
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        _, st = ora.update(g, st, p, param_dtypes={"q": "bfloat16"})
        times.append((time.perf_counter() - t0) * 1e3)
    sample_flops = (4 * 4096 ** 3 + 2 * 4096 ** 3) * 5
    return statistics.median(times), sample_flops


def cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------

def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def run_reference(args, rank, world):
    """--impl reference: the oracle port on host cores (rank 0 only)."""
    if rank != 0:
        return
    n = cores()
    for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ.setdefault(var, str(n))
    shapes = llama3_8b_shapes()
    step_flops = ns_alg_flops(shapes)
    samples = []
    for i in range(args.warmup + args.steps):
        ms, sflops = cpu_sample_ms(1)
        if i >= args.warmup:
            samples.append(ms * step_flops / sflops)
    val = statistics.median(samples)
    out = {
        "impl": "reference", "metric": METRIC, "value": round(val, 1), "unit": "ms",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(val, 1),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "llama3_8b_muon_step", "sample": "one 4096x4096 leaf, extrapolated by NS FLOPs"},
        "cpu_baseline": {"value": round(val, 1), "unit": "ms", "cores": n, "kind": "port",
                         "sample": "oracle NumPy fp32 Muon step of one 4096x4096 leaf per step, x NS-FLOP ratio "
                                   f"{step_flops / sflops:.1f}"},
        "e2e": {"value": round(val, 1), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


def run_e2e(args, tx, state, params, grad_sets, shapes, dev, barrier, dist):
    """Same step through host buffers: pinned gradients copied H2D and the
    update tree copied D2H inside the timed region, every step."""
    torch.cuda.empty_cache()
    host_g = map_shapes(shapes, lambda s: torch.empty(s, dtype=torch.bfloat16, pin_memory=True))
    for hg, dg in zip(leaves_of(host_g), leaves_of(grad_sets[0])):
        hg.copy_(dg)
    dev_g = grad_sets[1]
    host_u = map_shapes(shapes, lambda s: torch.empty(s, dtype=torch.float32, pin_memory=True))
    h2d = sum(t.numel() * t.element_size() for t in leaves_of(host_g))
    d2h = sum(t.numel() * t.element_size() for t in leaves_of(host_u))
    k = args.e2e_steps or max(2, min(args.steps, 5))
    upd, state = tx.update(dev_g, state, params)  # warm the output allocations
    del upd
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(k):
        for hg, dg in zip(leaves_of(host_g), leaves_of(dev_g)):
            dg.copy_(hg, non_blocking=True)
        upd, state = tx.update(dev_g, state, params)
        for hu, du in zip(leaves_of(host_u), leaves_of(upd)):
            hu.copy_(du, non_blocking=True)
        upd = None  # the copies are stream-ordered before any reuse of these blocks
    e1.record()
    barrier()
    e_ms = e0.elapsed_time(e1) / k
    if dist is not None:
        t = torch.tensor([e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    return {"value": round(e_ms, 2), "unit": "ms", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "steps": k, "path": "rollfast_b200.muon(...).update with pinned host grads/updates"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--precision", default="f16", choices=["f16", "bf16", "f32"])
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--layers", type=int, default=32,
                    help="reduced-size case for kernel profiles only (the headline is 32 layers)")
    ap.add_argument("--vocab", type=int, default=128256)
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")

    import rollfast_b200 as rf
    from rollfast_b200 import _lib

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        rf.distributed.configure()
    rf.set_ns_precision(args.precision)

    shapes = llama3_8b_shapes(args.layers, args.vocab)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234)

    def randn(s, scale=1.0):
        t = torch.empty(s, dtype=torch.bfloat16, device=dev)
        t.normal_(0.0, scale, generator=gen)
        return t

    params = map_shapes(shapes, lambda s: randn(s, 0.02))
    grad_sets = [map_shapes(shapes, lambda s: randn(s)) for _ in range(2)]
    specs = muon_specs(shapes, rf)
    tx = rf.muon(learning_rate=0.02, weight_decay=0.01, beta=0.95, muon_weight_dimension_numbers=specs)
    state = tx.init(params)
    torch.cuda.synchronize()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    # Like a training loop, each step's updates are dropped (applied) before
    # the next step: holding two update trees (2 x 30 GiB) beside the state
    # and two gradient sets would leave little of the 178 GiB free.
    for i in range(args.warmup):
        upd = None
        upd, state = tx.update(grad_sets[i % 2], state, params)
    barrier()

    launches0 = _lib.kernel_launch_count()
    _lib.profile_begin()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        start.record()
        for i in range(args.steps):
            upd = None
            upd, state = tx.update(grad_sets[i % 2], state, params)
        stop.record()
        barrier()
    prof = _lib.profile_end()
    del upd
    launches = _lib.kernel_launch_count() - launches0
    ms = start.elapsed_time(stop) / args.steps
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    _lib.sync_check(torch.cuda.current_stream().cuda_stream)

    peaks, peak_src = load_peaks()
    gemm_ms_launch = prof["gemm_ms"] / max(prof["launches"], 1)
    alg_per_launch = prof["algorithmic_flops"] / max(prof["launches"], 1)
    achieved = alg_per_launch / (gemm_ms_launch * 1e-3) / 1e12 if prof["launches"] else None
    executed = prof["executed_flops"] / (prof["gemm_ms"] * 1e-3) / 1e12 if prof["gemm_ms"] else None
    peak = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))

    # ---- e2e through host buffers (pinned grads H2D + updates D2H) ----------
    e2e = None
    if not args.no_e2e:
        try:
            e2e = run_e2e(args, tx, state, params, grad_sets, shapes, dev, barrier, dist)
        except (RuntimeError, MemoryError) as exc:  # host RAM for pinned buffers
            e2e = {"value": None, "unit": "ms", "unavailable": f"{type(exc).__name__}: {exc}"[:200]}
        grad_sets = None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        n = cores()
        s_ms, s_flops = cpu_sample_ms(1)
        cpu = {"value": round(s_ms * ns_alg_flops(shapes) / s_flops, 1), "unit": "ms", "cores": n, "kind": "port",
               "sample": f"oracle NumPy fp32 Muon step of one 4096x4096 leaf ({s_ms:.0f} ms), extrapolated by "
                         "NS FLOPs to the full step"}

    if rank == 0:
        out = {
            "metric": METRIC,
            "value": round(ms, 2),
            "unit": "ms",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 2),
            "higher_is_better": False,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": f"{args.precision} NS operands, fp32 accumulate/state, bf16 params+grads",
            "data": "synthetic: N(0,1) bf16 grads (2 seeded sets), N(0,0.02) bf16 params",
            "config": {"workload": "llama3_8b_muon_step" if (args.layers, args.vocab) == (32, 128256)
                       else f"reduced_{args.layers}_layers_vocab_{args.vocab}",
                       "model": f"Llama-3-8B ({args.layers} layers) parameter set",
                       "muon_leaves": 7 * args.layers, "adam_leaves": 2 * args.layers + 3, "ns_steps": 5,
                       "ns_coeffs": "standard",
                       "l2": "inputs (16 GB grads) >> 126 MB L2; no flush",
                       "parallelism": f"muon leaves FLOP-balanced over {world} GPU(s)"
                       + ({"ce": ", copy-engine all-gather into IPC-mapped peer buffers",
                           "nccl": ", NCCL all-gather"}.get(rf.distributed.active_transport(), "")
                          if world > 1 else "")},
            "ns_tflops_algorithmic": round(ns_alg_flops(shapes) / (ms * 1e-3) / 1e12, 1),
            "roofline": {
                "bound": "tensor",
                "kernel": "k_ns_tc (tcgen05 NS GEMM stages)",
                "achieved": round(achieved, 1) if achieved else None,
                "peak": peak,
                "unit": "TFLOP/s",
                "frac": round(achieved / peak, 3) if achieved else None,
                "peak_source": f"{peak_src} bf16_tflops_sustained",
                "executed_tflops": round(executed, 1) if executed else None,
                "launches": prof["launches"],
                "gemm_ms_per_step": round(prof["gemm_ms"] / args.steps, 2),
                # DRAM read+write bytes per launch of the 4096x14336 sub-batch
                # stages (80% of the step's FLOPs), from the ncu capture in
                # profiles/k_ns_tc2_4096x14336_b2.md: 449 MB per launch at 2
                # matrices, scaled to the bench's 48-matrix launches (the
                # per-matrix working set exceeds L2, so bytes grow with it).
                "traffic": TRAFFIC_PER_LAUNCH if (args.layers, args.vocab) == (32, 128256) else None,
                "traffic_unit": "bytes per launch",
            },
            "gpu_launches": launches,
            "clocks": clocks.summary(),
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        print(json.dumps(out), flush=True)
    if dist is not None:
        rf.distributed.clear()  # collective: unmaps the peers' buffers once every rank is idle
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
