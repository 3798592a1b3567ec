"""Batched Newton-Schulz sweep and the small-case driver
for kernel profiles.

    python -m rollfast_b200.sweep                      # the config-4 sweep
    python -m rollfast_b200.sweep --shapes 4096x14336 --batch 2 --iters 5 --reps 1

For each (m, n) a batch of inputs X ~ N(0,1) / ||X||_F runs through
``rf_newton_schulz`` (the orthogonalize_fn seam) with the polar_express (n,3)
schedule for 5 and 8 iterations.  TFLOP/s counts the dense algorithmic NS
FLOPs (4 m^2 n + 2 m^3 per matrix per iteration, m <= n) over the CUDA-event
time of the whole call (normalisation pass included); ``gemm`` is the same
FLOPs over the GEMM-kernel time alone (per-launch events).

``--graph``: the call is captured once in a CUDA graph and replayed, so small
shapes are timed without the host's per-launch cost (the 18 launches of a
5-iteration call take longer to issue than to run below ~2048^2); the
reported ``tflops`` is then the graph replay's.
"""

from __future__ import annotations

import argparse
import json
import os

import torch

from . import _lib, _runtime
from .orthogonalization import quintic_newton_schulz, resolve_ns_coeffs

CONFIG4 = [(256, 256), (512, 512), (1024, 1024), (2048, 2048), (4096, 4096), (8192, 8192), (4096, 16384),
           (8192, 28672)]


def peak_tflops() -> tuple[float, str]:
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    p = os.path.join(root, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured bf16_tflops (burst)"
    return 1590.0, "fallback bf16 burst"


def run_case(m: int, n: int, batch: int, iters: int, reps: int, warmup: int, dev, graph: bool = False) -> dict:
    g = torch.Generator(device=dev)
    g.manual_seed(m * 131 + n)
    x = torch.randn((batch, m, n), device=dev, generator=g)
    x /= torch.linalg.vector_norm(x, dim=(-2, -1), keepdim=True)
    coeffs = resolve_ns_coeffs("polar_express", iters)
    for _ in range(warmup):
        out = quintic_newton_schulz(x, coeffs, iters)
    torch.cuda.synchronize()
    graph_ms = None
    if graph:
        # The workspace exists after the warm-up, so capture allocates only
        # the output (from the graph's pool); every launch is recorded.
        cg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(cg):
            gout = quintic_newton_schulz(x, coeffs, iters)
        cg.replay()
        torch.cuda.synchronize()
        gs, ge = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        gs.record()
        for _ in range(reps):
            cg.replay()
        ge.record()
        torch.cuda.synchronize()
        graph_ms = gs.elapsed_time(ge) / reps
        del gout, cg
    _lib.profile_begin()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        out = quintic_newton_schulz(x, coeffs, iters)
    e.record()
    torch.cuda.synchronize()
    prof = _lib.profile_end()
    ms = s.elapsed_time(e) / reps
    mm, nn = min(m, n), max(m, n)
    flops = batch * iters * (4 * mm * mm * nn + 2 * mm ** 3)
    del out
    extra = {}
    if graph_ms is not None:
        extra = {"eager_ms": round(ms, 3), "eager_tflops": round(flops / (ms * 1e-3) / 1e12, 1), "graph": True}
        ms = graph_ms
    return {"m": m, "n": n, "batch": batch, "iters": iters, "ms": round(ms, 3), **extra,
            "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
            "gemm_tflops": round(prof["algorithmic_flops"] / (prof["gemm_ms"] * 1e-3) / 1e12, 1)
            if prof["gemm_ms"] else None,
            "executed_tflops": round(prof["executed_flops"] / (prof["gemm_ms"] * 1e-3) / 1e12, 1)
            if prof["gemm_ms"] else None}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default=None, help="comma list of MxN (default: the config-4 list)")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--iters", default="5,8")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--precision", default="f16")
    ap.add_argument("--graph", action="store_true", help="time CUDA-graph replays of the call")
    args = ap.parse_args(argv)
    _runtime.set_ns_precision(args.precision)
    dev = torch.device("cuda", 0)
    shapes = CONFIG4 if args.shapes is None else [tuple(int(v) for v in s.split("x")) for s in args.shapes.split(",")]
    peak, src = peak_tflops()
    for m, n in shapes:
        for it in (int(v) for v in args.iters.split(",")):
            r = run_case(m, n, args.batch, it, args.reps, args.warmup, dev, graph=args.graph)
            r["frac_of_peak"] = round(r["tflops"] / peak, 3)
            r["peak"] = f"{peak} ({src})"
            r["precision"] = args.precision
            print(json.dumps(r), flush=True)
    _lib.sync_check(torch.cuda.current_stream().cuda_stream)


if __name__ == "__main__":
    main()
