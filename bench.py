"""Benchmark: one Muon optimizer step (``tx.update``) on the Llama-3-8B-shaped
parameter set with rollfast_b200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

A step is ``updates, state = tx.update(grads, state, params)`` for the whole
tree: 224 Muon matrix leaves (32 layers x q,k,v,o,gate,up,down, bf16) and the
AdamW fallback leaves (65 RMSNorm vectors, 128256x4096 embed and unembed).
Gradients are N(0,1) bf16 (two seeded sets, alternated so consecutive steps
differ); inputs (16 GB) are far larger than L2, so no flush is needed.
``--workload`` selects the other configurations (GPT-2 small, Llama-3-70B on
more than one GPU); their lines name their own metric and L2 note.

Printed JSON (rank 0): ``value`` = ms per step (max over ranks, CUDA events),
``e2e`` = the same through host buffers (pinned gradients H2D + updates D2H
inside the timed region), ``roofline`` = the Newton-Schulz tcgen05 GEMM
kernel's algorithmic TFLOP/s (live per-launch CUDA events) against the
measured bf16 peak, ``parity`` = one fresh step of the four Llama-3-8B matrix
shapes checked against the NumPy oracle after the timed region (and, on more
than one GPU, the sharded update against an unsharded recompute),
``cpu_baseline`` = the NumPy restatement in ``oracle/`` timed on this host's
cores on one layer (7 Muon leaves + 1/32 of the AdamW leaves) x 32.

``--preconditioning``, ``--adaptive`` and ``--mu-dtype`` time the path's
options on the same tree (the headline is the default, Frobenius / float32).
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


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# BLAS thread pools are sized when numpy is first imported, so rank 0 -- the
# only rank that runs CPU work (the reference arm, the cpu_baseline leg and
# the oracle side of the parity check) -- gets every host core here, before
# that import.  torchrun exports OMP_NUM_THREADS=1 to every rank.
if os.environ.get("RANK", "0") == "0":
    for _var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[_var] = str(host_threads())

import numpy as np  # noqa: E402
import torch  # noqa: E402

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Llama-3-8B Muon step ms at 1/2/4/8 B200; NS bf16 TFLOP/s vs peak"
FALLBACK_PEAKS = {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0}
# DRAM bytes per NS GEMM launch: one ncu capture of a 2-matrix 4096x14336
# sub-batch read+wrote 6738 MB over the 15 stage launches of a 5-iteration NS
# (449 MB per launch); the bench's launches hold 48 such matrices, whose
# per-matrix working set exceeds L2, so the bytes scale by 48/2.
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


def llama3_70b_shapes(layers: int = 80):
    """80 layers, hidden 8192, 64 query heads of 128
    (8192x8192 q, o), 8 KV heads (8192x1024 k, v), 8192x28672 gate / up,
    28672x8192 down; RMSNorm vectors to AdamW (no embedding in the config)."""
    layer = {"q": (8192, 8192), "k": (8192, 1024), "v": (8192, 1024), "o": (8192, 8192),
             "gate": (8192, 28672), "up": (8192, 28672), "down": (28672, 8192),
             "attn_norm": (8192,), "mlp_norm": (8192,)}
    return {"layers": [dict(layer) for _ in range(layers)], "final_norm": (8192,)}


def gpt2_small_shapes(layers: int = 12, vocab: int = 50257):
    """12 scanned layers (stacked leaves, reduction axis
    1, output axis 2) of 768x2304 qkv, 768x768 proj, 768x3072 fc and 3072x768
    fc_out; LayerNorm gains and biases (stacked vectors) and the 50257x768
    embedding to AdamW."""
    L = layers
    return {"layers": [{"qkv": (L, 768, 2304), "proj": (L, 768, 768), "fc": (L, 768, 3072),
                        "fc_out": (L, 3072, 768), "ln1_g": (L, 768), "ln1_b": (L, 768), "ln2_g": (L, 768),
                        "ln2_b": (L, 768)}], "final_norm": (768,), "embed": (vocab, 768)}


def muon_specs(shapes, rf, name=None):
    """2-D weight matrices -> Muon; vectors, embed and unembed -> AdamW."""
    if isinstance(shapes, dict):
        return {k: muon_specs(v, rf, k) for k, v in shapes.items()}
    if isinstance(shapes, list):
        return [muon_specs(v, rf, name) for v in shapes]
    if len(shapes) == 3:  # a stack of scanned layers: (layer, rows, cols)
        return rf.MatrixDimensionNumbers(1, 2)
    if len(shapes) == 2 and name not in ("embed", "unembed") and not name.startswith("ln"):
        return rf.MatrixDimensionNumbers()
    return None


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
    for s in muon_matrix_shapes(shapes):
        b = s[0] if len(s) == 3 else 1
        m, n = min(s[-2:]), max(s[-2:])
        tot += b * (4 * m * m * n + 2 * m ** 3) * steps
    return tot


def muon_matrix_shapes(shapes):
    return [s for layer in shapes["layers"] for k, s in layer.items() if len(s) >= 2 and not k.startswith("ln")]


WORKLOADS = {
    # name: (shapes fn, muon kwargs, BASELINE config)
    "llama3_8b_muon_step": (llama3_8b_shapes, {}, "configs[2]"),
    "llama3_70b_muon_step": (llama3_70b_shapes, {"momentum_accumulator": "heavy_ball", "nesterov": False},
                             "configs[4]"),
    "gpt2_small_muon_step": (gpt2_small_shapes, {"ns_coeffs": "polar_express"}, "configs[1]"),
}


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

LAYERS = 32
LAYER_MATRICES = [("q", (4096, 4096)), ("k", (4096, 1024)), ("v", (4096, 1024)), ("o", (4096, 4096)),
                  ("gate", (4096, 14336)), ("up", (4096, 14336)), ("down", (14336, 4096))]
# One layer's share of the AdamW leaves: 1/32 of the embed and unembed rows,
# its two RMSNorm vectors (the final norm, 1/8 of a layer's, is left out).
ADAM_SLICE = {"embed": (128256 // LAYERS, 4096), "unembed": (128256 // LAYERS, 4096),
              "attn_norm": (4096,), "mlp_norm": (4096,)}
SAMPLE_KINDS = [k for k, _ in LAYER_MATRICES] + ["adamw"]
CPU_SAMPLE_TEXT = ("oracle NumPy fp32 update of one Llama-3-8B layer (its 7 Muon leaves + 1/32 of the AdamW "
                   "leaves, each a one-leaf oracle step with bf16 params), x 32")


class OracleLayerSample:
    """The reference path restated in NumPy (``oracle/``, the checker) timed
    on one Llama-3-8B layer: each of the layer's 7 Muon leaves, and its share
    of the AdamW leaves, as one oracle step (fresh state, lr 0.02, wd 0.01,
    beta 0.95, 5 standard NS iterations, bf16 parameter rounding)."""

    def __init__(self, seed: int = 0):
        import oracle as O

        self.O = O
        self.seed = seed

    def _case(self, kind: str):
        O = self.O
        rng = np.random.default_rng(self.seed + SAMPLE_KINDS.index(kind))
        shapes = dict(LAYER_MATRICES)
        tree = {kind: shapes[kind]} if kind != "adamw" else ADAM_SLICE
        specs = {k: None for k in tree} if kind == "adamw" else None
        p = {k: O.bf16_round((rng.standard_normal(s) * 0.02).astype(np.float32)) for k, s in tree.items()}
        g = {k: O.bf16_round(rng.standard_normal(s).astype(np.float32)) for k, s in tree.items()}
        ora = O.OracleMuon(learning_rate=0.02, weight_decay=0.01, beta=0.95, muon_weight_dimension_numbers=specs)
        return ora, ora.init(p), g, p, {k: "bfloat16" for k in tree}

    def time_kind(self, kind: str) -> float:
        ora, st, g, p, dts = self._case(kind)
        t0 = time.perf_counter()
        ora.update(g, st, p, param_dtypes=dts)
        return (time.perf_counter() - t0) * 1e3


def blas_threads() -> int | None:
    """Threads of the BLAS pool numpy uses, as it reports them."""
    try:
        from threadpoolctl import threadpool_info

        counts = [d.get("num_threads") for d in threadpool_info() if d.get("user_api") == "blas"]
        return max(c for c in counts if c) if counts else None
    except Exception:  # noqa: BLE001 - diagnostics only
        return None


def cpu_layer_baseline() -> dict:
    """``cpu_baseline`` of our own line: every sample kind once."""
    s = OracleLayerSample()
    per = {k: s.time_kind(k) for k in SAMPLE_KINDS}
    layer_ms = sum(per.values())
    return {"value": round(LAYERS * layer_ms, 1), "unit": "ms", "cores": blas_threads() or host_threads(),
            "kind": "port", "sample": f"{CPU_SAMPLE_TEXT} (one layer {layer_ms:.0f} ms)",
            "per_leaf_ms": {k: round(v, 1) for k, v in per.items()}}


# ---------------------------------------------------------------------------

def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def run_reference(args, rank, world):
    """--impl reference: the reference path's CPU restatement (the oracle
    port; the reference itself needs JAX, which this image lacks) on every
    host core, rank 0 only.  Each step times one leaf kind of one Llama-3-8B
    layer (the 7 Muon matrices and the layer's AdamW share, in turn); the
    reported step is 32 x the sum over kinds of each kind's median."""
    if rank != 0:
        return
    s = OracleLayerSample()
    n_timed = max(args.steps, len(SAMPLE_KINDS))
    times = {k: [] for k in SAMPLE_KINDS}
    for i in range(args.warmup + n_timed):
        kind = SAMPLE_KINDS[i % len(SAMPLE_KINDS)]
        ms = s.time_kind(kind)
        if i >= args.warmup:
            times[kind].append(ms)
    layer_ms = sum(statistics.median(v) for v in times.values())
    val = LAYERS * layer_ms
    threads = blas_threads() or host_threads()
    out = {
        "impl": "reference", "metric": METRIC, "value": round(val, 1), "unit": "ms",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(val, 1),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: N(0,1) grads, N(0,0.02) params, bf16-rounded",
        "config": {"workload": "llama3_8b_muon_step", "sample": "one layer x 32",
                   "timed_samples": n_timed, "blas_threads": threads},
        "cpu_baseline": {"value": round(val, 1), "unit": "ms", "cores": threads, "kind": "port",
                         "sample": f"{CPU_SAMPLE_TEXT}; one leaf kind per step, median per kind "
                                   f"(one layer {layer_ms:.0f} ms)",
                         "per_leaf_ms": {k: round(statistics.median(v), 1) for k, v in times.items()}},
        "e2e": {"value": round(val, 1), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


PARITY_SHAPES = {"q": (4096, 4096), "k": (4096, 1024), "gate": (4096, 14336), "down": (14336, 4096),
                 "norm": (4096,)}
# Llama-3-70B: the q and k/v shapes (the 8192x28672 leaves would take the
# oracle minutes on the host).
PARITY_SHAPES_70B = {"q": (8192, 8192), "k": (8192, 1024), "norm": (8192,)}
PARITY_TOL = {"muon": 1e-2, "adamw": 1e-6, "sharded": 1e-2}


def parity_check(rf, dev, dist, rank: int, world: int, shapes=None, muon_kw=None) -> dict:
    """One fresh step (lr 0.02, wd 0.01, beta 0.95, 5 standard iterations) of
    a tree with the workload's matrix shapes and one AdamW vector, run after
    the timed region.  Rank 0 compares the updates with the oracle (NumPy
    float32) on the same inputs; on more than one GPU every rank runs the
    sharded update (in the workload's mode) and rank 0 also recomputes it
    unsharded and compares the leaves it holds."""
    shapes = PARITY_SHAPES if shapes is None else shapes
    muon_kw = muon_kw or {}
    rng = np.random.default_rng(4321)
    import oracle as O

    p_np = {k: O.bf16_round((rng.standard_normal(s) * 0.02).astype(np.float32)) for k, s in shapes.items()}
    g_np = {k: O.bf16_round(rng.standard_normal(s).astype(np.float32)) for k, s in shapes.items()}
    to = lambda a: torch.from_numpy(a).to(dev).to(torch.bfloat16)  # noqa: E731
    params = {k: to(v) for k, v in p_np.items()}
    grads = {k: to(v) for k, v in g_np.items()}

    def step():
        tx = rf.muon(learning_rate=0.02, weight_decay=0.01, beta=0.95, **muon_kw)
        u, _ = tx.update(grads, tx.init(params), params)
        torch.cuda.synchronize()
        return {k: (None if v.is_meta else v.float().cpu().numpy()) for k, v in u.items()}

    got = step()
    out = {"leaves": {k: list(s) for k, s in shapes.items()}, "tol": dict(PARITY_TOL), "options": dict(muon_kw),
           "reference": "oracle NumPy fp32, one fresh step on the same bf16 inputs"}
    if world > 1:
        unsharded = None
        if rank == 0:
            prev = rf.distributed.use(None)
            try:
                unsharded = step()
            finally:
                rf.distributed.use(prev)
        dist.barrier()
        if rank == 0:
            held = [k for k in shapes if got[k] is not None]
            out["sharded_vs_unsharded"] = max(rel_err(got[k], unsharded[k]) for k in held) if held else 0.0
            out["sharded_leaves_compared"] = held
            got = unsharded
    if rank == 0:
        okw = {"momentum_accumulator": muon_kw.get("momentum_accumulator", "ema"),
               "nesterov": muon_kw.get("nesterov", True)}
        tx_o = O.OracleMuon(learning_rate=0.02, weight_decay=0.01, beta=0.95, **okw)
        ref, _ = tx_o.update(g_np, tx_o.init(p_np), p_np, param_dtypes={k: "bfloat16" for k in shapes})
        errs = {k: rel_err(got[k], ref[k]) for k in shapes}
        out["rel_err"] = {k: float(f"{v:.3e}") for k, v in errs.items()}
        out["max_rel_err_muon"] = max(v for k, v in errs.items() if k != "norm")
        out["max_rel_err_adamw"] = errs["norm"]
        ok = out["max_rel_err_muon"] <= PARITY_TOL["muon"] and out["max_rel_err_adamw"] <= PARITY_TOL["adamw"]
        if world > 1:
            ok = ok and out["sharded_vs_unsharded"] <= PARITY_TOL["sharded"]
        out["pass"] = bool(ok)
    if dist is not None:
        dist.barrier()
    return out


def rel_err(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def run_e2e(args, tx, state, params, grad_sets, shapes, dev, barrier, dist, rf=None):
    """Same step through host buffers: pinned gradients copied H2D and the
    update tree copied D2H inside the timed region, every step.  On one GPU
    the whole tree both ways.  Sharded, the host holds one gradient tree and
    receives one update tree, split across the GPUs: each rank copies in the
    gradient elements it owns and copies out the update elements it computed
    (``distributed.owned_parts``); under updates="owned" that is its owned
    leaves."""
    torch.cuda.empty_cache()
    dev_g = grad_sets[1]
    flat = leaves_of(dev_g)
    # (flat leaf view, element range) this rank copies, per leaf.
    if dist is not None and rf is not None and any(rf.distributed.owned_parts()):
        muon_pos, adam_parts = rf.distributed.owned_parts()
        ranges = {p: (0, flat[p].numel()) for p in muon_pos}
        ranges.update({p: (a, b) for p, a, b in adam_parts})
    else:
        ranges = {p: (0, t.numel()) for p, t in enumerate(flat) if not t.is_meta}
    pos = sorted(ranges)
    host_g = [torch.empty(ranges[p][1] - ranges[p][0], dtype=torch.bfloat16, pin_memory=True) for p in pos]
    src0 = leaves_of(grad_sets[0])
    for hg, p in zip(host_g, pos):
        a, b = ranges[p]
        hg.copy_(src0[p].reshape(-1)[a:b])
    host_u = [torch.empty(ranges[p][1] - ranges[p][0], dtype=torch.float32, pin_memory=True) for p in pos]
    h2d = sum(t.numel() * t.element_size() for t in host_g)
    d2h = sum(t.numel() * t.element_size() for t in host_u)
    k = args.e2e_steps or max(2, min(args.steps, 5))
    upd, state = tx.update(dev_g, state, params)  # warm the output allocations
    del upd
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(k):
        for hg, p in zip(host_g, pos):
            a, b = ranges[p]
            flat[p].view(-1)[a:b].copy_(hg, non_blocking=True)
        upd, state = tx.update(dev_g, state, params)
        ups = leaves_of(upd)
        for hu, p in zip(host_u, pos):
            a, b = ranges[p]
            hu.copy_(ups[p].reshape(-1)[a:b], non_blocking=True)
        upd = None  # the copies are stream-ordered before any reuse of these blocks
    e1.record()
    barrier()
    e_ms = e0.elapsed_time(e1) / k
    if dist is not None:
        t = torch.tensor([e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    split = dist is not None and rf is not None and any(rf.distributed.owned_parts())
    return {"value": round(e_ms, 2), "unit": "ms", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "steps": k, "bytes": "per rank" if dist is not None else "whole tree",
            "path": "rollfast_b200.muon(...).update with pinned host grads/updates"
                    + (": each rank copies the gradient elements it owns in and the updates it computed out"
                       if split else "")}


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
    ap.add_argument("--workload", default="llama3_8b_muon_step", choices=sorted(WORKLOADS))
    ap.add_argument("--layers", type=int, default=None,
                    help="reduced-size case for kernel profiles only (the headline is the full model)")
    ap.add_argument("--vocab", type=int, default=128256)
    ap.add_argument("--preconditioning", default="frobenius", choices=["frobenius", "aol", "schatten", "spectral"])
    ap.add_argument("--adaptive", action="store_true")
    ap.add_argument("--mu-dtype", default="float32", choices=["float32", "bfloat16"])
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--apply-updates", action="store_true",
                    help="time update_and_apply (the parameter apply fused into the update, bf16 stochastic "
                         "rounding, in place) instead of the update alone")
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
    shape_fn, muon_kw, baseline_cfg = WORKLOADS[args.workload]
    owned_mode = args.workload == "llama3_70b_muon_step"
    if owned_mode and world == 1 and args.layers is None:
        raise SystemExit("llama3_70b_muon_step needs 8 GPUs (replicated updates do not fit one B200); "
                         "use --layers for a reduced case")
    if world > 1:
        # The 70B tree runs with owners keeping their updates (no exchange):
        # its float32 update tree (274 GB) does not fit one GPU.
        rf.distributed.configure(updates="owned" if owned_mode else "all")
    rf.set_ns_precision(args.precision)

    full_size = args.layers is None and (args.vocab == 128256 or args.workload != "llama3_8b_muon_step")
    if args.workload == "llama3_8b_muon_step":
        shapes = llama3_8b_shapes(32 if args.layers is None else args.layers, args.vocab)
    elif args.workload == "gpt2_small_muon_step":
        shapes = gpt2_small_shapes(12 if args.layers is None else args.layers)
    else:
        shapes = llama3_70b_shapes(80 if args.layers is None else args.layers)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234)  # data-parallel: every rank holds the same (reduced) gradients

    specs = muon_specs(shapes, rf)
    if owned_mode and world > 1:
        meta = map_shapes(shapes, lambda s: torch.empty(s, dtype=torch.bfloat16, device="meta"))
        owners = rf.distributed.ownership(meta, specs, world)
    else:
        owners = map_shapes(shapes, lambda s: rank)

    def leaf_maker(scale):
        own = iter(leaves_of(owners))

        def make(s):
            if next(own) != rank:
                return torch.empty(s, dtype=torch.bfloat16, device="meta")  # another rank's leaf
            t = torch.empty(s, dtype=torch.bfloat16, device=dev)
            t.normal_(0.0, scale, generator=gen)
            return t
        return make

    params = map_shapes(shapes, leaf_maker(0.02))
    grad_sets = [map_shapes(shapes, leaf_maker(1.0)) for _ in range(2)]
    variant = {}
    if args.preconditioning != "frobenius":
        variant["preconditioning"] = args.preconditioning
    if args.adaptive:
        variant["adaptive"] = True
    if args.mu_dtype != "float32":
        variant["mu_dtype"] = torch.bfloat16
    tx = rf.muon(learning_rate=0.02, weight_decay=0.01, beta=0.95, muon_weight_dimension_numbers=specs, **muon_kw,
                 **variant)
    state = tx.init(params)
    torch.cuda.synchronize()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    # Like a training loop, each step's updates are dropped (applied) before
    # the next step: holding two update trees (2 x 30 GiB) beside the state
    # and two gradient sets would leave little of the 178 GiB free.
    apply_key = torch.tensor([0, 7])

    def one_step(i, state):
        if args.apply_updates:  # new parameters written in place; no update tree
            _, state = rf.update_and_apply(tx, grad_sets[i % 2], state, params, apply_key, stochastic=True,
                                           inplace=True)
            return None, state
        return tx.update(grad_sets[i % 2], state, params)

    for i in range(args.warmup):
        upd = None
        upd, state = one_step(i, state)
    barrier()

    launches0 = _lib.kernel_launch_count()
    _lib.profile_begin()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        start.record()
        for i in range(args.steps):
            upd = None
            upd, state = one_step(i, state)
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
    if not args.no_e2e and not args.apply_updates:
        try:
            e2e = run_e2e(args, tx, state, params, grad_sets, shapes, dev, barrier, dist, rf)
        except (RuntimeError, MemoryError) as exc:  # host RAM for pinned buffers
            e2e = {"value": None, "unit": "ms", "unavailable": f"{type(exc).__name__}: {exc}"[:200]}
        grad_sets = None

    # ---- parity of the same code path, after (outside) the timed region ---
    del tx, state, params
    torch.cuda.empty_cache()
    parity = None if args.no_parity else parity_check(
        rf, dev, dist, rank, world, PARITY_SHAPES_70B if owned_mode else PARITY_SHAPES,
        {k: v for k, v in muon_kw.items() if k != "ns_coeffs"})

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload == "llama3_8b_muon_step":
        cpu = cpu_layer_baseline()
    n_layers = len(shapes["layers"]) if args.workload != "gpt2_small_muon_step" else shapes["layers"][0]["qkv"][0]
    workload = args.workload if full_size else f"{args.workload}_reduced_{n_layers}_layers_vocab_{args.vocab}"
    model = {"llama3_8b_muon_step": "Llama-3-8B", "llama3_70b_muon_step": "Llama-3-70B",
             "gpt2_small_muon_step": "GPT-2 small"}[args.workload] + f" ({n_layers} layers) parameter set"
    transport = {"ce+owner_tail": ", copy-engine pushes into IPC-mapped peer update arenas: 16-bit O per Muon "
                                  "bucket (tail on every rank), float32 AdamW updates (split by element range)",
                 "ce": ", copy-engine all-gather of 16-bit O into IPC-mapped peer buffers",
                 "nccl": ", NCCL all-gather"}.get(rf.distributed.active_transport(), "") if world > 1 else ""
    if owned_mode and world > 1:
        transport = ", owners keep their leaves' updates (no exchange: the float32 update tree does not fit a GPU)"
    grad_gb = sum(math.prod(s) for s in leaves_of(shapes)) * 2 / 1e9  # one bf16 gradient set
    # The traffic figure comes from a capture of the one-GPU Llama-3-8B
    # 4096x14336 sub-batch launches; other workloads' launches, and sharded
    # ones (a rank's own leaves only), hold other matrices.
    traffic = TRAFFIC_PER_LAUNCH if (full_size and args.workload == "llama3_8b_muon_step" and world == 1) else None

    if rank == 0:
        out = {
            "metric": METRIC if args.workload == "llama3_8b_muon_step" else model.split(" (")[0] + " Muon step ms",
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
            "config": {"workload": workload
                       + "".join(f"+{k}={v if k != 'mu_dtype' else args.mu_dtype}" for k, v in variant.items())
                       + ("+update_and_apply" if args.apply_updates else ""),
                       "baseline_config": baseline_cfg,
                       "model": model,
                       "muon_leaves": len(muon_matrix_shapes(shapes)),
                       "adam_leaves": len(leaves_of(shapes)) - len(muon_matrix_shapes(shapes)), "ns_steps": 5,
                       "ns_coeffs": muon_kw.get("ns_coeffs", "standard"),
                       "options": {k: v for k, v in muon_kw.items() if k != "ns_coeffs"},
                       "l2": (f"inputs ({grad_gb:.2f} GB bf16 grads per step, plus state) > 126 MB L2; no flush"
                              if grad_gb > 0.126 else f"reduced: {grad_gb:.3f} GB of grads per step can sit in L2"),
                       "parallelism": f"muon leaves FLOP-balanced over {world} GPU(s)" + transport},
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
                # stages (80% of the step's FLOPs): see TRAFFIC_PER_LAUNCH.
                "traffic": traffic,
                "traffic_unit": "bytes per launch",
            },
            "gpu_launches": launches,
            "clocks": clocks.summary(),
            "e2e": e2e,
            "parity": parity,
            "cpu_baseline": cpu,
        }
        print(json.dumps(out), flush=True)
    if dist is not None:
        rf.distributed.clear()  # collective: unmaps the peers' buffers once every rank is idle
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
