"""Step time of the reference path's options on the Llama-3-8B-shaped tree
(one B200): the full ``muon(...).update`` with each preconditioning, with
``adaptive``, and with bfloat16 optimizer state, next to the default; and
``apply_updates`` over the whole tree (round-to-nearest and stochastic).
One JSON line per case, CUDA-event timed on the launching stream after
warm-up; inputs (16 GB of gradients) are far larger than L2.

    python -m rollfast_b200.bench_options [--steps 3] [--warmup 2] [--layers 32]
"""

from __future__ import annotations

import argparse
import json

import torch


def llama_shapes(layers: int, vocab: int = 128256, d: int = 4096, kv: int = 1024, ff: int = 14336) -> dict:
    tree = {"embed": (vocab, d), "unembed": (vocab, d), "final_norm": (d,)}
    for i in range(layers):
        tree[f"l{i:02d}"] = {"q": (d, d), "k": (d, kv), "v": (d, kv), "o": (d, d), "gate": (d, ff),
                             "up": (d, ff), "down": (ff, d), "attn_norm": (d,), "mlp_norm": (d,)}
    return tree


def _map(tree, fn):
    return {k: _map(v, fn) if isinstance(v, dict) else fn(v) for k, v in tree.items()}


def _specs(tree, rf):
    """Matrix leaves to Muon; embed / unembed and norm vectors to AdamW."""
    out = {}
    for k, v in tree.items():
        if isinstance(v, dict):
            out[k] = _specs(v, rf)
        else:
            out[k] = rf.MatrixDimensionNumbers() if (len(v) == 2 and k not in ("embed", "unembed")) else None
    return out


def _time(fn, steps: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


def main() -> None:
    import rollfast_b200 as rf
    from rollfast_b200.tree import tree_leaves

    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--layers", type=int, default=32)
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    shapes = llama_shapes(args.layers)
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)

    def randn(s, scale=1.0):
        t = torch.empty(s, dtype=torch.bfloat16, device=dev)
        return t.normal_(0.0, scale, generator=gen)

    params = _map(shapes, lambda s: randn(s, 0.02))
    grads = _map(shapes, randn)
    specs = _specs(shapes, rf)
    cases = [("default (frobenius)", {}), ("preconditioning=aol", {"preconditioning": "aol"}),
             ("preconditioning=schatten", {"preconditioning": "schatten"}),
             ("preconditioning=spectral", {"preconditioning": "spectral"}), ("adaptive", {"adaptive": True}),
             ("mu_dtype=bfloat16", {"mu_dtype": torch.bfloat16})]
    last = None
    for name, kw in cases:
        tx = rf.muon(learning_rate=0.02, weight_decay=0.01, muon_weight_dimension_numbers=specs, **kw)
        box = {"state": tx.init(params), "upd": None}

        def step():
            box["upd"] = None  # drop the previous updates, as a training loop does
            box["upd"], box["state"] = tx.update(grads, box["state"], params)

        ms = _time(step, args.steps, args.warmup)
        print(json.dumps({"case": name, "ms_per_step": round(ms, 2), "layers": args.layers,
                          "workload": "llama3_8b_muon_step"}), flush=True)
        last = box["upd"]
        del tx, box
        torch.cuda.empty_cache()
    key = torch.tensor([0, 42])
    for name, sto in (("apply_updates nearest", False), ("apply_updates stochastic", True)):
        ms = _time(lambda: rf.apply_updates(params, last, key if sto else None, stochastic=sto), args.steps,
                   args.warmup)
        n = sum(t.numel() for t in tree_leaves(params))
        print(json.dumps({"case": name, "ms": round(ms, 3), "elements": n,
                          "gbps_algorithmic": round(n * 8 / (ms * 1e-3) / 1e9, 1)}), flush=True)


if __name__ == "__main__":
    main()
