"""Regenerate the golden fixtures in this folder from the CPU oracle.

    python tests/golden/make_golden.py

The reference (JAX/Optax) is not installable in this image, so the fixtures
are produced by the oracle (``oracle/``), which is itself pinned to the
reference's known-answer tests (tests/test_oracle_known_answers.py).  All
inputs are seeded; values are stored as float32.
"""

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle as O  # noqa: E402


def ns_fixture():
    rng = np.random.default_rng(1)
    out = {}
    cases = {
        "wide": rng.standard_normal((40, 136)).astype(np.float32),
        "tall": rng.standard_normal((120, 48)).astype(np.float32),
        "batched": rng.standard_normal((3, 24, 56)).astype(np.float32),
    }
    scheds = {
        "standard5": (O.resolve_ns_coeffs("standard", 5), 5),
        "polar5": (O.resolve_ns_coeffs("polar_express", 5), 5),
        "polar8": (O.resolve_ns_coeffs("polar_express", 8), 8),
        "dion5": (O.resolve_ns_coeffs("dion", 5), 5),
    }
    for cn, x in cases.items():
        out[f"x_{cn}"] = x
        for sn, (c, k) in scheds.items():
            out[f"o_{cn}_{sn}"] = O.quintic_newton_schulz(x, c, k, dtype=np.float32)
    for sn, (c, k) in scheds.items():
        out[f"coeffs_{sn}"] = np.asarray(c, np.float32)
    np.savez_compressed(os.path.join(HERE, "ns_small.npz"), **out)


def muon_fixture():
    rng = np.random.default_rng(2)
    w = O.bf16_round(rng.standard_normal((64, 128)).astype(np.float32) * 0.02)
    v = O.bf16_round(rng.standard_normal((128, 32)).astype(np.float32) * 0.02)
    b = rng.standard_normal((128,)).astype(np.float32)
    params = {"w": w, "v": v, "b": b}
    dtypes = {"w": "bfloat16", "v": "bfloat16", "b": "float32"}
    out = {f"p_{k}": a for k, a in params.items()}
    for name, kw in {
        "ema_nesterov": dict(),
        "heavy_ball": dict(momentum_accumulator="heavy_ball", nesterov=False),
        "polar": dict(ns_coeffs="polar_express"),
    }.items():
        tx = O.OracleMuon(learning_rate=0.02, weight_decay=0.01, **kw)
        st = tx.init(params)
        for step in range(3):
            # Gradients are regenerated from these seeds by the tests.
            g = {k: O.bf16_round(np.random.default_rng(100 + step).standard_normal(a.shape).astype(np.float32))
                 for k, a in params.items()}
            g["b"] = np.random.default_rng(200 + step).standard_normal(b.shape).astype(np.float32)
            u, st = tx.update(g, st, params, param_dtypes=dtypes)
            for k in params:
                out[f"{name}_u{step}_{k}"] = u[k]
        out[f"{name}_mu_w"] = st["mu"]["w"]
        out[f"{name}_mu_v"] = st["mu"]["v"]
        out[f"{name}_adam_mu_b"] = st["adam_mu"]["b"]
        out[f"{name}_adam_nu_b"] = st["adam_nu"]["b"]
    np.savez_compressed(os.path.join(HERE, "muon_steps.npz"), **out)


if __name__ == "__main__":
    ns_fixture()
    muon_fixture()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))
