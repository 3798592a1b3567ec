"""bfloat16 optimizer state (mu_dtype=bfloat16; utils.py:342-371, 412-425,
adam.py:219-222) on the GPU against the oracle.

The momentum (and AdamW's two moments) are formed in float32 from the
previous bfloat16 state, the step's direction uses the float32 momentum, and
the stored state is stochastically rounded.  The library's noise is
SplitMix64 (the reference's Threefry bits need JAX), so the oracle is fed the
same stream: stored states must match bit for bit; updates within the usual
tolerances (float32 NS mode 1e-5, AdamW 1e-6).  Each place that stores the
momentum is covered: the operand load, the second load of a preconditioned
step, the adaptive pass, and the custom-hook direction kernel.
"""

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

SHAPES = {"w1": (96, 160), "w2": (160, 96), "stack": (2, 64, 96), "b": (160,)}


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(autouse=True)
def _precision():
    import rollfast_b200 as rf

    rf.set_ns_precision("f32")
    yield
    rf.set_ns_precision("f16")


def _specs(mod):
    return {"w1": mod.MatrixDimensionNumbers(), "w2": mod.MatrixDimensionNumbers(),
            "stack": mod.MatrixDimensionNumbers(1, 2), "b": None}


@pytest.mark.parametrize("pre,adaptive", [("frobenius", False), ("aol", False), ("frobenius", True)])
def test_muon_bf16_state_matches_oracle(pre, adaptive):
    import rollfast_b200 as rf
    from rollfast_b200.base import sr_step_seeds
    from rollfast_b200.tree import tree_flatten

    rng = np.random.default_rng(17)
    params = {k: (rng.standard_normal(s) * 0.02).astype(np.float32) for k, s in SHAPES.items()}
    lr, wd, beta, eps = 0.02, 0.01, 0.95, 1e-8
    tx = rf.muon(learning_rate=lr, weight_decay=wd, mu_dtype=torch.bfloat16, preconditioning=pre,
                 adaptive=adaptive, muon_weight_dimension_numbers=_specs(rf))
    tp = {k: torch.from_numpy(v).cuda() for k, v in params.items()}
    st = tx.init(tp)
    names = [k for k in sorted(SHAPES)]
    flat, _ = tree_flatten({k: k for k in SHAPES})
    order = [k for k in flat if k != "b"]                 # Muon leaves, library order
    mu = {k: np.zeros(SHAPES[k], np.float32) for k in names}
    am = np.zeros(SHAPES["b"], np.float32)
    an = np.zeros(SHAPES["b"], np.float32)
    km = ka = torch.tensor([0, 42])
    coeffs = O.resolve_ns_coeffs("standard", 5)
    specs = _specs(O)
    for step in range(3):
        grads = {k: rng.standard_normal(s).astype(np.float32) for k, s in SHAPES.items()}
        upd, st = tx.update({k: torch.from_numpy(v).cuda() for k, v in grads.items()}, st, tp)
        seeds_m, km = sr_step_seeds(km, len(order))
        seeds_a, ka = sr_step_seeds(ka, 2)
        inner = st.inner_states
        mu_gpu = inner["muon"].inner_state[0][0].mu
        for k, sd in zip(order, seeds_m):
            mu_new, d = O.momentum_runtime(grads[k], mu[k], step, beta, nesterov=True)
            o = O.orthogonalize_via_newton_schulz(d, coeffs, 5, pre, eps, specs[k])
            if adaptive:
                o = (np.sum(d * o, dtype=np.float32) * o).astype(np.float32)
            u = o * O.shape_scale_factor(SHAPES[k], specs[k]) + O.decay_term(params[k], wd, "float32")
            want = (np.float32(-lr) * u).astype(np.float32)
            mu[k] = O.store_state(mu_new, "bfloat16", sd)
            assert np.array_equal(mu_gpu[k].float().cpu().numpy(), mu[k]), (pre, adaptive, step, k)
            assert rel(upd[k].cpu().numpy(), want) <= 1e-5, (pre, adaptive, step, k)
        u, mn, nn = O.adam_leaf_update(grads["b"], am, an, step, nesterov=True, eps=eps)
        want_b = (np.float32(-lr) * (u + O.decay_term(params["b"], wd, "float32"))).astype(np.float32)
        am = O.store_state(mn, "bfloat16", seeds_a[0])
        an = O.store_state(nn, "bfloat16", seeds_a[1])
        adam = inner["adam"].inner_state[0]
        assert adam.mu["b"].dtype == torch.bfloat16
        assert np.array_equal(adam.mu["b"].float().cpu().numpy(), am)
        assert np.array_equal(adam.nu["b"].float().cpu().numpy(), an)
        assert rel(upd["b"].cpu().numpy(), want_b) <= 1e-6


def test_hook_path_bf16_momentum():
    """scale_by_muon with a custom orthogonalize_fn: the direction kernel
    stores the bfloat16 momentum; the hook sees the float32 direction."""
    import rollfast_b200 as rf
    from rollfast_b200.base import sr_step_seeds

    seen = {}

    def hook(x, ns_coeffs, ns_steps, preconditioning, eps, dimension_numbers):
        seen["d"] = x.detach().cpu().numpy().copy()
        return x * 2.0

    rng = np.random.default_rng(23)
    g = rng.standard_normal((64, 80)).astype(np.float32)
    tx = rf.scale_by_muon(mu_dtype="bfloat16", orthogonalize_fn=hook)
    tg = {"w": torch.from_numpy(g).cuda()}
    st = tx.init(tg)
    upd, st2 = tx.update(tg, st)
    mu_new, d = O.momentum_runtime(g, np.zeros_like(g), 0, 0.95, nesterov=True)
    (seed,), _ = sr_step_seeds(torch.tensor([0, 42]), 1)
    np.testing.assert_allclose(seen["d"], d, rtol=1e-6, atol=0)
    assert np.array_equal(st2.mu["w"].float().cpu().numpy(), O.store_state(mu_new, "bfloat16", seed))
    assert not torch.equal(st2.key, st.key)  # bf16 state consumes randomness: the key advances


def test_reference_bf16_momentum_storage_case():
    # test_muon.py:138-148: bf16 momentum state, finite updates.
    import rollfast_b200 as rf

    params = {"w": torch.ones((4, 4), device="cuda")}
    grads = {"w": torch.ones((4, 4), device="cuda") * 0.1}
    tx = rf.scale_by_muon(mu_dtype=torch.bfloat16, ns_steps=2)
    updates, state = tx.update(grads, tx.init(params), params)
    assert state.mu["w"].dtype == torch.bfloat16
    assert bool(torch.isfinite(updates["w"]).all())
