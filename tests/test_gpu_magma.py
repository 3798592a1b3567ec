"""Magma (momentum-aligned gradient masking, src/rollfast/optim/magma.py:16-132)
on the GPU path against the oracle, with the per-leaf Bernoulli draws given.

The reference draws each leaf's keep/drop bit from JAX's Threefry stream,
which cannot be reproduced without JAX; the library draws them from a
SplitMix64 stream of the state key (``base.magma_keeps``, same distribution,
checked in the CPU tests).  Here the oracle receives the library's draws, so
everything else -- the cosine between the raw gradient and the new first
moment, the score EMA, the factor keep * score after the decay, the state --
is compared deterministically: Newton-Schulz in float32 (<= 1e-5), AdamW
leaves and scores <= 1e-6.
"""

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def dev():
    return torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _f32_ns():
    import rollfast_b200 as rf

    rf.set_ns_precision("f32")
    yield
    rf.set_ns_precision("f16")


def test_muon_with_magma_matches_oracle_over_steps():
    """muon(use_magma=True): Muon leaves through scale_by_muon(shape_updates,
    in-transform decay, Magma) + lr; AdamW leaves through scale_by_adam(decay,
    Magma) + lr (muon.py:335-395, adam.py:380-404)."""
    import rollfast_b200 as rf
    from rollfast_b200.base import advance_key, magma_keeps

    shapes = {"a": (96, 256), "b": (256, 64), "c": (128, 128), "v": (256,), "w": (64,)}
    muon_keys, adam_keys = ["a", "b", "c"], ["v", "w"]
    lr, wd, p_keep, tau = 0.05, 0.02, 0.5, 2.0
    rng = np.random.default_rng(31)
    p_np = {k: rng.standard_normal(s).astype(np.float32) for k, s in shapes.items()}
    params = {k: torch.from_numpy(v).to(dev()) for k, v in p_np.items()}
    tx = rf.muon(learning_rate=lr, weight_decay=wd, use_magma=True, magma_p=p_keep, magma_tau=tau)
    st = tx.init(params)
    mu = {k: np.zeros(shapes[k], np.float32) for k in muon_keys}
    am = {k: np.zeros(shapes[k], np.float32) for k in adam_keys}
    an = {k: np.zeros(shapes[k], np.float32) for k in adam_keys}
    score = {k: np.float32(0.5) for k in shapes}
    mkey, akey = torch.tensor([0, 42]), torch.tensor([0, 42])
    coeffs = O.resolve_ns_coeffs("standard", 5)
    seen = set()
    for count in range(5):
        g_np = {k: rng.standard_normal(s).astype(np.float32) for k, s in shapes.items()}
        u, st = tx.update({k: torch.from_numpy(v).to(dev()) for k, v in g_np.items()}, st, params)
        torch.cuda.synchronize()
        mkeep = magma_keeps(mkey, len(muon_keys), p_keep)
        akeep = magma_keeps(akey, len(adam_keys), p_keep)
        mkey, akey = advance_key(mkey), advance_key(akey)
        for k, keep in zip(muon_keys, mkeep):
            mu[k], d = O.momentum_runtime(g_np[k], mu[k], count, 0.95, nesterov=True)
            o = O.quintic_newton_schulz(d, coeffs, 5)
            delta = (o * O.shape_scale_factor(shapes[k], O.MatrixDimensionNumbers())).astype(np.float32)
            delta = O.in_transform_decay(delta, p_np[k], wd)
            delta, score[k] = O.magma_leaf(g_np[k], mu[k], delta, score[k], keep, tau)
            ref = (np.float32(-lr) * delta).astype(np.float32)
            got = u[k].cpu().numpy()
            if keep:
                assert rel(got, ref) <= 1e-5, (k, count)
            else:
                assert np.all(got == 0), (k, count)
            seen.add(keep)
        for k, keep in zip(adam_keys, akeep):
            du, am[k], an[k] = O.adam_leaf_update(g_np[k], am[k], an[k], count, nesterov=True)
            du = O.in_transform_decay(du, p_np[k], wd)
            du, score[k] = O.magma_leaf(g_np[k], am[k], du, score[k], keep, tau)
            ref = (np.float32(-lr) * du).astype(np.float32)
            got = u[k].cpu().numpy()
            assert (rel(got, ref) <= 1e-6) if keep else np.all(got == 0), (k, count)
        ms = st.inner_states["muon"].inner_state[0][0].magma_s
        ams = st.inner_states["adam"].inner_state[0].magma_s
        for k in muon_keys:
            assert abs(float(ms[k]) - float(score[k])) <= 1e-6 * abs(float(score[k])), (k, count)
        for k in adam_keys:
            assert abs(float(ams[k]) - float(score[k])) <= 1e-6 * abs(float(score[k])), (k, count)
    assert seen == {0, 1}  # both branches of the mask were exercised


def test_scale_by_adam_magma_with_elementwise_mask():
    import rollfast_b200 as rf
    from rollfast_b200.base import magma_keeps

    rng = np.random.default_rng(41)
    shape = (40, 48)
    p = rng.standard_normal(shape).astype(np.float32)
    m_np = rng.random(shape) < 0.5
    params = {"x": torch.from_numpy(p).to(dev())}
    tx = rf.scale_by_adam(weight_decay=0.1, weight_decay_mask={"x": torch.from_numpy(m_np).to(dev())},
                          use_magma=True, magma_p=1.0, magma_tau=0.5)
    st = tx.init(params)
    mu = nu = np.zeros(shape, np.float32)
    score = np.float32(0.5)
    for c in range(3):
        g = rng.standard_normal(shape).astype(np.float32)
        u, st = tx.update({"x": torch.from_numpy(g).to(dev())}, st, params)
        du, mu, nu = O.adam_leaf_update(g, mu, nu, c)
        du = O.in_transform_decay(du, p, 0.1, m_np)
        assert magma_keeps(st.key, 1, 1.0) == [1]
        du, score = O.magma_leaf(g, mu, du, score, 1, 0.5)
        assert rel(u["x"].cpu().numpy(), du) <= 1e-6, c
        assert abs(float(st.magma_s["x"]) - float(score)) <= 1e-6


def test_scale_by_muon_magma_standalone_has_no_learning_rate():
    """scale_by_muon(use_magma=True) alone: shape scale, decay and the Magma
    factor, unscaled by any learning rate (muon.py:225-330)."""
    import rollfast_b200 as rf

    rng = np.random.default_rng(43)
    shape = (64, 192)
    p = rng.standard_normal(shape).astype(np.float32)
    params = {"w": torch.from_numpy(p).to(dev())}
    tx = rf.scale_by_muon(use_magma=True, magma_p=1.0, weight_decay=0.05, shape_updates=True,
                          weight_dimension_numbers={"w": rf.MatrixDimensionNumbers()})
    st = tx.init(params)
    g = rng.standard_normal(shape).astype(np.float32)
    u, st = tx.update({"w": torch.from_numpy(g).to(dev())}, st, params)
    mu, d = O.momentum_runtime(g, np.zeros(shape, np.float32), 0, 0.95, nesterov=True)
    o = O.quintic_newton_schulz(d, O.resolve_ns_coeffs("standard", 5), 5)
    delta = (o * O.shape_scale_factor(shape, O.MatrixDimensionNumbers())).astype(np.float32)
    delta = O.in_transform_decay(delta, p, 0.05)
    ref, s = O.magma_leaf(g, mu, delta, np.float32(0.5), 1, 2.0)
    assert rel(u["w"].cpu().numpy(), ref) <= 1e-5
    assert abs(float(st.magma_s["w"]) - float(s)) <= 1e-6
