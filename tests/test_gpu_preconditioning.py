"""GPU parity of the Newton-Schulz preconditioning variants
(orthogonalization.py:153-176, 233-250) through the C ABI, against the
oracle.

The CUDA path computes every variant from the first iteration's A~ of the
Frobenius-normalised operand (rf_precond.cu): aol as per-row operand factors,
schatten as a new per-matrix denominator, spectral from Lanczos on A.
Tolerances (relative Frobenius error): float32 NS mode <= 1e-5; 16-bit
operands <= 1e-2 (A~ itself is then 16-bit, so the scales carry ~1e-3).
"""

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

PRECONDS = ["aol", "schatten", "spectral"]


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(autouse=True)
def _precision():
    import rollfast_b200 as rf

    rf.set_ns_precision("f16")
    yield
    rf.set_ns_precision("f16")


def ns_gpu(x, coeffs, steps, pre, precision):
    import rollfast_b200 as rf

    rf.set_ns_precision(precision)
    out = rf.orthogonalize_via_newton_schulz(
        torch.from_numpy(np.ascontiguousarray(x)).cuda(), torch.from_numpy(np.asarray(coeffs, np.float32)), steps,
        pre, 1e-8, rf.MatrixDimensionNumbers(1, 2) if x.ndim == 3 else None)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("pre", PRECONDS)
@pytest.mark.parametrize("shape", [(192, 320), (320, 192), (3, 128, 256), (17, 40)])
@pytest.mark.parametrize("precision,tol", [("f32", 1e-5), ("f16", 1e-2)])
def test_preconditioning_matches_oracle(pre, shape, precision, tol):
    rng = np.random.default_rng(sum(shape))
    x = (rng.standard_normal(shape) * 0.7).astype(np.float32)
    c = O.resolve_ns_coeffs("standard", 5)
    ref = O.quintic_newton_schulz(x, c, 5, preconditioning=pre)
    got = ns_gpu(x, c, 5, pre, precision)
    assert np.all(np.isfinite(got))
    assert rel(got, ref) <= tol, (pre, shape, precision, rel(got, ref))


@pytest.mark.parametrize("pre", PRECONDS)
def test_preconditioning_with_schedule_rows(pre):
    # (n,3) schedules: the rescaled first iteration uses row 0 (lax.scan
    # index 0, orthogonalization.py:262-269).
    rng = np.random.default_rng(3)
    x = rng.standard_normal((256, 512)).astype(np.float32)
    c = np.asarray(O.polar_express_coeffs(num_iters=5), np.float32)
    ref = O.quintic_newton_schulz(x, c, 5, preconditioning=pre)
    got = ns_gpu(x, c, 5, pre, "f32")
    assert rel(got, ref) <= 1e-5, rel(got, ref)


@pytest.mark.parametrize("pre", PRECONDS)
def test_preconditioning_edge_cases(pre):
    c = O.resolve_ns_coeffs("standard", 5)
    zero = np.zeros((64, 96), np.float32)
    got = ns_gpu(zero, c, 5, pre, "f32")
    assert np.all(got == 0.0)
    # Rank one (Lanczos breaks down after one step) and a scaled identity.
    # On a rank-deficient input float32 rounding leaves ~1e-7 singular values
    # in the null space, and each iteration multiplies small singular values
    # by ~a = 3.4445 (~500x over 5): the reference's own float32 result is
    # ~6e-5 away from float64 there, for every preconditioning.  So the check
    # is against float64, within 3x the float32 oracle's own error.
    rng = np.random.default_rng(9)
    r1 = np.outer(rng.standard_normal(48), rng.standard_normal(80)).astype(np.float32)
    eye = (3.0 * np.eye(40)).astype(np.float32)
    for x in (r1, eye):
        ref64 = O.quintic_newton_schulz(x.astype(np.float64), c, 5, preconditioning=pre, dtype=np.float64)
        own = rel(O.quintic_newton_schulz(x, c, 5, preconditioning=pre), ref64)
        got = ns_gpu(x, c, 5, pre, "f32")
        assert rel(got, ref64) <= max(1e-5, 3 * own), (pre, x.shape, rel(got, ref64), own)


@pytest.mark.parametrize("pre", PRECONDS)
def test_muon_step_with_preconditioning(pre):
    """One full rollfast.muon step (momentum, preconditioned NS, shape scale,
    decay, LR; AdamW leaf) in float32 NS mode against OracleMuon."""
    import rollfast_b200 as rf

    rf.set_ns_precision("f32")
    rng = np.random.default_rng(21)
    shapes = {"w1": (96, 160), "w2": (160, 96), "b": (160,)}
    params = {k: (rng.standard_normal(s) * 0.02).astype(np.float32) for k, s in shapes.items()}
    grads = {k: rng.standard_normal(s).astype(np.float32) for k, s in shapes.items()}
    kw = dict(learning_rate=0.02, weight_decay=0.01, preconditioning=pre)
    ref = O.OracleMuon(**kw)
    st = ref.init(params)
    want, _ = ref.update(grads, st, params)
    tx = rf.muon(**kw)
    tp = {k: torch.from_numpy(v).cuda() for k, v in params.items()}
    tg = {k: torch.from_numpy(v).cuda() for k, v in grads.items()}
    got, _ = tx.update(tg, tx.init(tp), tp)
    for k in shapes:
        assert rel(got[k].cpu().numpy(), want[k]) <= 1e-5, (pre, k, rel(got[k].cpu().numpy(), want[k]))


# ---------------------------------------------------------------------------
# adaptive (muon.py:272-282): O <- <mu_hat, O> O per leaf.
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("pre", ["frobenius", "schatten"])
@pytest.mark.parametrize("precision,tol", [("f32", 1e-5), ("f16", 1e-2)])
def test_muon_step_adaptive(pre, precision, tol):
    import rollfast_b200 as rf

    rf.set_ns_precision(precision)
    rng = np.random.default_rng(31)
    shapes = {"w1": (128, 320), "w2": (320, 128), "stack": (2, 64, 96), "b": (320,)}
    params = {k: (rng.standard_normal(s) * 0.02).astype(np.float32) for k, s in shapes.items()}
    specs = {"w1": O.MatrixDimensionNumbers(), "w2": O.MatrixDimensionNumbers(),
             "stack": O.MatrixDimensionNumbers(1, 2), "b": None}
    kw = dict(learning_rate=0.02, weight_decay=0.01, preconditioning=pre, adaptive=True)
    ref = O.OracleMuon(muon_weight_dimension_numbers=specs, **kw)
    tx = rf.muon(muon_weight_dimension_numbers={k: (None if v is None else rf.MatrixDimensionNumbers(*v))
                                                for k, v in specs.items()}, **kw)
    tp = {k: torch.from_numpy(v).cuda() for k, v in params.items()}
    st_ref, st = ref.init(params), tx.init(tp)
    for step in range(2):
        grads = {k: rng.standard_normal(s).astype(np.float32) for k, s in shapes.items()}
        want, st_ref = ref.update(grads, st_ref, params)
        got, st = tx.update({k: torch.from_numpy(v).cuda() for k, v in grads.items()}, st, tp)
        for k in shapes:
            e = rel(got[k].cpu().numpy(), want[k])
            assert e <= tol, (pre, precision, step, k, e)


def test_scale_by_muon_adaptive_unfused():
    """scale_by_muon alone (no tail): the update is <mu_hat, O> O."""
    import rollfast_b200 as rf

    rf.set_ns_precision("f32")
    rng = np.random.default_rng(41)
    g = rng.standard_normal((96, 200)).astype(np.float32)
    tx = rf.scale_by_muon(adaptive=True)
    tg = {"w": torch.from_numpy(g).cuda()}
    got, _ = tx.update(tg, tx.init(tg))
    mu_new, d = O.momentum_runtime(g, np.zeros_like(g), 0, 0.95, nesterov=True)
    o = O.orthogonalize_via_newton_schulz(d, O.resolve_ns_coeffs("standard", 5), 5, "frobenius", 1e-8, None)
    want = np.sum(d * o, dtype=np.float32) * o
    assert rel(got["w"].cpu().numpy(), want) <= 1e-5
