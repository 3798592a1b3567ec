"""The Newton-Schulz kernels behind the reference's other Muon consumers
(the orthogonalize_fn seam), each exercised with the exact
call it makes, against the oracle:

  * NorMuon (src/rollfast/optim/normuon.py:82-97, called at 165-174) and
    TrasMuon (src/rollfast/optim/trasmuon.py:111-125, called at 160-163):
    ``orthogonalize_via_newton_schulz(matrix, coeffs, ns_steps=..,
    preconditioning=.., eps=float32, dimension_numbers=
    MuonDimensionNumbers(reduction_axis=-2, output_axis=-1))`` on the float32
    (batch, rows, cols) reshape of the direction;
  * muon_hyperball (src/rollfast/optim/hyperball.py:490-574): its matrix
    branch is ``_build_unscaled_muon_branch(..., orthogonalize_fn=
    orthogonalize_via_newton_schulz, weight_decay=0.0)`` (momentum, NS,
    shape scale, no learning rate);
  * soda_muon (src/rollfast/optim/soda.py:333-378): ``muon(...)`` driven by a
    learning-rate schedule (the SODA warmup-stable-decay pair).

The fine-tune builder ``muon_adam_from_plan`` (src/rollfast/finetune/builders.py:900-953)
constructs the same ``muon(...)`` from its MuonConfig; the compiler around
it is outside this library.

Tolerances: 16-bit NS operands <= 1e-2, float32 NS <= 1e-5.
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
def _restore_precision():
    yield
    import rollfast_b200 as rf

    rf.set_ns_precision("f16")


@pytest.mark.parametrize("precision,tol", [("f16", 1e-2), ("f32", 1e-5)])
@pytest.mark.parametrize("consumer,shape,coeffs,steps,precond", [
    ("normuon", (4, 384, 1024), "standard", 5, "frobenius"),
    ("normuon_tall", (3, 640, 256), "standard", 5, "frobenius"),
    ("trasmuon_polar", (2, 512, 768), "polar_express", 5, "frobenius"),
    ("trasmuon_schatten", (2, 256, 512), "standard", 5, "schatten"),
])
def test_batched_negative_axis_seam_matches_oracle(consumer, shape, coeffs, steps, precond, precision, tol):
    import rollfast_b200 as rf

    rf.set_ns_precision(precision)
    rng = np.random.default_rng(abs(hash(consumer)) % 2**32)
    x = rng.standard_normal(shape).astype(np.float32)
    c = O.resolve_ns_coeffs(coeffs, steps)
    dims = rf.MuonDimensionNumbers(reduction_axis=-2, output_axis=-1)
    out = rf.orthogonalize_via_newton_schulz(torch.from_numpy(x).to(dev()), torch.from_numpy(c), ns_steps=steps,
                                             preconditioning=precond, eps=np.float32(1e-8), dimension_numbers=dims)
    torch.cuda.synchronize()
    ref = O.orthogonalize_via_newton_schulz(x, c, steps, precond, 1e-8, O.MatrixDimensionNumbers(-2, -1))
    assert out.shape == x.shape
    assert rel(out.cpu().numpy(), ref) <= tol, (consumer, precision)


def test_hyperball_matrix_branch_matches_oracle():
    """The unscaled Muon branch Hyperball wraps: momentum + NS + shape scale
    (no weight decay, no learning rate), three steps."""
    import rollfast_b200 as rf
    from rollfast_b200.muon import _build_unscaled_muon_branch

    rf.set_ns_precision("f32")
    shapes = {"w": (256, 768), "v": (768, 256)}
    specs = {k: rf.MatrixDimensionNumbers() for k in shapes}
    branch = _build_unscaled_muon_branch(
        ns_coeffs="standard", ns_steps=5, beta=0.95, eps=1e-8, mu_dtype=None, nesterov=True, adaptive=False,
        preconditioning="frobenius", weight_dimension_numbers=specs,
        orthogonalize_fn=rf.orthogonalize_via_newton_schulz, momentum_accumulator="ema", use_magma=False,
        magma_p=0.5, magma_tau=2.0, consistent_rms=None, weight_decay=0.0, weight_decay_mask=None,
        axis_name=None, key=None)
    rng = np.random.default_rng(17)
    p = {k: rng.standard_normal(s).astype(np.float32) for k, s in shapes.items()}
    params = {k: torch.from_numpy(v).to(dev()) for k, v in p.items()}
    st = branch.init(params)
    mu = {k: np.zeros(s, np.float32) for k, s in shapes.items()}
    coeffs = O.resolve_ns_coeffs("standard", 5)
    for count in range(3):
        g = {k: rng.standard_normal(s).astype(np.float32) for k, s in shapes.items()}
        u, st = branch.update({k: torch.from_numpy(v).to(dev()) for k, v in g.items()}, st, params)
        torch.cuda.synchronize()
        for k in shapes:
            mu[k], d = O.momentum_runtime(g[k], mu[k], count, 0.95, nesterov=True)
            o = O.quintic_newton_schulz(d, coeffs, 5)
            ref = (o * O.shape_scale_factor(shapes[k], O.MatrixDimensionNumbers())).astype(np.float32)
            assert rel(u[k].cpu().numpy(), ref) <= 1e-5, (k, count)


def test_soda_muon_schedule_driven_muon_matches_oracle():
    """soda_muon's base optimizer: muon(...) with a warmup-stable-decay
    learning-rate schedule for the Muon and AdamW branches."""
    import rollfast_b200 as rf

    rf.set_ns_precision("f32")

    def wsd(step, peak=0.02, total=6, warm=2, decay=2):
        if step < warm:
            return peak * (step + 1) / warm
        if step >= total - decay:
            return peak * max(0.0, (total - step) / decay)
        return peak

    shapes = {"w": (128, 384), "b": (384,)}
    rng = np.random.default_rng(23)
    p_np = {k: O.bf16_round((rng.standard_normal(s) * 0.02).astype(np.float32)) for k, s in shapes.items()}
    dts = {k: "bfloat16" for k in shapes}
    params = {k: torch.from_numpy(v).to(dev()).to(torch.bfloat16) for k, v in p_np.items()}
    tx = rf.muon(learning_rate=wsd, weight_decay=0.0)
    ora = O.OracleMuon(learning_rate=wsd, weight_decay=0.0)
    st, ost = tx.init(params), ora.init(p_np)
    for step in range(6):
        g_np = {k: O.bf16_round(rng.standard_normal(s).astype(np.float32)) for k, s in shapes.items()}
        u_ref, ost = ora.update(g_np, ost, p_np, param_dtypes=dts)
        u, st = tx.update({k: torch.from_numpy(v).to(dev()).to(torch.bfloat16) for k, v in g_np.items()}, st,
                          params)
        torch.cuda.synchronize()
        assert rel(u["w"].cpu().numpy(), u_ref["w"]) <= 1e-5 or np.all(u_ref["w"] == 0), step
        assert rel(u["b"].cpu().numpy(), u_ref["b"]) <= 1e-6 or np.all(u_ref["b"] == 0), step
