"""Parity of the BASELINE configurations at their full sizes, against the
CPU oracle (NumPy float32 restatement of the reference path).

  * config 3 (Llama-3-8B): two ``muon()`` steps on one leaf of each matrix
    shape of the benchmarked tree (4096x4096, 4096x1024, 4096x14336,
    14336x4096) plus an RMSNorm vector routed to AdamW;
  * config 4 (NS sweep): 8192x8192, 4096x16384 and 8192x28672 under the
    polar-express schedule at 5 and 8 iterations, inputs N(0,1) divided by
    their Frobenius norm; plus the float16 operand range at these widths;
  * config 2 (GPT-2 small): all 12 stacked layers, the 50257x768 embedding
    on AdamW, polar express, ten steps with fresh gradients.

Tolerances (relative Frobenius error): Muon updates <= 1e-2 (16-bit NS
operands, float32 accumulation, against the reference's float32 NS), AdamW
updates <= 1e-6, float32 momentum bit-exact.  The oracle runs on the host
cores; these cases take minutes of CPU time.
"""

import math

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

MUON_TOL, ADAM_TOL = 1e-2, 1e-6
F16_MAX = 65504.0


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(autouse=True)
def _f16():
    import rollfast_b200 as rf

    rf.set_ns_precision("f16")
    yield


def dev():
    return torch.device("cuda:0")


def to_dev(x, dtype):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev()).to(dtype)


# ---------------------------------------------------------------------------
# Config 3: the Llama-3-8B leaf shapes.
# ---------------------------------------------------------------------------
def test_config3_llama_leaf_shapes_two_steps_match_oracle():
    import rollfast_b200 as rf

    shapes = {"q": (4096, 4096), "k": (4096, 1024), "gate": (4096, 14336), "down": (14336, 4096),
              "norm": (4096,)}
    rng = np.random.default_rng(83)
    p_np = {k: O.bf16_round((rng.standard_normal(s) * 0.02).astype(np.float32)) for k, s in shapes.items()}
    dts = {k: "bfloat16" for k in shapes}
    kw = dict(learning_rate=0.02, weight_decay=0.01, beta=0.95)
    ora = O.OracleMuon(**kw)
    tx = rf.muon(**kw)
    params = {k: to_dev(v, torch.bfloat16) for k, v in p_np.items()}
    ost, st = ora.init(p_np), tx.init(params)
    for step in range(2):
        gr = np.random.default_rng(900 + step)
        g_np = {k: O.bf16_round(gr.standard_normal(s).astype(np.float32)) for k, s in shapes.items()}
        u_ref, ost = ora.update(g_np, ost, p_np, param_dtypes=dts)
        u, st = tx.update({k: to_dev(v, torch.bfloat16) for k, v in g_np.items()}, st, params)
        torch.cuda.synchronize()
        for k in shapes:
            e = rel(u[k].cpu().numpy(), u_ref[k])
            assert e <= (ADAM_TOL if k == "norm" else MUON_TOL), (step, k, e)
        mu = st.inner_states["muon"].inner_state[0][0].mu
        for k in ("q", "k", "gate", "down"):
            np.testing.assert_array_equal(mu[k].cpu().numpy(), ost["mu"][k])


# ---------------------------------------------------------------------------
# Config 4: the widest Newton-Schulz shapes, polar express at 5 and 8
# iterations.
# ---------------------------------------------------------------------------
CFG4_SHAPES = [(8192, 8192), (4096, 16384), (8192, 28672)]


def _normalized_input(shape, seed):
    """N(0,1) divided by its Frobenius norm, stored in bf16 (the config's
    dtype); both sides see the same bf16 values."""
    x = np.random.default_rng(seed).standard_normal(shape).astype(np.float32)
    return O.bf16_round((x / np.float32(np.linalg.norm(x.astype(np.float64)))).astype(np.float32))


@pytest.mark.parametrize("iters", [5, 8])
@pytest.mark.parametrize("shape", CFG4_SHAPES, ids=lambda s: f"{s[0]}x{s[1]}")
def test_config4_ns_matches_oracle(shape, iters):
    import rollfast_b200 as rf

    x = _normalized_input(shape, seed=shape[0] // 1024 + shape[1] // 1024 + iters)
    coeffs = O.resolve_ns_coeffs("polar_express", iters)
    ref = O.quintic_newton_schulz(x, coeffs, iters)
    out = rf.orthogonalize_via_newton_schulz(to_dev(x, torch.bfloat16), torch.from_numpy(coeffs), iters,
                                             "frobenius", 1e-8, None)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    assert np.all(np.isfinite(got))
    e = rel(got, ref)
    print(f"config 4 {shape} polar_express x{iters}: relative error {e:.3e}")
    assert e <= MUON_TOL, (shape, iters, e)


def _ns_scales(m):
    lg = int(math.floor(math.log2(m)))
    sa = float(2 ** lg)
    return float(2 ** ((lg + 1) // 2)), sa, max(1.0, sa / 8.0)


@pytest.mark.parametrize("shape,schedule,iters", [((8192, 28672), "polar_express", 8),
                                                  ((8192, 28672), "polar_express", 5),
                                                  ((8192, 8192), "standard", 5)])
def test_config4_float16_operands_stay_in_range(shape, schedule, iters):
    """The 16-bit operands are stored pre-scaled by powers of two (sx ~ sqrt(m)
    on X, sa = 2^floor(log2 m) on A = X X^T, sb = sa / 8 on B = bA + cA^2).
    With ||X||_2 <= 1 after the Frobenius normalisation, |A_ij| <= 1 and
    |B_ij| <= max over s in [0, 1] of |b s + c s^2| (8.05 for the first
    polar-express row), so at m = 8192 the stored magnitudes are bounded by
    8192 (A~) and 8.2e3 (B~), an 8x margin to float16's 65504.  This replays
    the iteration in float32 on the GPU with the same scales and checks the
    largest stored magnitude of each operand against a 4x margin."""
    m, n = shape
    g = torch.Generator(device=dev())
    g.manual_seed(m + n + iters)
    x = torch.randn(shape, generator=g, device=dev(), dtype=torch.float32)
    x = x / torch.linalg.norm(x)
    sx, sa, sb = _ns_scales(min(shape))
    coeffs = O.resolve_ns_coeffs(schedule, iters)
    rows = [coeffs] * iters if coeffs.ndim == 1 else list(coeffs)
    peak = {"X": 0.0, "A": 0.0, "B": 0.0}
    for a, b, c in rows:
        peak["X"] = max(peak["X"], float(x.abs().max()) * sx)
        A = x @ x.T
        B = float(b) * A + float(c) * (A @ A)
        peak["A"] = max(peak["A"], float(A.abs().max()) * sa)
        peak["B"] = max(peak["B"], float(B.abs().max()) * sb)
        x = float(a) * x + B @ x
        del A, B
    print(f"largest stored magnitudes {shape} {schedule}x{iters}: {peak}")
    for k, v in peak.items():
        assert math.isfinite(v) and v <= F16_MAX / 4, (k, v)


# ---------------------------------------------------------------------------
# Config 2: GPT-2 small, all 12 stacked layers, ten steps.
# ---------------------------------------------------------------------------
def test_config2_full_gpt2_small_ten_steps():
    import rollfast_b200 as rf

    L = 12
    shapes = {"qkv": (L, 768, 2304), "proj": (L, 768, 768), "fc": (L, 768, 3072), "fc_out": (L, 3072, 768),
              "ln1_g": (L, 768), "ln1_b": (L, 768), "ln2_g": (L, 768), "ln2_b": (L, 768),
              "emb": (50257, 768)}
    stacked = {"qkv", "proj", "fc", "fc_out"}
    specs = {k: (O.MatrixDimensionNumbers(1, 2) if k in stacked else None) for k in shapes}
    specs_rf = {k: (rf.MatrixDimensionNumbers(1, 2) if k in stacked else None) for k in shapes}
    rng = np.random.default_rng(2)
    p_np = {k: O.bf16_round((rng.standard_normal(s) * 0.02).astype(np.float32)) for k, s in shapes.items()}
    dts = {k: "bfloat16" for k in shapes}
    kw = dict(learning_rate=0.02, weight_decay=0.01, ns_coeffs="polar_express", ns_steps=5)
    ora = O.OracleMuon(muon_weight_dimension_numbers=specs, **kw)
    tx = rf.muon(muon_weight_dimension_numbers=specs_rf, **kw)
    params = {k: to_dev(v, torch.bfloat16) for k, v in p_np.items()}
    ost, st = ora.init(p_np), tx.init(params)
    worst = {}
    for step in range(10):
        gr = np.random.default_rng(7000 + step)
        g_np = {k: O.bf16_round(gr.standard_normal(s).astype(np.float32)) for k, s in shapes.items()}
        u_ref, ost = ora.update(g_np, ost, p_np, param_dtypes=dts)
        u, st = tx.update({k: to_dev(v, torch.bfloat16) for k, v in g_np.items()}, st, params)
        torch.cuda.synchronize()
        for k in shapes:
            e = rel(u[k].cpu().numpy(), u_ref[k])
            worst[k] = max(worst.get(k, 0.0), e)
            assert e <= (MUON_TOL if k in stacked else ADAM_TOL), (step, k, e)
    mu = st.inner_states["muon"].inner_state[0][0].mu
    for k in stacked:
        np.testing.assert_array_equal(mu[k].cpu().numpy(), ost["mu"][k])
    print("config 2 worst relative errors over ten steps:", worst)
