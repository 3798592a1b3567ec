"""Pin the CPU oracle against the reference's own known-answer tests.

The reference (rollfast, JAX/Optax) cannot be installed in this image, so
these restate the exact expectations of its test-suite for the Muon path;
each test names the reference test it mirrors.
"""

import math

import numpy as np
import pytest

import oracle as O


def test_standard_coeffs_constant():
    # tests/test_orthogonalization.py:16-17
    assert O.MUON_NS_COEFFS == (3.4445, -4.7750, 2.0315)


def test_polar_express_coeffs_match_published_values_without_safety():
    # tests/test_muon.py:308-325 (rtol 1e-8)
    expected = [
        (8.28721201814563, -23.595886519098837, 17.300387312530933),
        (4.107059111542203, -2.9478499167379106, 0.5448431082926601),
        (3.9486908534822946, -2.908902115962949, 0.5518191394370137),
        (3.3184196573706015, -2.488488024314874, 0.51004894012372),
        (2.300652019954817, -1.6689039845747493, 0.4188073119525673),
        (1.891301407787398, -1.2679958271945868, 0.37680408948524835),
        (1.8750014808534479, -1.2500016453999487, 0.3750001645474248),
        (1.875, -1.25, 0.375),
    ]
    got = O.polar_express_coeffs(l=1e-3, num_iters=8, safety_factor_eps=0.0,
                                 cushion=0.02407327424182761)
    np.testing.assert_allclose(np.asarray(got), np.asarray(expected), rtol=1e-8)


def test_resolve_ns_coeffs_presets_and_schedules():
    # tests/test_orthogonalization.py:20-34
    np.testing.assert_allclose(O.resolve_ns_coeffs("standard", 5), (3.4445, -4.7750, 2.0315))
    polar = O.resolve_ns_coeffs("polar_express", 3)
    assert polar.shape == (3, 3)
    np.testing.assert_allclose(polar, np.asarray(O.polar_express_coeffs(num_iters=3), np.float32))
    sched = ((1.0, 0.0, 0.0), (2.0, 0.0, 0.0), (3.0, 0.0, 0.0))
    np.testing.assert_allclose(O.resolve_ns_coeffs(sched, 2), ((1.0, 0.0, 0.0), (2.0, 0.0, 0.0)))


def test_resolve_ns_coeffs_errors():
    # tests/test_orthogonalization.py:37-45
    with pytest.raises(ValueError, match="Unknown ns_coeff"):
        O.resolve_ns_coeffs("unknown", 2)
    with pytest.raises(ValueError, match="shape"):
        O.resolve_ns_coeffs((1.0, 2.0), 2)
    with pytest.raises(ValueError, match="Not enough coeffs"):
        O.resolve_ns_coeffs(((1.0, 0.0, 0.0),), 2)


def test_polar_express_schedule_depends_on_num_iters():
    five = np.asarray(O.polar_express_coeffs(num_iters=5))
    eight = np.asarray(O.polar_express_coeffs(num_iters=8))
    assert not np.allclose(five, eight[:5])


def test_isotropic_matrix_has_equal_singular_values():
    # tests/test_muon.py:30-46: beta=0, no Nesterov, 5 steps on eye(4).
    g = np.eye(4, dtype=np.float32)
    mu_new, d = O.momentum_runtime(g, np.zeros_like(g), 0, 0.0, nesterov=False)
    out = O.orthogonalize_via_newton_schulz(d, O.resolve_ns_coeffs("standard", 5), 5)
    s = np.linalg.svd(out, compute_uv=False)
    assert out.shape == (4, 4) and np.all(np.isfinite(out))
    np.testing.assert_allclose(s, s[0], rtol=1e-6, atol=1e-6)


def test_shape_scaling_width_transfer_and_consistent_rms():
    # tests/test_muon.py:85-96
    spec = O.MatrixDimensionNumbers()
    assert O.shape_scale_factor((2, 8), spec) == pytest.approx(2.0)
    assert O.shape_scale_factor((2, 8), spec, 0.2) == pytest.approx(math.sqrt(8.0) * 0.2, rel=1e-6)


def test_ema_nesterov_target_value():
    # tests/test_matrix_runtime.py:132-156: g=2, beta=.5, t=1 -> mu=1, d=8/3.
    g = np.full((2, 2), 2.0, np.float32)
    mu, d = O.momentum_runtime(g, np.zeros_like(g), 0, 0.5, nesterov=True)
    np.testing.assert_allclose(mu, 1.0)
    np.testing.assert_allclose(d, 8.0 / 3.0, rtol=1e-6)


def test_heavy_ball_nesterov_target_value():
    # tests/test_matrix_runtime.py:194-218: heavy ball -> mu=g, d=3.
    g = np.full((2, 2), 2.0, np.float32)
    mu, d = O.momentum_runtime(g, np.zeros_like(g), 0, 0.5, nesterov=True, accumulator="heavy_ball")
    np.testing.assert_allclose(mu, g)
    np.testing.assert_allclose(d, 3.0)


def test_momentum_accumulators_differ_after_two_steps():
    # tests/test_muon.py:283-305
    g = np.full((4, 4), 0.1, np.float32)
    mus = {}
    for acc in ("ema", "heavy_ball"):
        mu = np.zeros_like(g)
        for c in range(2):
            mu, _ = O.momentum_runtime(g, mu, c, 0.5, nesterov=False, accumulator=acc)
        mus[acc] = mu
    assert not np.allclose(mus["ema"], mus["heavy_ball"])


def test_invalid_accumulator_rejected():
    # utils.py:336-339
    with pytest.raises(ValueError, match="momentum_accumulator"):
        O.momentum_runtime(np.ones((2, 2), np.float32), np.zeros((2, 2), np.float32), 0, 0.5,
                           nesterov=False, accumulator="bogus")


def _params():
    # tests/test_muon.py:19-27
    return {"w": (np.arange(1, 17, dtype=np.float32).reshape(4, 4) / 10.0),
            "b": np.ones((4,), np.float32)}


def test_muon_partitions_vectors_to_adamw_and_matrix_updates_negative():
    # tests/test_muon.py:49-61
    params = _params()
    grads = {k: np.full_like(v, 0.1) for k, v in params.items()}
    tx = O.OracleMuon(learning_rate=0.01, ns_steps=2)
    updates, _ = tx.update(grads, tx.init(params), params)
    assert updates["w"].shape == (4, 4) and updates["b"].shape == (4,)
    assert np.all(np.isfinite(updates["w"])) and np.all(np.isfinite(updates["b"]))
    assert np.all(updates["w"] < 0.0)


def test_conv_kernel_dimension_numbers_route_through_transpose():
    # tests/test_muon.py:64-82
    params = {"kernel": np.ones((8, 3, 3, 4), np.float32)}
    grads = {"kernel": np.full_like(params["kernel"], 0.01)}
    specs = {"kernel": O.MatrixDimensionNumbers(reduction_axis=(1, 2, 3), output_axis=0)}
    tx = O.OracleMuon(learning_rate=0.01, ns_steps=2, muon_weight_dimension_numbers=specs)
    updates, _ = tx.update(grads, tx.init(params), params)
    assert updates["kernel"].shape == params["kernel"].shape
    assert np.all(np.isfinite(updates["kernel"]))


def test_fallback_adam_inherits_weight_decay():
    # tests/test_muon.py:249-280
    params = {"w": np.ones((4, 4), np.float32), "b": np.ones((4,), np.float32)}
    grads = {k: np.zeros_like(v) for k, v in params.items()}
    mask = {"w": False, "b": True}
    inherit = O.OracleMuon(learning_rate=1.0, ns_steps=2, beta=0.0, nesterov=False,
                           weight_decay=0.2, weight_decay_mask=mask)
    override = O.OracleMuon(learning_rate=1.0, ns_steps=2, beta=0.0, nesterov=False,
                            weight_decay=0.2, adam_weight_decay=0.0, weight_decay_mask=mask)
    u1, _ = inherit.update(grads, inherit.init(params), params)
    u2, _ = override.update(grads, override.init(params), params)
    np.testing.assert_allclose(u1["b"], -0.2 * params["b"], rtol=1e-6)
    np.testing.assert_allclose(u2["b"], 0.0)


def test_adam_constant_gradient_direction_is_sign():
    # tests/test_adam.py:85-100 (rollfast scale_by_adam == optax.scale_by_adam
    # over 3 steps): with a constant gradient the bias-corrected Adam direction
    # is g / (|g| + eps) at every step.
    # In float64 this holds to rounding; in float32 the reference (and Optax)
    # form 1 - f32(0.999)**t, whose rounding moves the result by ~6.5e-6.
    g = np.array([0.1, -0.2], np.float64)
    for dt, tol in ((np.float64, 1e-12), (np.float32, 1e-5)):
        mu = nu = np.zeros_like(g, dtype=dt)
        for c in range(3):
            u, mu, nu = O.adam_leaf_update(g, mu, nu, c, b1=0.9, b2=0.999, eps=1e-8, dtype=dt)
            np.testing.assert_allclose(u, g / (np.abs(g) + 1e-8), rtol=tol)


def test_adamw_masked_decoupled_weight_decay_matches_optax_formula():
    # tests/test_adam.py:140-170: adamw(lr=.01, wd=.1, mask) == optax.adamw.
    p = {"w": np.array([1.0, -2.0], np.float32), "b": np.array([0.5], np.float32)}
    g = {"w": np.array([0.1, -0.2], np.float32), "b": np.array([0.0], np.float32)}
    mask = {"w": True, "b": False}
    mu = {k: np.zeros_like(v) for k, v in p.items()}
    nu = {k: np.zeros_like(v) for k, v in p.items()}
    for c in range(3):
        for k in p:
            u, mu[k], nu[k] = O.adam_leaf_update(g[k], mu[k], nu[k], c)
            if mask[k]:
                u = u + O.decay_term(p[k], 0.1, "float32")
            upd = -0.01 * u
            expected = -0.01 * (g[k] / (np.abs(g[k]) + 1e-8) + (0.1 * p[k] if mask[k] else 0.0))
            np.testing.assert_allclose(upd, expected, rtol=2e-5, atol=1e-9)
            p[k] = p[k] + upd


def test_dimension_numbers_default_routing_and_partition():
    # tests/test_dimension_numbers.py:38-111
    params = {"matrix": np.ones((2, 3)), "vector": np.ones((3,)), "none": None}
    d = O.get_dimension_numbers(None, params)
    assert d["matrix"] == O.MatrixDimensionNumbers() and d["vector"] is None and d["none"] is None
    _, labels, masked, default_mask = O.make_matrix_partition_fns(None, "matrix_opt")
    assert labels(params) == {"matrix": "matrix_opt", "vector": "adam", "none": None}
    assert isinstance(masked(params)["vector"], O.MaskedNode)
    assert default_mask(params) == {"matrix": True, "vector": False, "none": False}
    _, labels2, _, mask2 = O.make_matrix_partition_fns({"matrix": O.MaskedNode(), "vector": None},
                                                       "matrix_opt")
    p2 = {"matrix": np.ones((2, 3)), "vector": np.ones((3,))}
    assert labels2(p2) == {"matrix": "adam", "vector": "adam"}
    assert mask2(p2) == {"matrix": False, "vector": False}


def test_bare_dimension_numbers_single_leaf_only():
    # tests/test_dimension_numbers.py:52-59
    spec = O.MatrixDimensionNumbers(reduction_axis=1, output_axis=0)
    x = np.ones((2, 3), np.float32)
    assert O.get_dimension_numbers(spec, x) == spec
    with pytest.raises(ValueError, match="bare MatrixDimensionNumbers"):
        O.get_dimension_numbers(spec, {"w": x})


def test_reshape_round_trip_high_rank():
    # tests/test_dimension_numbers.py:113-122
    x = np.arange(2 * 3 * 4 * 5).reshape((2, 3, 4, 5))
    fwd, bwd = O.compute_matrix_reshape(x.shape, O.MatrixDimensionNumbers((1, 2), 3))
    m = fwd(x)
    assert m.shape == (2, 12, 5)
    np.testing.assert_array_equal(bwd(m), x)


@pytest.mark.parametrize("dn,match", [
    (O.MatrixDimensionNumbers(99, 1), "out of bounds"),
    (O.MatrixDimensionNumbers(-4, 1), "out of bounds"),
    (O.MatrixDimensionNumbers((0, -3), 1), "duplicate"),
    (O.MatrixDimensionNumbers(0, (1, -2)), "duplicate"),
    (O.MatrixDimensionNumbers(0, -3), "disjoint"),
    (O.MatrixDimensionNumbers((), 1), "must not be empty"),
    (O.MatrixDimensionNumbers(0, ()), "must not be empty"),
])
def test_reshape_rejects_invalid_specs(dn, match):
    # tests/test_dimension_numbers.py:125-162
    with pytest.raises(ValueError, match=match):
        O.compute_matrix_reshape((2, 3, 4), dn)


def test_fp32_newton_schulz_close_to_fp64_truth():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((64, 256)).astype(np.float32)
    c = O.resolve_ns_coeffs("standard", 5)
    a = O.quintic_newton_schulz(x, c, 5, dtype=np.float32)
    b = O.quintic_newton_schulz(x, c, 5, dtype=np.float64)
    assert np.linalg.norm(a - b) / np.linalg.norm(b) < 1e-5


# ---------------------------------------------------------------------------
# Preconditioning variants (orthogonalization.py:153-176, 233-250).  On a
# scaled identity or a diagonal matrix every iteration acts on each singular
# value as sigma -> a sigma + b sigma^3 + c sigma^5, which gives closed forms.
# ---------------------------------------------------------------------------


def _scalar_ns(sigma, coeffs, steps):
    a, b, c = (float(v) for v in coeffs)
    for _ in range(steps):
        sigma = a * sigma + b * sigma ** 3 + c * sigma ** 5
    return sigma


def test_schatten_scales_first_iterate_by_the_fourth_root():
    # ||(3I)(3I)^T||_F = 9 * sqrt(4) = 18, so X / sqrt(18) = I / sqrt(2).
    c = O.MUON_NS_COEFFS
    out = O.quintic_newton_schulz(3.0 * np.eye(4), c, 3, dtype=np.float64, preconditioning="schatten")
    np.testing.assert_allclose(out, _scalar_ns(1 / np.sqrt(2.0), c, 3) * np.eye(4), rtol=1e-12, atol=1e-14)


def test_aol_maps_a_diagonal_matrix_to_its_signs():
    # A = D^2, row sums d_i^2, s_i = 1/|d_i|: the first iterate is sign(D).
    d = np.array([4.0, -0.5, 2.0, 9.0])
    c = O.MUON_NS_COEFFS
    out = O.quintic_newton_schulz(np.diag(d), c, 2, dtype=np.float64, preconditioning="aol")
    np.testing.assert_allclose(out, _scalar_ns(1.0, c, 2) * np.diag(np.sign(d)), rtol=1e-12, atol=1e-14)


def test_spectral_divides_by_the_largest_singular_value():
    d = np.array([4.0, -0.5, 2.0, 8.0])
    c = O.MUON_NS_COEFFS
    out = O.quintic_newton_schulz(np.diag(d), c, 4, eps=1e-8, dtype=np.float64, preconditioning="spectral")
    want = np.diag([np.sign(v) * _scalar_ns(abs(v) / (8.0 + 1e-8), c, 4) for v in d])
    np.testing.assert_allclose(out, want, rtol=1e-10, atol=1e-14)


def test_reference_schatten_mode_runs_case():
    # test_muon.py:358-368: arange(1..16) 4x4, polar express 2 steps.
    mat = np.arange(1, 17, dtype=np.float32).reshape(4, 4)
    out = O.orthogonalize_via_newton_schulz(mat, np.asarray(O.polar_express_coeffs(num_iters=2)), ns_steps=2,
                                            preconditioning="schatten",
                                            dimension_numbers=O.MatrixDimensionNumbers())
    assert out.shape == mat.shape and np.all(np.isfinite(out))


def test_unknown_preconditioning_is_rejected():
    with pytest.raises(ValueError, match="Unknown preconditioning"):
        O.quintic_newton_schulz(np.eye(3), O.MUON_NS_COEFFS, 1, preconditioning="nuclear")


@pytest.mark.parametrize("shape", [(24, 40), (40, 24), (2, 16, 48)])
def test_aol_and_schatten_equal_rescaled_standard_iterations(shape):
    """The CUDA path's reformulation: the rescaled first iteration equals the
    standard iteration applied to diag(s) X (aol) or s X (schatten), where s
    comes from A = X X^T of the raw matrix."""
    rng = np.random.default_rng(5)
    x = rng.standard_normal(shape) * 3.0
    c = O.MUON_NS_COEFFS
    m = np.swapaxes(x, -1, -2) if shape[-2] > shape[-1] else x
    A = m @ np.swapaxes(m, -1, -2)
    s_row = 1.0 / np.sqrt(np.maximum(np.abs(A).sum(-1), 1e-8))[..., :, None]
    s_mat = 1.0 / np.sqrt(np.maximum(np.sqrt((A * A).sum(axis=(-2, -1), keepdims=True)), 1e-8))
    for pre, scaled in (("aol", m * s_row), ("schatten", m * s_mat)):
        got = O.quintic_newton_schulz(x, c, 4, dtype=np.float64, preconditioning=pre)
        y = scaled
        for _ in range(4):
            B = c[1] * (y @ np.swapaxes(y, -1, -2)) + c[2] * np.linalg.matrix_power(y @ np.swapaxes(y, -1, -2), 2)
            y = c[0] * y + B @ y
        want = np.swapaxes(y, -1, -2) if shape[-2] > shape[-1] else y
        np.testing.assert_allclose(got, want, rtol=1e-10, atol=1e-12)


# ---------------------------------------------------------------------------
# apply_updates / bf16 stochastic rounding (utils.py:342-371, 648-708).
# ---------------------------------------------------------------------------


def test_splitmix64_published_first_outputs():
    # SplitMix64 from state 0: the sequence's first two outputs.
    assert int(O.splitmix64(np.uint64(0))) == 0xE220A8397B1DCDAF
    assert int(O.splitmix64(np.uint64(0x9E3779B97F4A7C15))) == 0x6E789E6AA1B965F4
    n = O.noise16(0, 5)
    assert n.tolist() == [0xCDAF, 0x7B1D, 0xA839, 0xE220, 0x65F4]


def test_stochastic_round_bf16_known_answers():
    f = np.float32
    # exactly representable values never move, whatever the noise
    for x in (1.0, -2.5, 0.0, 2.0 ** 127):
        for nz in (0, 0x7FFF, 0xFFFF):
            assert O.stochastic_round_bf16(np.array([x], f), np.array([nz]))[0] == f(x)
    # halfway between 1 and 1 + 2^-7: rounds up exactly when noise >= 0x8000
    half = np.array([1.0 + 2.0 ** -8], f)
    assert O.stochastic_round_bf16(half, np.array([0x7FFF]))[0] == 1.0
    assert O.stochastic_round_bf16(half, np.array([0x8000]))[0] == f(1.0 + 2.0 ** -7)
    # utils.py:344-346: +-Inf with the largest noise stays +-Inf; NaN stays NaN
    inf = O.stochastic_round_bf16(np.array([np.inf, -np.inf, np.nan], f), np.array([0xFFFF] * 3))
    assert inf[0] == np.inf and inf[1] == -np.inf and np.isnan(inf[2])


def test_apply_updates_deterministic_and_unbiased():
    rng = np.random.default_rng(0)
    p = O.bf16_round(np.ones(200000, np.float32))
    u = np.full(200000, 1e-3, np.float32)  # below half a bf16 ulp at 1.0 (2^-8)
    det = O.apply_updates(p, u, "bfloat16", stochastic=False)
    assert np.all(det == 1.0)  # round-to-nearest loses the update (utils.py:653-656)
    sr = O.apply_updates(p, u, "bfloat16", stochastic=True, seed=int(rng.integers(1 << 62)))
    assert set(np.unique(sr).tolist()) <= {1.0, 1.0078125}
    assert abs(float(sr.mean()) - 1.001) < 2e-5  # E[SR(x)] = x
    x = rng.standard_normal(1000).astype(np.float32)
    assert np.array_equal(O.apply_updates(x, x, "float32"), x + x)
    assert np.array_equal(O.apply_updates(x, x, "float16"), O.f16_round(x + x))


def test_store_state_bf16_is_stochastic_rounding_of_the_float32_state():
    # utils.py:412-425: bfloat16 state is the stochastic cast of the float32
    # moment; float32 state is unchanged.
    x = np.array([1.0 + 2.0 ** -8, -3.0, 2.0 ** -130, np.inf], np.float32)
    assert np.array_equal(O.store_state(x, "float32"), x)
    got = O.store_state(x, "bfloat16", seed=5)
    n = O.noise16(5, 4)
    assert np.array_equal(got, O.stochastic_round_bf16(x, n))
    assert got[1] == -3.0 and got[3] == np.inf
    assert got[0] in (1.0, 1.0078125)
