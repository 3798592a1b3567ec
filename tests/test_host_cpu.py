"""CPU tests of the host side: the C ABI library loads and exports every
symbol the header declares, argument validation that never reaches a
kernel, the Optax-shaped API surface and state layout, routing / reshape
logic (mirrors tests/test_dimension_numbers.py of the reference), and the
product's host-side coefficient code against the reference's known answers."""

import ctypes
import os
import re

import numpy as np
import pytest
import torch

import rollfast_b200 as rf
from rollfast_b200 import _lib
from rollfast_b200.dimension_numbers import (
    _compute_matrix_reshape,
    _get_dimension_numbers,
    _make_matrix_partition_fns,
    _mask_dimension_numbers,
)
from rollfast_b200.tree import MaskedNode, tree_map

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_library_exports_every_header_symbol():
    header = open(os.path.join(ROOT, "include", "rollfast_b200.h")).read()
    declared = set(re.findall(r"^\s*(?:rf_status|const char\*|int64_t)\s+(rf_\w+)\(", header, re.M))
    assert declared, "no declarations parsed"
    lib = _lib.load()
    for name in declared:
        assert hasattr(lib, name), name
    assert declared == set(_lib.EXPORTED)


def test_version_and_error_strings():
    assert _lib.version() == (0, 1, 0)
    lib = _lib.load()
    st = lib.rf_version(None, None, None)
    assert st == _lib.RF_EINVAL
    assert b"null" in lib.rf_last_error()


def test_workspace_size_validation_without_gpu():
    lib = _lib.load()
    n = ctypes.c_size_t()
    assert lib.rf_newton_schulz_workspace_size(1, 0, 4, _lib.RF_NS_F16, ctypes.byref(n)) == _lib.RF_EINVAL
    assert lib.rf_newton_schulz_workspace_size(1, 4, 4, 9, ctypes.byref(n)) == _lib.RF_EINVAL
    assert lib.rf_newton_schulz_workspace_size(2, 1024, 4096, _lib.RF_NS_F16, ctypes.byref(n)) == _lib.RF_OK
    # partials + denominators + two X buffers + A + B (f16, padded to 256).
    expect_ns = 2 * 2 * 1024 * 4096 * 2 + 2 * 2 * 1024 * 1024 * 2
    assert n.value >= expect_ns
    leaf = _lib.RfMuonLeaf()
    leaf.batch, leaf.rows, leaf.cols = 1, 8, 8
    leaf.grad_dtype = 7
    assert lib.rf_muon_workspace_size(ctypes.byref(leaf), 1, _lib.RF_NS_F16, 0, ctypes.byref(n)) == _lib.RF_EINVAL
    assert b"dtype" in lib.rf_last_error()


def test_muon_update_rejects_bad_params_before_any_launch():
    lib = _lib.load()
    prm = _lib.RfMuonParams()
    prm.beta, prm.eps, prm.ns_steps, prm.n_coeff_rows = 1.5, 1e-8, 5, 1
    assert lib.rf_muon_update(None, 0, ctypes.byref(prm), None, 0, None) == _lib.RF_EINVAL
    prm.beta = 0.9
    prm.coeffs = None
    assert lib.rf_muon_update(None, 0, ctypes.byref(prm), None, 0, None) == _lib.RF_EINVAL
    c = (ctypes.c_float * 3)(3.4445, -4.775, 2.0315)
    prm.coeffs = ctypes.cast(c, ctypes.POINTER(ctypes.c_float))
    prm.n_coeff_rows, prm.ns_steps = 0, 0
    assert lib.rf_muon_update(None, 0, ctypes.byref(prm), None, 0, None) == _lib.RF_EINVAL
    assert b"ns_steps" in lib.rf_last_error()
    prm.n_coeff_rows = -1
    assert lib.rf_muon_update(None, 0, ctypes.byref(prm), None, 0, None) == _lib.RF_EINVAL


# ---------------------------------------------------------------------------
# Coefficient code (product host side) vs the reference's known answers.
# ---------------------------------------------------------------------------


def test_polar_express_known_answer():
    # tests/test_muon.py:308-325
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
    got = rf.polar_express_coeffs(l=1e-3, num_iters=8, safety_factor_eps=0.0, cushion=0.02407327424182761)
    np.testing.assert_allclose(np.asarray(got), np.asarray(expected), rtol=1e-8)


def test_resolve_ns_coeffs_matches_reference_contract():
    # tests/test_orthogonalization.py:16-45
    assert rf.MUON_NS_COEFFS == (3.4445, -4.7750, 2.0315)
    np.testing.assert_allclose(rf.resolve_ns_coeffs("standard", 5).numpy(), (3.4445, -4.7750, 2.0315))
    p = rf.resolve_ns_coeffs("polar_express", 3)
    assert tuple(p.shape) == (3, 3)
    np.testing.assert_allclose(p.numpy(), np.asarray(rf.polar_express_coeffs(num_iters=3), np.float32))
    s = ((1.0, 0.0, 0.0), (2.0, 0.0, 0.0), (3.0, 0.0, 0.0))
    np.testing.assert_allclose(rf.resolve_ns_coeffs(s, 2).numpy(), s[:2])
    with pytest.raises(ValueError, match="Unknown ns_coeff"):
        rf.resolve_ns_coeffs("unknown", 2)
    with pytest.raises(ValueError, match="shape"):
        rf.resolve_ns_coeffs((1.0, 2.0), 2)
    with pytest.raises(ValueError, match="Not enough coeffs"):
        rf.resolve_ns_coeffs(((1.0, 0.0, 0.0),), 2)


def test_product_coefficients_equal_oracle():
    import oracle as O

    for n in (3, 5, 8):
        np.testing.assert_array_equal(rf.resolve_ns_coeffs("polar_express", n).numpy(),
                                      O.resolve_ns_coeffs("polar_express", n))
    np.testing.assert_array_equal(rf.resolve_ns_coeffs("dion", 5).numpy(), O.resolve_ns_coeffs("dion", 5))


# ---------------------------------------------------------------------------
# Validation contracts (tests/test_muon.py:107-135)
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("kwargs", [{"beta": -0.1}, {"beta": 1.0}, {"eps": 0.0}, {"ns_steps": 0}])
def test_scale_by_muon_rejects_invalid_static_parameters(kwargs):
    with pytest.raises(ValueError):
        rf.scale_by_muon(**kwargs)


def test_scale_by_muon_shape_rejects_invalid_consistent_rms():
    with pytest.raises(ValueError, match="consistent_rms"):
        rf.scale_by_muon_shape(consistent_rms=0.0)


def test_scale_by_muon_weight_decay_only_with_magma():
    with pytest.raises(ValueError, match="Magma"):
        rf.scale_by_muon(weight_decay=0.1)


def test_adamw_rejects_negative_weight_decay():
    with pytest.raises(ValueError, match="nonnegative"):
        rf.adamw(learning_rate=0.01, weight_decay=-0.1)


def test_unsupported_options_fail_loudly():
    with pytest.raises(NotImplementedError, match="adaptive"):
        rf.scale_by_muon(use_magma=True, adaptive=True)
    with pytest.raises(NotImplementedError, match="orthogonalize_fn"):
        rf.scale_by_muon(use_magma=True, orthogonalize_fn=lambda x, *a: x)
    with pytest.raises(ValueError, match="magma_p"):
        rf.scale_by_muon(use_magma=True, magma_p=1.5)  # magma.py:8-13
    with pytest.raises(ValueError, match="magma_tau"):
        rf.adamw(learning_rate=0.1, use_magma=True, magma_tau=0.0)
    with pytest.raises(ValueError, match="Unknown preconditioning"):
        rf.scale_by_muon(preconditioning="nuclear")
    with pytest.raises(NotImplementedError, match="adaptive"):
        rf.scale_by_muon(adaptive=True, orthogonalize_fn=lambda x, *a: x)
    with pytest.raises(NotImplementedError, match="mu_dtype"):
        rf.muon(learning_rate=0.1, mu_dtype=torch.float16)  # float32 / bfloat16 state only


def test_scale_by_muon_rejects_fallback_leaves():
    # tests/test_muon.py:126-135 -- validation happens before any kernel.
    params = {"w": torch.ones(2, 2), "b": torch.ones(2)}
    tx = rf.scale_by_muon(ns_steps=2)
    with pytest.raises(ValueError, match=r"scale_by_muon.*matrix dimension specs"):
        tx.update({k: v * 0.1 for k, v in params.items()}, tx.init(params), params)


def test_complex_matrix_leaves_rejected():
    # tests/test_complex_matrix_policy.py:13-32
    params = {"w": torch.eye(2, dtype=torch.complex64)}
    tx = rf.scale_by_muon(ns_steps=2)
    with pytest.raises(ValueError, match="complex"):
        tx.update({"w": torch.ones(2, 2, dtype=torch.complex64)}, tx.init(params), params)


def test_callable_specs_require_params():
    # tests/test_dimension_numbers.py:202-212
    params = {"w": torch.ones(4, 4)}
    tx = rf.scale_by_muon(ns_steps=2, weight_dimension_numbers=lambda m: tree_map(
        lambda _: rf.MatrixDimensionNumbers(), m))
    with pytest.raises(ValueError, match=r"params.*scale_by_muon"):
        tx.update({"w": torch.ones(4, 4)}, tx.init(params))


def test_muon_state_layout_mirrors_optax_partition():
    params = {"w": torch.ones(4, 8), "b": torch.ones(8)}
    tx = rf.muon(learning_rate=0.1, weight_decay=0.01)
    st = tx.init(params)
    assert type(st).__name__ == "PartitionState"
    m = st.inner_states["muon"].inner_state
    (ms, shape_state, wd_state), lr_state = m
    assert isinstance(ms, rf.MuonState)
    assert int(ms.count) == 0 and ms.mu["w"].dtype == torch.float32 and isinstance(ms.mu["b"], MaskedNode)
    np.testing.assert_allclose(ms.ns_coeffs.numpy(), (3.4445, -4.7750, 2.0315))
    a = st.inner_states["adam"].inner_state
    assert isinstance(a[0], rf.ScaleByAdamState) and isinstance(a[0].mu["w"], MaskedNode)
    assert a[0].mu["b"].shape == (8,)
    # Schedules keep a count.
    tx2 = rf.muon(learning_rate=lambda c: 0.1 / (1 + c))
    lr_state2 = tx2.init(params).inner_states["muon"].inner_state[1]
    assert int(lr_state2.count) == 0


def test_cpu_tensors_are_rejected_at_update():
    params = {"w": torch.ones(4, 8)}
    tx = rf.muon(learning_rate=0.1)
    with pytest.raises(ValueError, match="CUDA"):
        tx.update({"w": torch.ones(4, 8)}, tx.init(params), params)


# ---------------------------------------------------------------------------
# Routing / reshape (tests/test_dimension_numbers.py)
# ---------------------------------------------------------------------------


def test_default_routing_and_partition_helpers():
    params = {"matrix": torch.ones(2, 3), "vector": torch.ones(3), "none": None}
    d = _get_dimension_numbers(None, params)
    assert d["matrix"] == rf.MatrixDimensionNumbers() and d["vector"] is None and d["none"] is None
    part = _make_matrix_partition_fns(None, "matrix_opt")
    assert part.labels(params) == {"matrix": "matrix_opt", "vector": "adam", "none": None}
    assert isinstance(part.masked_specs(params)["vector"], MaskedNode)
    assert part.default_mask(params) == {"matrix": True, "vector": False, "none": False}
    masked = _mask_dimension_numbers({"matrix": rf.MatrixDimensionNumbers(), "vector": None})
    assert isinstance(masked["vector"], MaskedNode)


def test_bare_spec_single_leaf_only():
    spec = rf.MatrixDimensionNumbers(reduction_axis=1, output_axis=0)
    x = torch.ones(2, 3)
    assert _get_dimension_numbers(spec, x) == spec
    with pytest.raises(ValueError, match="bare MatrixDimensionNumbers"):
        _get_dimension_numbers(spec, {"w": x})


def test_reshape_round_trip():
    x = torch.arange(2 * 3 * 4 * 5).reshape(2, 3, 4, 5)
    fwd, bwd = _compute_matrix_reshape(x, rf.MatrixDimensionNumbers((1, 2), 3))
    m = fwd(x)
    assert tuple(m.shape) == (2, 12, 5)
    assert torch.equal(bwd(m), x)


@pytest.mark.parametrize("dn,match", [
    (rf.MatrixDimensionNumbers(99, 1), "out of bounds"),
    (rf.MatrixDimensionNumbers(-4, 1), "out of bounds"),
    (rf.MatrixDimensionNumbers((0, -3), 1), "duplicate"),
    (rf.MatrixDimensionNumbers(0, (1, -2)), "duplicate"),
    (rf.MatrixDimensionNumbers(0, -3), "disjoint"),
    (rf.MatrixDimensionNumbers((), 1), "must not be empty"),
    (rf.MatrixDimensionNumbers(0, ()), "must not be empty"),
])
def test_reshape_rejects_invalid_specs(dn, match):
    with pytest.raises(ValueError, match=match):
        _compute_matrix_reshape(torch.ones(2, 3, 4), dn)


def test_shape_factor_known_answers():
    # tests/test_muon.py:85-96 plus the configs' leaves.
    from rollfast_b200.muon import shape_factor

    spec = rf.MatrixDimensionNumbers()
    assert shape_factor((2, 8), spec) == pytest.approx(2.0)
    assert shape_factor((2, 8), spec, 0.2) == pytest.approx(np.sqrt(8.0) * 0.2, rel=1e-6)
    assert shape_factor((4096, 14336), spec) == pytest.approx(np.sqrt(3.5), rel=1e-6)
    assert shape_factor((14336, 4096), spec) == 1.0
    assert shape_factor((12, 768, 2304), rf.MatrixDimensionNumbers(1, 2)) == pytest.approx(np.sqrt(3.0), rel=1e-6)


def test_tree_map_aux_leaf_semantics():
    t = {"a": torch.ones(1), "b": None, "c": MaskedNode(), "d": [torch.zeros(1), (None, torch.ones(2))]}
    out = tree_map(lambda x: x + 1, t)
    assert out["b"] is None and isinstance(out["c"], MaskedNode)
    assert float(out["d"][1][1][0]) == 2.0
    out2 = tree_map(lambda x: "aux" if (x is None or isinstance(x, MaskedNode)) else "leaf", t,
                    is_leaf=lambda x: x is None or isinstance(x, MaskedNode))
    assert out2["b"] == "aux" and out2["c"] == "aux" and out2["a"] == "leaf"


def test_apply_updates_requires_key_when_stochastic():
    # utils.py:674-678
    with pytest.raises(ValueError, match="requires a PRNG `key`"):
        rf.apply_updates({"w": torch.ones(4)}, {"w": torch.ones(4)})


def test_key_seed_layouts():
    from rollfast_b200.base import key_seed

    assert key_seed(torch.tensor([0, 42])) == 42
    assert key_seed([1, 2]) == (1 << 32) | 2
    assert key_seed(7) == 7
    with pytest.raises(ValueError):
        key_seed([1, 2, 3])


def test_state_dtype_and_init_trees():
    from rollfast_b200.base import state_dtype

    assert state_dtype(None) == torch.float32 and state_dtype("bf16") == torch.bfloat16
    params = {"w": torch.zeros(8, 16), "b": torch.zeros(16)}
    st = rf.muon(learning_rate=0.1, mu_dtype=torch.bfloat16).init(params)
    muon_state = st.inner_states["muon"].inner_state[0][0]
    adam_state = st.inner_states["adam"].inner_state[0]
    assert muon_state.mu["w"].dtype == torch.bfloat16          # muon.py:207-223
    assert adam_state.mu["b"].dtype == torch.bfloat16           # adam.py:98-112: both moments
    assert adam_state.nu["b"].dtype == torch.bfloat16
    st32 = rf.muon(learning_rate=0.1).init(params)
    assert st32.inner_states["muon"].inner_state[0][0].mu["w"].dtype == torch.float32


def test_sr_step_seeds_are_deterministic_and_advance_the_key():
    from rollfast_b200.base import sr_step_seeds

    k0 = torch.tensor([0, 42])
    s1, k1 = sr_step_seeds(k0, 5)
    s1b, k1b = sr_step_seeds(k0, 5)
    assert s1 == s1b and torch.equal(k1, k1b)          # same key -> same streams
    assert len(set(s1)) == 5                           # one stream per leaf
    s2, k2 = sr_step_seeds(k1, 5)
    assert not torch.equal(k1, k0) and set(s1).isdisjoint(s2)   # the next step draws new streams
    assert k1.dtype == torch.int64 and k1.shape == (2,) and int(k1.max()) < 2 ** 32


def test_decay_typing_follows_jax_promotion():
    """A Python scalar is weakly typed (product in the parameter dtype); a
    NumPy scalar or array is strongly typed float32."""
    from rollfast_b200.base import decay_at

    import oracle as O

    for fn in (decay_at, O.decay_at):
        assert fn(0.25, 7) == (0.25, True)
        assert fn(lambda c: 0.1 * c, 3)[1] is True
        assert fn(lambda c: np.float32(0.1 * c), 3)[1] is False
        assert fn(lambda c: np.float64(0.5), 0)[1] is False
        assert fn(lambda c: np.array(0.5, np.float32), 0)[1] is False
    assert decay_at(lambda c: 0.1 * c, 3)[0] == pytest.approx(0.3)


def test_scheduled_decay_states_count_from_zero():
    params = {"w": torch.zeros(8, 16), "b": torch.zeros(16)}
    st = rf.muon(learning_rate=0.1, weight_decay=lambda c: 0.01).init(params)
    assert int(st.inner_states["muon"].inner_state[0][2].count) == 0
    assert int(st.inner_states["adam"].inner_state[1].count) == 0
    st_const = rf.muon(learning_rate=0.1, weight_decay=0.01).init(params)
    assert st_const.inner_states["muon"].inner_state[0][2].count is None
    st_adamw = rf.adamw(learning_rate=0.1, weight_decay=lambda c: 0.01, weight_decay_mask={"w": True, "b": False})
    assert int(st_adamw.init(params)[1].inner_state.count) == 0


def test_in_transform_decay_oracle_masks_elementwise():
    import oracle as O

    u = np.array([[1.0, 2.0], [3.0, 4.0]], np.float32)
    p = np.array([[10.0, 20.0], [30.0, 40.0]], np.float32)
    m = np.array([[True, False], [False, True]])
    np.testing.assert_array_equal(O.in_transform_decay(u, p, 0.5, m), [[6.0, 2.0], [3.0, 24.0]])
    np.testing.assert_array_equal(O.in_transform_decay(u, p, 0.5, np.array([[True, False]])),
                                  [[6.0, 2.0], [18.0, 4.0]])  # broadcast row mask
    np.testing.assert_array_equal(O.in_transform_decay(u, p, 0.5, False), u)


def test_magma_state_and_draws():
    """Magma state: a 0.5 float32 score per leaf (utils.py:64-69); the per-leaf
    Bernoulli(p) draws are deterministic in the state key and have mean p."""
    from rollfast_b200.base import magma_keeps

    params = {"w": torch.zeros(8, 16), "b": torch.zeros(16)}
    st = rf.muon(learning_rate=0.1, use_magma=True).init(params)
    ms = st.inner_states["muon"].inner_state[0][0].magma_s
    assert float(ms["w"]) == 0.5 and ms["w"].dtype == torch.float32
    ast = st.inner_states["adam"].inner_state[0].magma_s
    assert float(ast["b"]) == 0.5
    k = torch.tensor([0, 42])
    draws = magma_keeps(k, 20000, 0.3)
    assert draws == magma_keeps(k, 20000, 0.3)
    assert abs(sum(draws) / len(draws) - 0.3) < 0.015
    assert set(magma_keeps(k, 100, 0.0)) == {0} and set(magma_keeps(k, 100, 1.0)) == {1}
