"""Weight-decay forms the reference accepts, on the GPU path, against the oracle.

  * a scheduled ``weight_decay`` in ``muon()`` / ``adamw()`` (Optax
    ``add_decayed_weights`` with a schedule, utils.py:105-111): evaluated at
    the transform's step count; a schedule returning a Python float is weakly
    typed (``wd * p`` in the parameter dtype), one returning a NumPy float32
    is strongly typed (the product in float32);
  * ``scale_by_adam``'s in-transform decay (adam.py:185-201, utils.py:79-90)
    with a schedule and element-wise array masks (full-shape and broadcast).

Parameters are N(0, 1) bf16 and the decay is large, so the decay term
dominates the update and its rounding is visible at the tolerances used:
Newton-Schulz in float32 (<= 1e-5), AdamW leaves <= 1e-6.
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


SCHEDULES = {
    "python_float": lambda c: 0.3 + 0.1 * c,                # weakly typed
    "float32_array": lambda c: np.float32(0.3 + 0.1 * c),   # strongly typed
}


def _tree(seed):
    rng = np.random.default_rng(seed)
    shapes = {"w": (64, 128), "b": (32,)}
    return {k: O.bf16_round(rng.standard_normal(s).astype(np.float32)) for k, s in shapes.items()}


@pytest.mark.parametrize("kind", list(SCHEDULES))
def test_muon_scheduled_weight_decay_matches_oracle(kind):
    import rollfast_b200 as rf

    sched = SCHEDULES[kind]
    p_np = _tree(1)
    dts = {k: "bfloat16" for k in p_np}
    params = {k: torch.from_numpy(v).to(dev()).to(torch.bfloat16) for k, v in p_np.items()}
    tx = rf.muon(learning_rate=0.1, weight_decay=sched)
    ora = O.OracleMuon(learning_rate=0.1, weight_decay=sched)
    st, ost = tx.init(params), ora.init(p_np)
    for step in range(3):
        g_np = _tree(100 + step)
        u_ref, ost = ora.update(g_np, ost, p_np, param_dtypes=dts)
        u, st = tx.update({k: torch.from_numpy(v).to(dev()).to(torch.bfloat16) for k, v in g_np.items()},
                          st, params)
        torch.cuda.synchronize()
        assert rel(u["w"].cpu().numpy(), u_ref["w"]) <= 1e-5, (kind, step)
        assert rel(u["b"].cpu().numpy(), u_ref["b"]) <= 1e-6, (kind, step)
    # Both branches' add_decayed_weights states counted the three updates.
    assert int(st.inner_states["muon"].inner_state[0][2].count) == 3
    assert int(st.inner_states["adam"].inner_state[1].count) == 3


def test_weak_and_strong_schedules_differ_in_the_oracle():
    """The two typings give measurably different updates on these inputs, so
    the GPU test above tells them apart."""
    p_np, g_np = _tree(1), _tree(100)
    dts = {k: "bfloat16" for k in p_np}
    outs = {}
    for kind, sched in SCHEDULES.items():
        ora = O.OracleMuon(learning_rate=0.1, weight_decay=sched)
        outs[kind], _ = ora.update(g_np, ora.init(p_np), p_np, param_dtypes=dts)
    for k in ("w", "b"):
        assert rel(outs["python_float"][k], outs["float32_array"][k]) > 1e-4


@pytest.mark.parametrize("kind", list(SCHEDULES))
def test_adamw_scheduled_weight_decay_matches_oracle(kind):
    import rollfast_b200 as rf

    sched = SCHEDULES[kind]
    p = O.bf16_round(np.random.default_rng(3).standard_normal(256).astype(np.float32))
    params = {"v": torch.from_numpy(p).to(dev()).to(torch.bfloat16)}
    tx = rf.adamw(learning_rate=0.05, weight_decay=sched)
    st = tx.init(params)
    mu = nu = np.zeros(256, np.float32)
    for c in range(3):
        g = O.bf16_round(np.random.default_rng(30 + c).standard_normal(256).astype(np.float32))
        u, st = tx.update({"v": torch.from_numpy(g).to(dev()).to(torch.bfloat16)}, st, params)
        ur, mu, nu = O.adam_leaf_update(g, mu, nu, c)
        wd, weak = O.decay_at(sched, c)
        ur = (np.float32(-0.05) * (ur + O.decay_term(p, wd, "bfloat16" if weak else "float32"))).astype(np.float32)
        assert rel(u["v"].cpu().numpy(), ur) <= 1e-6, (kind, c)
    assert int(st[1].count) == 3


@pytest.mark.parametrize("mask_kind", ["full", "broadcast_row", "per_leaf_false"])
@pytest.mark.parametrize("wd", [0.3, SCHEDULES["python_float"]], ids=["constant", "schedule"])
def test_scale_by_adam_elementwise_decay_masks_match_oracle(mask_kind, wd):
    import rollfast_b200 as rf

    rng = np.random.default_rng(5)
    shape = (48, 64)
    p = rng.standard_normal(shape).astype(np.float32)
    if mask_kind == "full":
        m_np = rng.random(shape) < 0.5
    elif mask_kind == "broadcast_row":
        m_np = rng.random((1, shape[1])) < 0.5
    else:
        m_np = False
    mask = {"w": torch.from_numpy(np.asarray(m_np)).to(dev()) if mask_kind != "per_leaf_false" else False}
    params = {"w": torch.from_numpy(p).to(dev())}
    tx = rf.scale_by_adam(weight_decay=wd, weight_decay_mask=mask)
    st = tx.init(params)
    mu = nu = np.zeros(shape, np.float32)
    for c in range(3):
        g = rng.standard_normal(shape).astype(np.float32)
        u, st = tx.update({"w": torch.from_numpy(g).to(dev())}, st, params)
        ur, mu, nu = O.adam_leaf_update(g, mu, nu, c)
        wd_c, _ = O.decay_at(wd, c)
        ur = O.in_transform_decay(ur, p, wd_c, m_np)
        assert rel(u["w"].cpu().numpy(), ur) <= 1e-6, (mask_kind, c)


def test_add_decayed_weights_rejects_array_masks():
    import rollfast_b200 as rf

    params = {"v": torch.ones(8, device=dev())}
    tx = rf.adamw(learning_rate=0.1, weight_decay=0.1,
                  weight_decay_mask={"v": torch.ones(8, dtype=torch.bool, device=dev())})
    with pytest.raises((ValueError, RuntimeError)):
        tx.update({"v": torch.ones(8, device=dev())}, tx.init(params), params)
