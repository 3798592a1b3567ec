"""apply_updates (utils.py:648-708) on the rf_apply_updates kernel against
the oracle: bit-exact in round-to-nearest mode for every parameter dtype, and
bit-exact against the oracle's restatement of the bf16 stochastic rounding
(utils.py:342-371) fed with the same noise stream; unbiasedness and special
values checked directly."""

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

TORCH = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


def _case(n, pdt, udt, seed):
    rng = np.random.default_rng(seed)
    p = rng.standard_normal(n).astype(np.float32)
    u = (rng.standard_normal(n) * 1e-2).astype(np.float32)
    tp = torch.from_numpy(p).cuda().to(TORCH[pdt])
    tu = torch.from_numpy(u).cuda().to(TORCH[udt])
    # the oracle sees the stored values
    return tp, tu, tp.float().cpu().numpy(), tu.float().cpu().numpy()


@pytest.mark.parametrize("pdt", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("udt", ["float32", "bfloat16"])
@pytest.mark.parametrize("n", [1024, 1001, 3 * 8192 + 8])
def test_apply_round_to_nearest_bit_exact(pdt, udt, n):
    import rollfast_b200 as rf

    tp, tu, p, u = _case(n, pdt, udt, n)
    got = rf.apply_updates({"w": tp}, {"w": tu}, stochastic=False)["w"]
    assert got.dtype == tp.dtype
    want = O.apply_updates(p, u, pdt, stochastic=False)
    assert np.array_equal(got.float().cpu().numpy(), want)


@pytest.mark.parametrize("n", [4096, 1001])
def test_apply_stochastic_bf16_matches_oracle_stream(n):
    import rollfast_b200 as rf
    from rollfast_b200.base import _splitmix64, key_seed

    key = torch.tensor([3, 77])
    tp, tu, p, u = _case(n, "bfloat16", "float32", 5)
    tq, tv, q, v = _case(n + 8, "float32", "float32", 6)   # second leaf: not bf16 -> nearest
    out = rf.apply_updates({"a": tp, "b": tq}, {"a": tu, "b": tv}, key=key, stochastic=True)
    seed = key_seed(key)
    want_a = O.apply_updates(p, u, "bfloat16", stochastic=True, seed=_splitmix64(seed + 0))
    assert np.array_equal(out["a"].float().cpu().numpy(), want_a)
    assert np.array_equal(out["b"].cpu().numpy(), O.apply_updates(q, v, "float32"))
    # same key -> same bits; another key -> different bits
    again = rf.apply_updates({"a": tp, "b": tq}, {"a": tu, "b": tv}, key=key, stochastic=True)
    assert torch.equal(again["a"], out["a"])
    other = rf.apply_updates({"a": tp, "b": tq}, {"a": tu, "b": tv}, key=torch.tensor([3, 78]), stochastic=True)
    assert not torch.equal(other["a"], out["a"])


def test_apply_stochastic_is_unbiased_and_keeps_specials():
    import rollfast_b200 as rf

    n = 1 << 20
    p = torch.ones(n, dtype=torch.bfloat16, device="cuda")
    u = torch.full((n,), 1e-3, dtype=torch.float32, device="cuda")
    det = rf.apply_updates({"w": p}, {"w": u}, stochastic=False)["w"]
    assert bool((det == 1.0).all())          # nearest rounding loses the update
    sr = rf.apply_updates({"w": p}, {"w": u}, key=torch.tensor([0, 42]))["w"].float()
    assert set(torch.unique(sr).tolist()) <= {1.0, 1.0078125}
    assert abs(float(sr.mean()) - 1.001) < 5e-5   # E[SR(x)] = x (binomial sd ~7e-6)
    sp = torch.tensor([float("inf"), -float("inf"), float("nan"), 0.0] * 2, dtype=torch.bfloat16, device="cuda")
    z = torch.zeros(8, dtype=torch.float32, device="cuda")
    out = rf.apply_updates({"w": sp}, {"w": z}, key=torch.tensor([1, 2]))["w"].float().cpu()
    assert out[0] == float("inf") and out[1] == -float("inf") and torch.isnan(out[2]) and out[3] == 0.0


def test_reference_pure_bf16_apply_case():
    # test_stochastic_rounding.py:81-99 (adamw entry): bf16 params and grads,
    # stochastic apply keeps bf16.
    import rollfast_b200 as rf

    params = {"w": torch.ones((4, 4), dtype=torch.bfloat16, device="cuda")}
    grads = {"w": torch.ones((4, 4), dtype=torch.bfloat16, device="cuda") * 0.1}
    tx = rf.adamw(learning_rate=1e-3)
    updates, _ = tx.update(grads, tx.init(params), params)
    new = rf.apply_updates(params, updates, torch.tensor([0, 0]), stochastic=True)
    assert new["w"].dtype == torch.bfloat16 and bool(torch.isfinite(new["w"].float()).all())
