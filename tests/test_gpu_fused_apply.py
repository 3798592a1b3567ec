"""The parameter apply fused into the update: for
``rollfast_b200.muon(...)``, ``update_and_apply`` writes p + u from the
Newton-Schulz final epilogue and the AdamW kernel (the float32 update is never
stored) and must equal ``tx.update`` followed by ``apply_updates``
(utils.py:648-708) bit for bit -- round-to-nearest and bf16 stochastic
rounding with the same key -- on plain, transposed and stacked Muon leaves and
on AdamW leaves, in place or into new buffers."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def dev():
    return torch.device("cuda:0")


def _tree(seed, scale):
    g = torch.Generator(device=dev())
    g.manual_seed(seed)
    shapes = {"wide": (256, 512), "tall": (768, 256), "stack": (3, 128, 384), "vec": (512,), "odd": (1001,)}
    out = {}
    for k, s in shapes.items():
        t = torch.randn(s, device=dev(), generator=g) * scale
        out[k] = t if k == "odd" else t.to(torch.bfloat16)  # one float32 leaf
    return out


def _specs(rf):
    return {"wide": rf.MatrixDimensionNumbers(), "tall": rf.MatrixDimensionNumbers(),
            "stack": rf.MatrixDimensionNumbers(1, 2), "vec": None, "odd": None}


@pytest.mark.parametrize("stochastic", [False, True])
@pytest.mark.parametrize("inplace", [False, True])
def test_update_and_apply_equals_update_then_apply(stochastic, inplace):
    import rollfast_b200 as rf

    params = _tree(1, 0.02)
    kw = dict(learning_rate=0.05, weight_decay=0.01, muon_weight_dimension_numbers=_specs(rf))
    tx_a, tx_b = rf.muon(**kw), rf.muon(**kw)
    st_a, st_b = tx_a.init(params), tx_b.init(params)
    key = torch.tensor([7, 11])
    cur_a = {k: v.clone() for k, v in params.items()}
    cur_b = {k: v.clone() for k, v in params.items()}
    for step in range(3):
        grads = _tree(10 + step, 1.0)
        u, st_a = tx_a.update(grads, st_a, cur_a)
        cur_a = rf.apply_updates(cur_a, u, key if stochastic else None, stochastic=stochastic)
        ptrs = {k: v.data_ptr() for k, v in cur_b.items()}
        cur_b, st_b = rf.update_and_apply(tx_b, grads, st_b, cur_b, key if stochastic else None,
                                          stochastic=stochastic, inplace=inplace)
        torch.cuda.synchronize()
        for k in params:
            assert cur_b[k].dtype == params[k].dtype and cur_b[k].shape == params[k].shape
            assert torch.equal(cur_a[k], cur_b[k]), (k, step)
            if inplace:
                assert cur_b[k].data_ptr() == ptrs[k], k  # written in place
        key = key + 1
    mu_a = st_a.inner_states["muon"].inner_state[0][0].mu
    mu_b = st_b.inner_states["muon"].inner_state[0][0].mu
    for k in ("wide", "tall", "stack"):
        assert torch.equal(mu_a[k], mu_b[k])


def test_update_and_apply_requires_a_key_when_stochastic():
    import rollfast_b200 as rf

    params = _tree(1, 0.02)
    tx = rf.muon(learning_rate=0.05, muon_weight_dimension_numbers=_specs(rf))
    with pytest.raises(ValueError, match="PRNG"):
        rf.update_and_apply(tx, params, tx.init(params), params, None, stochastic=True)
