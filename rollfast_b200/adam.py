"""(N)AdamW fallback (restates src/rollfast/optim/adam.py) on the
``rf_adamw_update`` kernel."""

from __future__ import annotations

import ctypes
from typing import Any, NamedTuple

import torch

from . import _lib, _runtime
from .base import (
    AddDecayedWeightsState,
    GradientTransformation,
    advance_key,
    decay_at,
    init_magma_state,
    magma_keeps,
    validate_magma_args,
    MaskedState,
    ScaleByScheduleState,
    ScaleState,
    has_nonzero_or_scheduled,
    host_count,
    new_count,
    rf_dtype,
    require_cuda,
    resolve_mask,
    resolve_scalar,
    round_to_dtype,
    safe_increment,
    sr_step_seeds,
    state_dtype,
)
from .tree import MaskedNode, is_aux_leaf, tree_flatten, tree_unflatten


class ScaleByAdamState(NamedTuple):
    """adam.py:28-35."""

    count: torch.Tensor
    mu: Any
    nu: Any
    magma_s: Any
    key: Any


def fresh_key(key=None) -> torch.Tensor:
    """utils.py:73-76: the reference keeps a PRNG key in the state
    (PRNGKey(42) = [0, 42] by default); the hot path consumes no randomness."""
    if key is None:
        return torch.tensor([0, 42], dtype=torch.int64)
    return torch.as_tensor(key).clone()


def zeros_like_tree(params, dtype=torch.float32):
    """utils.py:25-43."""
    leaves, treedef = tree_flatten(params, is_leaf=is_aux_leaf)
    return tree_unflatten(
        treedef, [x if is_aux_leaf(x) else torch.zeros(x.shape, dtype=dtype, device=x.device) for x in leaves]
    )


def run_adam(items, *, b1, b2, eps, eps_root, count: int, nesterov: bool, lr: float,
             max_ctas_per_sm: int = 0, seeds=None, magma=None, magma_tau: float = 2.0, apply=None) -> None:
    """items: (g, mu, nu, p_or_None, out, decay, decay_rounding_dtype[, mask]);
    ``mask``: an optional uint8 tensor shaped like g (element-wise decay
    mask); ``seeds``: two noise seeds per item (mu, nu) for bfloat16 state;
    ``magma``: None, or per item (score tensor, keep) for Magma; ``apply``:
    None, or per item (mode, seed) of the fused parameter apply (``out`` then
    receives the new parameter, in the parameter dtype)."""
    if not items:
        return
    lib = _lib.load()
    arr = (_lib.RfAdamLeaf * len(items))()
    if magma is not None:
        for i, (score, keep) in enumerate(magma):
            arr[i].magma_score = score.data_ptr()
            arr[i].magma_keep = int(keep)
    if apply is not None:
        for i, (mode, seed) in enumerate(apply):
            arr[i].apply_mode, arr[i].apply_seed = int(mode), int(seed)
    for i, item in enumerate(items):
        g, mu, nu, p, out, decay, rdt = item[:7]
        mask = item[7] if len(item) > 7 else None
        arr[i].decay_mask = mask.data_ptr() if mask is not None else None
        arr[i].grad = g.data_ptr()
        arr[i].mu = mu.data_ptr()
        arr[i].nu = nu.data_ptr()
        arr[i].param = p.data_ptr() if p is not None else None
        arr[i].out = out.data_ptr()
        arr[i].n = g.numel()
        arr[i].grad_dtype = rf_dtype(g)
        arr[i].param_dtype = rf_dtype(p) if p is not None else _lib.RF_F32
        arr[i].out_dtype = rf_dtype(out)
        arr[i].decay = decay
        arr[i].decay_rounding = rdt
        arr[i].state_dtype = rf_dtype(mu)
        if seeds is not None:
            arr[i].sr_seed_mu, arr[i].sr_seed_nu = seeds[2 * i], seeds[2 * i + 1]
    prm = _lib.RfAdamParams(float(b1), float(b2), float(eps), float(eps_root), int(count), int(bool(nesterov)),
                            float(lr), int(max_ctas_per_sm), float(magma_tau))
    if magma is not None:
        nbytes = ctypes.c_size_t()
        _lib.check(lib.rf_adamw_workspace_size(arr, len(items), ctypes.byref(nbytes)))
        ws = _runtime.workspace(items[0][0].device, nbytes.value)
        prm.workspace, prm.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.check(lib.rf_adamw_update(arr, len(items), prm,
                                   torch.cuda.current_stream(items[0][0].device).cuda_stream))


def _elementwise_mask(m, g: torch.Tensor) -> torch.Tensor:
    """An array mask broadcast to the leaf's shape, as one byte per element."""
    t = torch.as_tensor(m, device=g.device)
    return t.to(torch.bool).expand(g.shape).contiguous().to(torch.uint8)


def _adam_items(updates, state, params, *, decay: float, decay_mask, decay_rounding_param: bool,
                decay_weak: bool = True):
    """Leaf list for run_adam plus the output tree skeleton.

    ``decay_rounding_param``: the decay of optax.add_decayed_weights (per-leaf
    boolean masks; ``weight_decay * p`` in the parameter dtype when
    ``decay_weak``, else float32); otherwise the in-transform decay of
    scale_by_adam (utils.py:79-90: float32 product, array masks applied
    element-wise)."""
    leaves, treedef = tree_flatten(updates, is_leaf=is_aux_leaf)
    mus = tree_flatten(state.mu, is_leaf=is_aux_leaf)[0]
    nus = tree_flatten(state.nu, is_leaf=is_aux_leaf)[0]
    ps = tree_flatten(params, is_leaf=is_aux_leaf)[0] if params is not None else [None] * len(leaves)
    ms = (tree_flatten(decay_mask, is_leaf=is_aux_leaf)[0] if decay_mask is not None else [True] * len(leaves))
    items, outs = [], []
    for g, mu, nu, p, m in zip(leaves, mus, nus, ps, ms):
        if is_aux_leaf(g):
            outs.append(g)
            continue
        require_cuda(g, "gradient")
        if g.dtype.is_complex:
            raise NotImplementedError("complex leaves are not on the B200 hot path")
        elementwise = not isinstance(m, bool) and getattr(m, "ndim", 0) > 0
        if elementwise and decay_rounding_param:
            raise ValueError("The truth value of an array with more than one element is ambiguous: "
                             "add_decayed_weights masks take one boolean per leaf.")
        use = decay != 0.0 and (elementwise or bool(m)) and p is not None and not is_aux_leaf(p)
        out = torch.empty(g.shape, dtype=torch.float32, device=g.device)
        if use:
            weak = decay_rounding_param and decay_weak
            rdt = rf_dtype(p) if weak else _lib.RF_F32
            d = round_to_dtype(decay, p.dtype) if weak else decay
            items.append((g.contiguous(), mu, nu, p.contiguous(), out, d, rdt,
                          _elementwise_mask(m, g) if elementwise else None))
        else:
            items.append((g.contiguous(), mu, nu, None, out, 0.0, _lib.RF_F32))
        outs.append(out)
    return items, outs, treedef


def _magma_items(updates, state, use_magma: bool, p: float, n_items: int):
    """(per item (score, keep), key) for Magma, or (None, key)."""
    if not use_magma:
        return None, state.key
    leaves = tree_flatten(updates, is_leaf=is_aux_leaf)[0]
    scores = tree_flatten(state.magma_s, is_leaf=is_aux_leaf)[0]
    pos = [i for i, g in enumerate(leaves) if not is_aux_leaf(g)]
    keeps = magma_keeps(state.key, n_items, p)
    return [(scores[i], k) for i, k in zip(pos, keeps)], state.key


def wd_count(st) -> int:
    """Step count of an add_decayed_weights state (0 for a constant decay)."""
    inner = st.inner_state if isinstance(st, MaskedState) else st
    return 0 if inner.count is None else host_count(inner.count)


def bump_wd_state(st):
    """The add_decayed_weights state after one update (a scheduled decay's
    count advances; a constant decay's state is empty)."""
    if isinstance(st, MaskedState):
        return MaskedState(bump_wd_state(st.inner_state))
    if isinstance(st, AddDecayedWeightsState) and st.count is not None:
        return AddDecayedWeightsState(safe_increment(st.count))
    return st


def adam_seeds(items, key):
    """(seeds, next key) for the items' bfloat16 moments: two streams per
    leaf (adam.py:219-222 splits its rounding key into one per moment); no
    randomness and an unchanged key for float32 state."""
    if not any(it[1].dtype == torch.bfloat16 for it in items):
        return None, key
    return sr_step_seeds(key, 2 * len(items))


def scale_by_adam(b1=0.9, b2=0.999, eps=1e-8, eps_root=0.0, mu_dtype=None, *, weight_decay=0.0,
                  weight_decay_mask=None, nesterov: bool = False, use_magma: bool = False, magma_p: float = 0.5,
                  magma_tau: float = 2.0, axis_name=None, key=None) -> GradientTransformation:
    """adam.py:38-235: returns the Adam direction
    m_hat / (sqrt(v_hat + eps_root) + eps), plus the in-transform decoupled
    decay when ``params`` are given (adam.py:185-201), then with ``use_magma``
    the Magma factor keep * score per leaf (adam.py:204-215)."""
    if use_magma:
        validate_magma_args(magma_p, magma_tau)
    sdt = state_dtype(mu_dtype)

    def init_fn(params):
        # adam.py:98-112: both moments in mu_dtype (float32 by default).
        return ScaleByAdamState(new_count(0), zeros_like_tree(params, sdt), zeros_like_tree(params, sdt),
                                init_magma_state(params) if use_magma else (), fresh_key(key))

    def update_fn(updates, state, params=None):
        if has_nonzero_or_scheduled(weight_decay) and params is None:
            raise ValueError(
                "`params` must be provided to `scale_by_adam.update` when "
                "`weight_decay` is nonzero or scheduled."
            )
        count = host_count(state.count)
        mask = resolve_mask(weight_decay_mask, params) if params is not None else None
        # adam.py:185-201: the decay at the transform's count (utils.py:93-102).
        wd_step, _ = decay_at(weight_decay, count)
        items, outs, treedef = _adam_items(updates, state, params, decay=wd_step, decay_mask=mask,
                                           decay_rounding_param=False)
        magma, _ = _magma_items(updates, state, use_magma, magma_p, len(items))
        seeds, key_next = adam_seeds(items, state.key)
        if use_magma and key_next is state.key:
            key_next = advance_key(state.key)  # the Magma subkey splits the key (adam.py:128-131)
        run_adam(items, b1=b1, b2=b2, eps=eps, eps_root=eps_root, count=count, nesterov=nesterov, lr=-1.0,
                 seeds=seeds, magma=magma, magma_tau=magma_tau)
        new_state = ScaleByAdamState(safe_increment(state.count), state.mu, state.nu, state.magma_s, key_next)
        return tree_unflatten(treedef, outs), new_state

    return GradientTransformation(init_fn, update_fn)


def adamw(learning_rate, b1=0.9, b2=0.999, eps=1e-8, eps_root=0.0, mu_dtype=None, weight_decay=1e-4,
          weight_decay_mask=None, *, nesterov: bool = False, use_magma: bool = False, magma_p: float = 0.5,
          magma_tau: float = 2.0, axis_name=None, key=None) -> GradientTransformation:
    """adam.py:238-404: chain(scale_by_adam, add_decayed_weights, scale_by_learning_rate),
    executed as one fused kernel per step.  State layout matches the chain:
    (ScaleByAdamState, [AddDecayedWeightsState], ScaleState | ScaleByScheduleState)."""
    decay_on = has_nonzero_or_scheduled(weight_decay)
    if use_magma:
        validate_magma_args(magma_p, magma_tau)
    state_dtype(mu_dtype)  # validates
    scheduled = callable(weight_decay)
    inner = scale_by_adam(b1, b2, eps, eps_root, mu_dtype, nesterov=nesterov, use_magma=use_magma, magma_p=magma_p,
                          magma_tau=magma_tau, key=key)

    def init_fn(params):
        states = [inner.init(params)]
        if decay_on and not use_magma:  # with Magma the decay is inside scale_by_adam (adam.py:385-401)
            wd_state = AddDecayedWeightsState(new_count(0)) if scheduled else AddDecayedWeightsState()
            states.append(MaskedState(wd_state) if weight_decay_mask is not None else wd_state)
        states.append(ScaleByScheduleState(new_count(0)) if callable(learning_rate) else ScaleState())
        return tuple(states)

    def update_fn(updates, state, params=None):
        adam_state = state[0]
        lr_state = state[-1]
        if decay_on and params is None:
            raise ValueError(
                "You are using a transformation that requires the current value of parameters, "
                "but you are not passing `params` when calling `update`."
            )
        lr = resolve_scalar(learning_rate, host_count(lr_state.count)) if callable(learning_rate) else float(
            learning_rate)
        mask = resolve_mask(weight_decay_mask, params) if (decay_on and params is not None) else None
        if use_magma:
            # In-transform decay at the Adam count, float32 product, array masks.
            wd, _ = decay_at(weight_decay, host_count(adam_state.count)) if decay_on else (0.0, True)
            items, outs, treedef = _adam_items(updates, adam_state, params, decay=wd, decay_mask=mask,
                                               decay_rounding_param=False)
        else:
            wd, weak = decay_at(weight_decay, host_count(wd_count(state[1]))) if decay_on else (0.0, True)
            items, outs, treedef = _adam_items(updates, adam_state, params, decay=wd, decay_mask=mask,
                                               decay_rounding_param=True, decay_weak=weak)
        magma, _ = _magma_items(updates, adam_state, use_magma, magma_p, len(items))
        seeds, key_next = adam_seeds(items, adam_state.key)
        if use_magma and key_next is adam_state.key:
            key_next = advance_key(adam_state.key)
        run_adam(items, b1=b1, b2=b2, eps=eps, eps_root=eps_root, count=host_count(adam_state.count),
                 nesterov=nesterov, lr=lr, seeds=seeds, magma=magma, magma_tau=magma_tau)
        new_adam = ScaleByAdamState(safe_increment(adam_state.count), adam_state.mu, adam_state.nu,
                                    adam_state.magma_s, key_next)
        new_lr = ScaleByScheduleState(safe_increment(lr_state.count)) if callable(learning_rate) else lr_state
        rest = [bump_wd_state(s) for s in state[1:-1]]
        return tree_unflatten(treedef, outs), (new_adam, *rest, new_lr)

    return GradientTransformation(init_fn, update_fn)


__all__ = ["ScaleByAdamState", "adamw", "scale_by_adam"]
