"""Muon (restates src/rollfast/optim/muon.py) on the B200 kernels.

``muon(...)`` keeps the reference signature and state layout
(``partition({"muon": chain(chain(scale_by_muon, scale_by_shape,
[add_decayed_weights]), scale_by_learning_rate), "adam": adamw(...)})``,
muon.py:398-486).  Its update runs the whole Muon branch as one
``rf_muon_update`` call (momentum, Frobenius normalisation, grouped
Newton-Schulz on tcgen05, shape scale, decay and learning rate fused into
the last GEMM's epilogue) and the fallback leaves as one ``rf_adamw_update``
call.  State buffers are updated in place (the equivalent of JAX buffer
donation); the returned state holds the same tensors.
"""

from __future__ import annotations

import ctypes
import math
from typing import Any, NamedTuple

import torch

from . import _lib, _runtime
from .adam import (
    ScaleByAdamState,
    _elementwise_mask,
    adam_seeds,
    adamw,
    bump_wd_state,
    fresh_key,
    run_adam,
    wd_count,
    zeros_like_tree,
)
from .base import (
    AddDecayedWeightsState,
    EmptyState,
    SIDE_CTAS_PER_SM,
    GradientTransformation,
    MaskedState,
    PartitionState,
    ScaleByScheduleState,
    ScaleState,
    add_decayed_weights,
    advance_key,
    chain,
    decay_at,
    has_nonzero_or_scheduled,
    host_count,
    init_empty_state,
    init_magma_state,
    key_seed,
    magma_keeps,
    new_count,
    partition,
    resolve_mask,
    resolve_scalar,
    rf_dtype,
    require_cuda,
    round_to_dtype,
    run_tail,
    safe_increment,
    scale_by_learning_rate,
    sr_step_seeds,
    state_dtype,
    stream_handle,
    validate_beta,
    validate_magma_args,
    validate_positive,
    _splitmix64,
)
from .base import apply_updates as apply_updates_fn
from .dimension_numbers import (
    MatrixDimensionNumbers,
    MuonDimensionNumbers,
    _compute_matrix_layout,
    _is_dimension_numbers_leaf,
    _make_matrix_partition_fns,
    _normalize_axes,
    _resolve_update_dimension_numbers,
    _validate_matrix_operand,
)
from .orthogonalization import (
    MUON_NS_COEFFS,
    coeff_buffer,
    orthogonalize_via_newton_schulz,
    polar_express_coeffs,
    resolve_ns_coeffs,
)
from .tree import MaskedNode, is_aux_leaf, tree_flatten, tree_unflatten

_DEFAULT_NS_COEFFS = MUON_NS_COEFFS


class MuonState(NamedTuple):
    """muon.py:60-67."""

    count: torch.Tensor
    mu: Any
    ns_coeffs: torch.Tensor
    magma_s: Any
    key: Any


# ---------------------------------------------------------------------------
# Shape factors (muon.py:70-120)
# ---------------------------------------------------------------------------


def _get_shape_products(shape, dim_nums: MatrixDimensionNumbers) -> tuple[int, int]:
    """muon.py:70-76."""
    red, out = _normalize_axes(shape, dim_nums)
    return math.prod(shape[a] for a in red), math.prod(shape[a] for a in out)


def shape_factor(shape, dim_nums, consistent_rms=None) -> float:
    """muon.py:79-100 as a float32 scalar: sqrt(max(1, fan_out/fan_in)) or
    sqrt(max(fan_in, fan_out)) * consistent_rms."""
    fan_in, fan_out = _get_shape_products(tuple(shape), dim_nums)
    if consistent_rms is None:
        v = torch.sqrt(torch.tensor(max(1.0, fan_out / fan_in), dtype=torch.float32))
        return float(v)
    v = torch.sqrt(torch.tensor(float(max(fan_in, fan_out)), dtype=torch.float32)) * torch.tensor(
        float(consistent_rms), dtype=torch.float32)
    return float(v)


# ---------------------------------------------------------------------------
# Leaf gathering
# ---------------------------------------------------------------------------


def _flatten_specs(dim_nums, n: int):
    if isinstance(dim_nums, MatrixDimensionNumbers):
        return [dim_nums]
    specs = tree_flatten(dim_nums, is_leaf=_is_dimension_numbers_leaf)[0]
    if len(specs) != n:
        raise ValueError("weight_dimension_numbers tree does not match the update tree")
    return specs


class _MuonLeaf(NamedTuple):
    pos: int
    g: torch.Tensor       # (batch, R, O) view / copy
    mu: torch.Tensor      # (batch, R, O) view / copy of the state buffer
    mu_state: torch.Tensor
    p: torch.Tensor | None
    out: torch.Tensor     # (batch, R, O)
    layout: Any
    shape: tuple
    spec: MatrixDimensionNumbers
    seed: int = 0         # noise seed of a bfloat16 momentum store


def _as_matrix(t: torch.Tensor, lay) -> torch.Tensor:
    if lay.is_identity:
        return t.contiguous().view(lay.flat_shape)
    return t.permute(lay.perm).contiguous().view(lay.flat_shape)


def _gather_muon_leaves(leaves, mus, ps, specs, transform_name: str, allow_meta: bool = False):
    """Muon leaves in their (batch, R, O) layout.  ``allow_meta``: leaves held
    as meta tensors (shape only, no data: not owned by this rank under
    ``distributed.configure(updates="owned")``) are kept as meta."""
    out = []
    for i, (g, spec) in enumerate(zip(leaves, specs)):
        if is_aux_leaf(g):
            continue
        _validate_matrix_operand(g, spec, transform_name)
        if not (allow_meta and isinstance(g, torch.Tensor) and g.is_meta):
            require_cuda(g, "gradient")
        lay = _compute_matrix_layout(g.shape, g.dtype, spec)
        mu_state = mus[i]
        p = ps[i] if ps is not None else None
        if p is not None and is_aux_leaf(p):
            p = None
        out.append(_MuonLeaf(
            pos=i,
            g=_as_matrix(g, lay),
            mu=mu_state.view(lay.flat_shape) if lay.is_identity else _as_matrix(mu_state, lay),
            mu_state=mu_state,
            p=None if p is None else _as_matrix(p, lay),
            out=torch.empty(lay.flat_shape, dtype=torch.float32, device="meta" if allow_meta else g.device),
            layout=lay,
            shape=tuple(g.shape),
            spec=spec,
        ))
    return out


def _leaf_table(ml: list, scales, decays, decay_f32=None, magma=None, apply=None):
    """``magma``: None, or (scores, keeps) per leaf (device score tensors and
    this step's Bernoulli draws); ``apply``: None, or (mode, seed) per leaf for
    the fused parameter apply (``out`` then holds the new parameter)."""
    arr = (_lib.RfMuonLeaf * max(1, len(ml)))()
    for i, L in enumerate(ml):
        b, r, c = L.layout.flat_shape
        e = arr[i]
        e.grad = L.g.data_ptr()
        e.mu = L.mu.data_ptr()
        needs_p = decays[i] != 0.0 or (apply is not None and apply[i][0])
        e.param = L.p.data_ptr() if (L.p is not None and needs_p) else None
        e.out = L.out.data_ptr()
        e.batch, e.rows, e.cols = b, r, c
        e.grad_dtype = rf_dtype(L.g)
        e.param_dtype = rf_dtype(L.p) if L.p is not None else _lib.RF_F32
        e.out_dtype = rf_dtype(L.out)
        e.shape_scale = scales[i]
        e.decay = decays[i]
        e.skip_ns = 0
        e.mu_dtype = rf_dtype(L.mu)
        e.sr_seed = L.seed
        e.decay_in_f32 = int(bool(decay_f32[i])) if decay_f32 is not None else 0
        if magma is not None:
            e.magma_score = magma[0][i].data_ptr()
            e.magma_keep = int(magma[1][i])
        if apply is not None:
            e.apply_mode, e.apply_seed = int(apply[i][0]), int(apply[i][1])
    return arr


def _seed_leaves(ml: list, key):
    """Per-leaf noise seeds for bfloat16 momentum (utils.py:545-562 splits the
    state key when it rounds stochastically) and the state's next key; float32
    momentum consumes no randomness and keeps the key."""
    if not any(L.mu.dtype == torch.bfloat16 for L in ml):
        return ml, key
    seeds, key_next = sr_step_seeds(key, len(ml))
    return [L._replace(seed=sd) for L, sd in zip(ml, seeds)], key_next


def _muon_params(*, beta, eps, count, nesterov, accumulator, ns_coeffs, ns_steps, lr, fuse_tail, reserve_sms=0,
                 preconditioning: str = "frobenius", adaptive: bool = False, magma_tau: float = 2.0):
    cbuf, rows = coeff_buffer(ns_coeffs)
    prm = _lib.RfMuonParams()
    prm.beta = float(beta)
    prm.eps = float(eps)
    prm.count = int(count)
    prm.nesterov = int(bool(nesterov))
    prm.accumulator = _lib.RF_EMA if accumulator == "ema" else _lib.RF_HEAVY_BALL
    prm.ns_steps = int(ns_steps)
    prm.n_coeff_rows = rows
    prm.coeffs = ctypes.cast(cbuf, ctypes.POINTER(ctypes.c_float))
    prm.precision = _runtime.ns_precision()
    prm.lr = float(lr)
    prm.fuse_tail = int(fuse_tail)
    prm.aux_stream = None
    prm.reserve_sms = int(reserve_sms)
    prm.preconditioning = _lib.PRECONDITIONING_CODES[preconditioning]
    prm.adaptive = int(bool(adaptive))
    prm.magma_tau = float(magma_tau)
    return prm, cbuf


def run_muon_table(arr, n: int, prm, dev: torch.device) -> None:
    """rf_muon_update on a prepared leaf table, with the library's
    preparation pipelined on the device's aux stream when enabled."""
    lib = _lib.load()
    pipe = _runtime.pipelined()
    main = torch.cuda.current_stream(dev)
    prm.aux_stream = _runtime.aux_stream(dev).cuda_stream if pipe else None
    nbytes = ctypes.c_size_t()
    _lib.check(lib.rf_muon_workspace_size(arr, n, prm.precision, int(pipe), ctypes.byref(nbytes)))
    ws = _runtime.workspace(dev, nbytes.value)
    _lib.check(lib.rf_muon_update(arr, n, ctypes.byref(prm), ws.data_ptr(), ws.numel(), main.cuda_stream))


def _run_muon_update(ml, prm, cbuf, scales, decays, decay_f32=None, magma=None, apply=None):
    if not ml:
        return
    run_muon_table(_leaf_table(ml, scales, decays, decay_f32, magma, apply), len(ml), prm, ml[0].g.device)
    del cbuf


def _finish_leaves(ml):
    """Copy permuted momentum back and return outputs in leaf layout."""
    outs = []
    for L in ml:
        if not L.layout.is_identity:
            L.mu_state.copy_(L.mu.view(L.layout.unflat_shape).permute(L.layout.inv_perm))
            outs.append(L.out.view(L.layout.unflat_shape).permute(L.layout.inv_perm).contiguous())
        else:
            outs.append(L.out.view(L.shape))
    return outs


def _validate_accumulator(acc: str) -> None:
    if acc not in ("ema", "heavy_ball"):
        raise ValueError(f"momentum_accumulator must be 'ema' or 'heavy_ball', got {acc!r}.")


# ---------------------------------------------------------------------------
# Transforms
# ---------------------------------------------------------------------------


def scale_by_muon_shape(weight_dimension_numbers=None, consistent_rms=None) -> GradientTransformation:
    """muon.py:123-139."""
    validate_positive("consistent_rms", consistent_rms)

    def update_fn(updates, state, params=None):
        dim_nums = _resolve_update_dimension_numbers(weight_dimension_numbers, params=params, updates=updates,
                                                     transform_name="scale_by_muon_shape")
        leaves, treedef = tree_flatten(updates, is_leaf=is_aux_leaf)
        specs = _flatten_specs(dim_nums, len(leaves))
        items, outs = [], []
        for u, d in zip(leaves, specs):
            if is_aux_leaf(u) or d is None or isinstance(d, MaskedNode):
                outs.append(u)
                continue
            require_cuda(u, "update")
            o = torch.empty_like(u)
            items.append((u.contiguous(), None, o, shape_factor(u.shape, d, consistent_rms), 0.0))
            outs.append(o)
        run_tail(items, -1.0)
        return tree_unflatten(treedef, outs), state

    return GradientTransformation(init_empty_state, update_fn)


scale_by_shape = scale_by_muon_shape
_resolve_ns_coeffs = resolve_ns_coeffs


def _check_supported(*, adaptive, preconditioning, use_magma, mu_dtype, orthogonalize_fn):
    if use_magma and adaptive:
        raise NotImplementedError("use_magma together with adaptive=True is not supported")
    if use_magma and orthogonalize_fn is not orthogonalize_via_newton_schulz:
        raise NotImplementedError("use_magma with a custom orthogonalize_fn is not supported (the Magma factor is "
                                  "applied in the fused Newton-Schulz epilogue)")
    if adaptive and orthogonalize_fn is not orthogonalize_via_newton_schulz:
        raise NotImplementedError("adaptive=True with a custom orthogonalize_fn is not supported "
                                  "(the default Newton-Schulz path computes <mu_hat, O> on the GPU)")
    state_dtype(mu_dtype)  # float32, or bfloat16 with stochastic rounding
    if preconditioning not in ("frobenius", "spectral", "aol", "schatten"):
        raise ValueError(f"Unknown preconditioning {preconditioning!r}.")


def scale_by_muon(ns_coeffs=_DEFAULT_NS_COEFFS, ns_steps=5, beta=0.95, eps=1e-8, mu_dtype=None, *,
                  nesterov: bool = True, adaptive: bool = False, preconditioning: str = "frobenius",
                  weight_dimension_numbers=None, orthogonalize_fn=orthogonalize_via_newton_schulz,
                  momentum_accumulator: str = "ema", use_magma: bool = False, magma_p: float = 0.5,
                  magma_tau: float = 2.0, shape_updates: bool = False, consistent_rms=None,
                  weight_decay=0.0, weight_decay_mask=None, axis_name=None, key=None) -> GradientTransformation:
    """muon.py:163-332: momentum + Nesterov + bias correction, then the
    orthogonalisation hook (default: Newton-Schulz on the GPU)."""
    if isinstance(ns_steps, (int, float)) and ns_steps < 1:
        raise ValueError(f"ns_steps must be >= 1, got {ns_steps!r}.")
    validate_beta("beta", beta)
    validate_positive("eps", eps)
    if shape_updates:
        validate_positive("consistent_rms", consistent_rms)
    if not use_magma and has_nonzero_or_scheduled(weight_decay):
        raise ValueError(
            "`weight_decay` in `scale_by_muon` is only applied by the Magma path. "
            "Use `use_magma=True` or chain `optax.add_decayed_weights` separately."
        )
    _validate_accumulator(momentum_accumulator)
    if use_magma:
        validate_magma_args(magma_p, magma_tau)
    _check_supported(adaptive=adaptive, preconditioning=preconditioning, use_magma=use_magma, mu_dtype=mu_dtype,
                     orthogonalize_fn=orthogonalize_fn)

    def init_fn(params):
        # muon.py:207-223: momentum in mu_dtype (float32 by default), Magma
        # scores of 0.5 per leaf when use_magma.
        return MuonState(new_count(0), zeros_like_tree(params, state_dtype(mu_dtype)),
                         resolve_ns_coeffs(ns_coeffs, ns_steps), init_magma_state(params) if use_magma else (),
                         fresh_key(key))

    def update_fn(updates, state, params=None):
        dim_nums = _resolve_update_dimension_numbers(weight_dimension_numbers, params=params, updates=updates,
                                                     transform_name="scale_by_muon")
        leaves, treedef = tree_flatten(updates, is_leaf=is_aux_leaf)
        specs = _flatten_specs(dim_nums, len(leaves))
        for u, d in zip(leaves, specs):
            _validate_matrix_operand(u, d, "scale_by_muon")
        mus = tree_flatten(state.mu, is_leaf=is_aux_leaf)[0]
        count = host_count(state.count)
        decay_on = use_magma and has_nonzero_or_scheduled(weight_decay)
        if decay_on and params is None:
            raise ValueError(
                "`params` must be provided to `scale_by_muon.update` when `weight_decay` is nonzero or scheduled."
            )
        ps = tree_flatten(params, is_leaf=is_aux_leaf)[0] if decay_on else None
        ml = _gather_muon_leaves(leaves, mus, ps, specs, "scale_by_muon")
        keeps = magma_keeps(state.key, len(ml), magma_p) if use_magma else None
        ml, key_next = _seed_leaves(ml, state.key)
        if use_magma and key_next is state.key:
            key_next = advance_key(state.key)  # utils.py:545-562: the Magma subkey splits the key
        # Shape scaling (shape_updates, muon.py:285-290), in-transform decay
        # (use_magma, 297-304: wd at the state count, float32 product) and the
        # Magma factor (309-322) all run in the fused final epilogue; lr = -1
        # leaves the update unscaled.
        fused = use_magma or shape_updates
        ones, zeros = [1.0] * len(ml), [0.0] * len(ml)
        scales = [shape_factor(L.shape, L.spec, consistent_rms) for L in ml] if shape_updates else ones
        decays, decay_f32 = list(zeros), [False] * len(ml)
        if decay_on:
            wd_step, _ = decay_at(weight_decay, count)
            mask_tree = resolve_mask(weight_decay_mask, params)
            masks = (tree_flatten(mask_tree, is_leaf=is_aux_leaf)[0] if mask_tree is not None
                     else [True] * len(leaves))
            for j, L in enumerate(ml):
                m = masks[L.pos]
                if not isinstance(m, bool) and getattr(m, "ndim", 0) > 0:
                    raise NotImplementedError("element-wise weight-decay masks on Muon leaves with use_magma")
                if bool(m) and L.p is not None:
                    decays[j], decay_f32[j] = float(wd_step), True
        magma = None
        if use_magma:
            scores = tree_flatten(state.magma_s, is_leaf=is_aux_leaf)[0]
            magma = ([scores[L.pos] for L in ml], keeps)
        prm, cbuf = _muon_params(beta=beta, eps=eps, count=count, nesterov=nesterov,
                                 accumulator=momentum_accumulator, ns_coeffs=state.ns_coeffs, ns_steps=ns_steps,
                                 lr=-1.0 if fused else 0.0, fuse_tail=int(fused), preconditioning=preconditioning,
                                 adaptive=adaptive, magma_tau=magma_tau)
        if orthogonalize_fn is orthogonalize_via_newton_schulz:
            _run_muon_update(ml, prm, cbuf, scales if fused else ones, decays, decay_f32, magma)
            outs = _finish_leaves(ml)
        else:
            # Caller-supplied hook: materialise the direction (mu_hat), then
            # call the hook per leaf exactly as muon.py:258-271 does.
            if ml:
                arr = _leaf_table(ml, ones, zeros)
                _lib.check(_lib.load().rf_muon_direction(arr, len(ml), ctypes.byref(prm), stream_handle(ml[0].g)))
            dirs = _finish_leaves(ml)
            outs = [orthogonalize_fn(d, state.ns_coeffs, ns_steps, preconditioning, eps, L.spec)
                    for d, L in zip(dirs, ml)]
            if shape_updates:  # muon.py:285-290 on the hook's output
                scaled = [torch.empty_like(o) for o in outs]
                run_tail([(o.contiguous(), None, s, sc, 0.0) for o, s, sc in zip(outs, scaled, scales)], -1.0)
                outs = scaled
        full = list(leaves)
        for L, o in zip(ml, outs):
            full[L.pos] = o
        new_state = MuonState(safe_increment(state.count), state.mu, state.ns_coeffs, state.magma_s, key_next)
        return tree_unflatten(treedef, full), new_state

    return GradientTransformation(init_fn, update_fn)


def _build_unscaled_muon_branch(*, ns_coeffs, ns_steps, beta, eps, mu_dtype, nesterov, adaptive, preconditioning,
                                weight_dimension_numbers, orthogonalize_fn, momentum_accumulator, use_magma,
                                magma_p, magma_tau, consistent_rms, weight_decay, weight_decay_mask, axis_name,
                                key) -> GradientTransformation:
    """muon.py:335-395."""
    components = [
        scale_by_muon(ns_coeffs=ns_coeffs, ns_steps=ns_steps, beta=beta, eps=eps, mu_dtype=mu_dtype,
                      nesterov=nesterov, adaptive=adaptive, preconditioning=preconditioning,
                      weight_dimension_numbers=weight_dimension_numbers, orthogonalize_fn=orthogonalize_fn,
                      momentum_accumulator=momentum_accumulator, use_magma=use_magma, magma_p=magma_p,
                      magma_tau=magma_tau, shape_updates=use_magma, consistent_rms=consistent_rms,
                      weight_decay=weight_decay if use_magma else 0.0,
                      weight_decay_mask=weight_decay_mask if use_magma else None, axis_name=axis_name, key=key)
    ]
    if not use_magma:
        components.append(scale_by_shape(weight_dimension_numbers=weight_dimension_numbers,
                                         consistent_rms=consistent_rms))
        if has_nonzero_or_scheduled(weight_decay):
            components.append(add_decayed_weights(weight_decay, weight_decay_mask))
    return chain(*components)


def muon(learning_rate, ns_coeffs=_DEFAULT_NS_COEFFS, ns_steps=5, beta=0.95, eps=1e-8, weight_decay=0.0,
         weight_decay_mask=None, mu_dtype=None, *, nesterov: bool = True, adaptive: bool = False,
         preconditioning: str = "frobenius", adam_b1=0.9, adam_b2=0.999, adam_eps=None, adam_eps_root=0.0,
         adam_weight_decay=None, adam_learning_rate=None, muon_weight_dimension_numbers=None,
         consistent_rms=None, orthogonalize_fn=orthogonalize_via_newton_schulz,
         momentum_accumulator: str = "ema", use_magma: bool = False, magma_p: float = 0.5,
         magma_tau: float = 2.0, axis_name=None, key=None) -> GradientTransformation:
    """muon.py:398-486: Muon with automatic Muon/AdamW partitioning."""
    if adam_learning_rate is None:
        adam_learning_rate = learning_rate
    if adam_eps is None:
        adam_eps = eps
    eff_adam_wd = weight_decay if adam_weight_decay is None else adam_weight_decay
    part = _make_matrix_partition_fns(muon_weight_dimension_numbers, "muon")
    branch = _build_unscaled_muon_branch(
        ns_coeffs=ns_coeffs, ns_steps=ns_steps, beta=beta, eps=eps, mu_dtype=mu_dtype, nesterov=nesterov,
        adaptive=adaptive, preconditioning=preconditioning, weight_dimension_numbers=part.masked_specs,
        orthogonalize_fn=orthogonalize_fn, momentum_accumulator=momentum_accumulator, use_magma=use_magma,
        magma_p=magma_p, magma_tau=magma_tau, consistent_rms=consistent_rms, weight_decay=weight_decay,
        weight_decay_mask=weight_decay_mask, axis_name=axis_name, key=key)
    adam_tx = adamw(learning_rate=adam_learning_rate, b1=adam_b1, b2=adam_b2, eps=adam_eps, eps_root=adam_eps_root,
                    weight_decay=eff_adam_wd, weight_decay_mask=weight_decay_mask, mu_dtype=mu_dtype,
                    nesterov=nesterov, use_magma=use_magma, magma_p=magma_p, magma_tau=magma_tau,
                    axis_name=axis_name, key=key)
    composite = partition({"muon": chain(branch, scale_by_learning_rate(learning_rate)), "adam": adam_tx},
                          part.labels)
    if orthogonalize_fn is not orthogonalize_via_newton_schulz:
        return composite  # custom hook: run the chain transform by transform

    muon_wd_on = has_nonzero_or_scheduled(weight_decay)
    adam_wd_on = has_nonzero_or_scheduled(eff_adam_wd)

    def fused_update(updates, state, params=None, *, apply_updates=None):
        """``apply_updates=(key, stochastic, inplace)`` (see ``update_and_apply``):
        return the new parameters instead of the updates."""
        from . import distributed  # late import: optional torch.distributed plumbing

        if params is None:
            # scale_by_muon resolves the callable partition specs from params
            # (dimension_numbers.py:127-132).
            raise ValueError(
                "`params` must be provided to `scale_by_muon` when `weight_dimension_numbers` is callable."
            )
        labels = part.labels(updates)
        specs_tree = part.masked_specs(params)
        leaves, treedef = tree_flatten(updates, is_leaf=is_aux_leaf)
        lab = tree_flatten(labels, is_leaf=lambda x: x is None or isinstance(x, str))[0]
        specs = _flatten_specs(specs_tree, len(leaves))
        ps = tree_flatten(params, is_leaf=is_aux_leaf)[0]
        mask_tree = resolve_mask(weight_decay_mask, params)
        masks = tree_flatten(mask_tree, is_leaf=is_aux_leaf)[0] if mask_tree is not None else [True] * len(leaves)

        mstate = state.inner_states["muon"].inner_state  # ((MuonState, Empty, [wd]), lr_state)
        astate = state.inner_states["adam"].inner_state  # (ScaleByAdamState, [wd], lr_state)
        muon_st: MuonState = mstate[0][0]
        mlr_state = mstate[1]
        adam_st: ScaleByAdamState = astate[0]
        alr_state = astate[-1]
        lr = resolve_scalar(learning_rate, host_count(mlr_state.count)) if callable(learning_rate) else float(
            learning_rate)
        alr = resolve_scalar(adam_learning_rate, host_count(alr_state.count)) if callable(
            adam_learning_rate) else float(adam_learning_rate)

        mus = tree_flatten(muon_st.mu, is_leaf=is_aux_leaf)[0]
        muon_leaves = [g if (not is_aux_leaf(g) and l == "muon") else None for g, l in zip(leaves, lab)]
        muon_specs = [s if l == "muon" else None for s, l in zip(specs, lab)]
        for g, s in zip(muon_leaves, muon_specs):
            if g is not None:
                _validate_matrix_operand(g, s, "scale_by_muon")
        ctx = distributed.current()
        sharded = ctx is not None and ctx.world_size > 1
        owned_only = sharded and ctx.updates == "owned"
        if use_magma and sharded:
            raise NotImplementedError("use_magma with the sharded multi-GPU update is not supported")
        ml = _gather_muon_leaves(muon_leaves, mus, ps, muon_specs, "scale_by_muon", allow_meta=owned_only)
        mkeeps = magma_keeps(muon_st.key, len(ml), magma_p) if use_magma else None
        ml, muon_key_next = _seed_leaves(ml, muon_st.key)
        if use_magma and muon_key_next is muon_st.key:
            muon_key_next = advance_key(muon_st.key)
        scales = [shape_factor(L.shape, L.spec, consistent_rms) for L in ml]
        if use_magma:
            # Decay inside scale_by_muon / scale_by_adam (muon.py:297-304,
            # adam.py:185-201): at each branch's state count, float32 product.
            mwd, mweak = (decay_at(weight_decay, host_count(muon_st.count))[0], False) if muon_wd_on else (0.0, True)
            awd, aweak = (decay_at(eff_adam_wd, host_count(adam_st.count))[0], False) if adam_wd_on else (0.0, True)
        else:
            # add_decayed_weights of each branch: a constant, or a schedule at
            # the transform's own count (its state is mstate[0][2] / astate[1]).
            mwd, mweak = decay_at(weight_decay, wd_count(mstate[0][2])) if muon_wd_on else (0.0, True)
            awd, aweak = decay_at(eff_adam_wd, wd_count(astate[1])) if adam_wd_on else (0.0, True)
        decays, decay_f32 = [], []
        for L in ml:
            m = masks[L.pos]
            if use_magma and not isinstance(m, bool) and getattr(m, "ndim", 0) > 0:
                raise NotImplementedError("element-wise weight-decay masks on Muon leaves with use_magma")
            on = muon_wd_on and bool(m) and L.p is not None
            decays.append((round_to_dtype(mwd, L.p.dtype) if mweak else mwd) if on else 0.0)
            decay_f32.append(on and not mweak)
        mmagma = None
        if use_magma:
            mscores = tree_flatten(muon_st.magma_s, is_leaf=is_aux_leaf)[0]
            mmagma = ([mscores[L.pos] for L in ml], mkeeps)
        # AdamW fallback leaves (their `out` is allocated below unless the
        # sharded owner-side path writes them into its update arena).
        a_items, a_pos = [], []
        amus = tree_flatten(adam_st.mu, is_leaf=is_aux_leaf)[0]
        anus = tree_flatten(adam_st.nu, is_leaf=is_aux_leaf)[0]
        for i, (g, l) in enumerate(zip(leaves, lab)):
            if is_aux_leaf(g) or l != "adam":
                continue
            if not (owned_only and g.is_meta):
                require_cuda(g, "gradient")
            if g.dtype.is_complex:
                raise NotImplementedError("complex leaves are not on the B200 hot path")
            p = ps[i]
            m = masks[i]
            elementwise = use_magma and not isinstance(m, bool) and getattr(m, "ndim", 0) > 0
            on = adam_wd_on and (elementwise or bool(m)) and p is not None and not is_aux_leaf(p)
            if on:
                a_items.append((g.contiguous(), amus[i], anus[i], p.contiguous(), None,
                                round_to_dtype(awd, p.dtype) if aweak else awd,
                                rf_dtype(p) if aweak else _lib.RF_F32,
                                _elementwise_mask(m, g) if elementwise else None))
            else:
                a_items.append((g.contiguous(), amus[i], anus[i], None, None, 0.0, _lib.RF_F32))
            a_pos.append(i)
        akeeps = magma_keeps(adam_st.key, len(a_items), magma_p) if use_magma else None
        a_seeds, adam_key_next = adam_seeds(a_items, adam_st.key)
        if use_magma and adam_key_next is adam_st.key:
            adam_key_next = advance_key(adam_st.key)
        adam_kw = dict(b1=adam_b1, b2=adam_b2, eps=adam_eps, eps_root=adam_eps_root,
                       count=host_count(adam_st.count), nesterov=nesterov, lr=alr)
        if use_magma:
            ascores = tree_flatten(adam_st.magma_s, is_leaf=is_aux_leaf)[0]
            adam_kw.update(magma=[(ascores[i], k) for i, k in zip(a_pos, akeeps)], magma_tau=magma_tau)

        prm, cbuf = _muon_params(beta=beta, eps=eps, count=host_count(muon_st.count), nesterov=nesterov,
                                 accumulator=momentum_accumulator, ns_coeffs=muon_st.ns_coeffs,
                                 ns_steps=ns_steps, lr=lr, fuse_tail=1,
                                 reserve_sms=ctx.reserve_sms if sharded else 0,
                                 preconditioning=preconditioning, adaptive=adaptive, magma_tau=magma_tau)
        fused_apply = apply_updates is not None and not sharded
        m_apply = a_apply = None
        if fused_apply:
            # The final epilogues write p + u straight into the new parameters
            # (utils.py:648-708): the float32 updates never reach memory.  The
            # noise seeds are apply_updates' (one stream per leaf position).
            akey, stoch, inplace = apply_updates
            seed0 = key_seed(akey) if stoch else 0

            def mode_seed(pos, p):
                return (2 if (stoch and p.dtype == torch.bfloat16) else 1), (_splitmix64(seed0 + pos) if stoch else 0)

            for L in ml:
                if L.p is None:
                    raise ValueError(f"leaf {L.pos}: apply_updates needs its parameter")
            m_apply = [mode_seed(L.pos, L.p) for L in ml]
            ml = [L._replace(out=L.p if (inplace and L.layout.is_identity) else
                             torch.empty(L.layout.flat_shape, dtype=L.p.dtype, device=L.g.device)) for L in ml]
            a_apply = [mode_seed(pos, ps[pos]) for pos in a_pos]
        res = None
        if owned_only:
            res = distributed.owned_update(ctx, ml, prm, cbuf, scales, decays, decay_f32, a_items, adam_kw, a_seeds,
                                           a_pos)
        elif sharded and ctx.owner_tail and ctx.transport in ("ce", "auto") and not adaptive and (ml or a_items):
            res = distributed.sharded_update(ctx, ml, prm, cbuf, scales, decays, lr, decay_f32, a_items, adam_kw,
                                             a_seeds, a_pos)
            if res is None:
                ctx.owner_tail = False  # peers cannot be mapped (same answer on every rank)
        if res is not None:
            outs, a_outs = res
        else:
            if sharded:
                outs = distributed.sharded_muon_update(ctx, ml, prm, cbuf, scales, decays, lr, decay_f32)
            else:
                _run_muon_update(ml, prm, cbuf, scales, decays, decay_f32, mmagma, m_apply)
                outs = _finish_leaves(ml)
            if fused_apply:
                a_outs = [ps[pos] if (apply_updates[2] and ps[pos].is_contiguous()) else
                          torch.empty(ps[pos].shape, dtype=ps[pos].dtype, device=ps[pos].device) for pos in a_pos]
                a_items = [(it[0], it[1], it[2], ps[pos].contiguous(), *it[4:]) for it, pos in zip(a_items, a_pos)]
                adam_kw["apply"] = a_apply
            else:
                a_outs = [torch.empty(it[0].shape, dtype=torch.float32, device=it[0].device) for it in a_items]
            a_items = [(*it[:4], o, *it[5:]) for it, o in zip(a_items, a_outs)]
            if a_items:
                # The fallback leaves are independent of the Muon branch: with
                # pipelining they run on the aux stream, beside the last GEMMs.
                dev = a_items[0][0].device
                main = torch.cuda.current_stream(dev)
                side = _runtime.aux_stream(dev) if _runtime.pipelined() else main
                if side is not main:
                    side.wait_stream(main)
                with torch.cuda.stream(side):
                    run_adam(a_items, max_ctas_per_sm=SIDE_CTAS_PER_SM if side is not main else 0, seeds=a_seeds,
                             **adam_kw)
                if side is not main:
                    main.wait_stream(side)
                    for it in a_items:
                        for t in it[:5]:
                            if t is not None:
                                t.record_stream(side)

        if apply_updates is not None and not fused_apply:
            # Sharded paths: the updates, then apply_updates as its own pass.
            full_u = list(leaves)
            for L, o in zip(ml, outs):
                full_u[L.pos] = o
            for i2, o in zip(a_pos, a_outs):
                full_u[i2] = o
            outs = [None] * len(ml)
            applied = apply_updates_fn(tree_unflatten(treedef, ps), tree_unflatten(treedef, full_u), apply_updates[0],
                                       stochastic=apply_updates[1])
            ps_new = tree_flatten(applied, is_leaf=is_aux_leaf)[0]
            outs = [ps_new[L.pos] for L in ml]
            a_outs = [ps_new[i2] for i2 in a_pos]
        full = list(ps) if apply_updates is not None else list(leaves)
        for L, o in zip(ml, outs):
            full[L.pos] = o
        for i, o in zip(a_pos, a_outs):
            full[i] = o

        new_muon = MuonState(safe_increment(muon_st.count), muon_st.mu, muon_st.ns_coeffs, muon_st.magma_s,
                             muon_key_next)
        new_mlr = ScaleByScheduleState(safe_increment(mlr_state.count)) if callable(learning_rate) else mlr_state
        new_adam = ScaleByAdamState(safe_increment(adam_st.count), adam_st.mu, adam_st.nu, adam_st.magma_s,
                                    adam_key_next)
        new_alr = ScaleByScheduleState(safe_increment(alr_state.count)) if callable(
            adam_learning_rate) else alr_state
        new_state = PartitionState({
            "muon": MaskedState(((new_muon, *[bump_wd_state(s) for s in mstate[0][1:]]), new_mlr)),
            "adam": MaskedState((new_adam, *[bump_wd_state(s) for s in astate[1:-1]], new_alr)),
        })
        return tree_unflatten(treedef, full), new_state

    fused_update.supports_fused_apply = True
    return GradientTransformation(composite.init, fused_update)


__all__ = [
    "MuonDimensionNumbers",
    "MuonState",
    "muon",
    "orthogonalize_via_newton_schulz",
    "polar_express_coeffs",
    "resolve_ns_coeffs",
    "scale_by_muon",
    "scale_by_muon_shape",
    "scale_by_shape",
]
