"""Optax-shaped plumbing for the drop-in API.

The reference's transforms are Optax ``GradientTransformation`` objects
(``init(params) -> state``, ``update(updates, state, params) -> (updates,
state)``) combined with ``optax.chain`` / ``optax.partition`` and wrapped
with ``optax.masked`` (muon.py:395, 462-486; adam.py:380-404).  Optax is not
a dependency here; this module restates the pieces of it the Muon path uses,
with the same state types, over trees of ``torch.Tensor`` device buffers.

Elementwise transforms (``scale_by_muon_shape``, ``add_decayed_weights``,
``scale_by_learning_rate``) run through the library's ``rf_muon_tail``
kernel; nothing on the update path computes with torch ops.
"""

from __future__ import annotations

from typing import Any, Callable, NamedTuple

import torch

from . import _lib
from .tree import MaskedNode, is_aux_leaf, tree_flatten, tree_leaves, tree_map, tree_unflatten

Params = Any
Updates = Any
ScalarOrSchedule = Any


class GradientTransformation(NamedTuple):
    """optax.GradientTransformation."""

    init: Callable[[Params], Any]
    update: Callable[..., tuple[Updates, Any]]


class EmptyState(NamedTuple):
    """optax.EmptyState."""


class ScaleState(NamedTuple):
    """State of ``optax.scale`` (constant learning rate)."""


class ScaleByScheduleState(NamedTuple):
    """State of ``optax.scale_by_schedule``: the step count fed to the schedule."""

    count: torch.Tensor


class AddDecayedWeightsState(NamedTuple):
    """State of ``optax.add_decayed_weights``: empty (``count`` None) for a
    constant weight decay; for a scheduled one, the step count the schedule
    is evaluated at (0 on the first update)."""

    count: Any = None


class MaskedState(NamedTuple):
    """State of ``optax.masked``."""

    inner_state: Any


class PartitionState(NamedTuple):
    """State of ``optax.partition``."""

    inner_states: dict


NO_PARAMS_MSG = (
    "You are using a transformation that requires the current value of parameters, "
    "but you are not passing `params` when calling `update`."
)


def init_empty_state(params: Params) -> EmptyState:
    del params
    return EmptyState()


def host_count(x) -> int:
    """Step counters live on the host (int32 CPU tensors) so bias corrections
    and schedules never synchronise with the device."""
    return int(x.item()) if isinstance(x, torch.Tensor) else int(x)


def new_count(value: int = 0) -> torch.Tensor:
    return torch.tensor(value, dtype=torch.int32)


def safe_increment(count: torch.Tensor) -> torch.Tensor:
    """optax numerics.safe_increment: saturating int32 increment."""
    c = host_count(count)
    return new_count(c + 1 if c < 2**31 - 1 else c)


# ---------------------------------------------------------------------------
# dtype helpers
# ---------------------------------------------------------------------------
_RF_DTYPE = {torch.float32: _lib.RF_F32, torch.bfloat16: _lib.RF_BF16, torch.float16: _lib.RF_F16}


def rf_dtype(t: torch.Tensor) -> int:
    try:
        return _RF_DTYPE[t.dtype]
    except KeyError as exc:
        raise ValueError(f"unsupported dtype {t.dtype}; expected float32, bfloat16 or float16") from exc


def round_to_dtype(x: float, dtype: torch.dtype) -> float:
    """The value of Python float ``x`` once cast to ``dtype`` (JAX weak typing
    forms ``weight_decay * p`` in the parameter dtype)."""
    return float(torch.tensor(x, dtype=torch.float32).to(dtype).to(torch.float32))


def stream_handle(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(t: torch.Tensor, what: str) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{what} must be a CUDA torch.Tensor (the update path runs on the GPU only)")


def resolve_scalar(value: ScalarOrSchedule, count: int) -> float:
    """utils.py:93-102."""
    return float(value(count)) if callable(value) else float(value)


def decay_at(weight_decay: ScalarOrSchedule, count: int) -> tuple[float, bool]:
    """Weight decay at ``count`` and whether it is weakly typed.

    A Python scalar (a constant, or a schedule that returns one) is weakly
    typed under JAX's promotion rules, so ``weight_decay * p`` is formed in
    the parameter dtype; a schedule that returns an array or a NumPy scalar
    (a float32 value, as Optax schedules computed from the int32 step count
    return) is strongly typed and the product is formed in float32."""
    if not callable(weight_decay):
        return float(weight_decay), True
    v = weight_decay(count)
    return float(v), type(v) in (int, float)


def has_nonzero_or_scheduled(value: ScalarOrSchedule) -> bool:
    """utils.py:105-111."""
    if isinstance(value, (int, float)):
        if value < 0.0:
            raise ValueError("Scalar optimizer coefficients must be nonnegative.")
        return value != 0.0
    return True


def validate_positive(name: str, value) -> None:
    """utils.py:114-120."""
    if isinstance(value, (int, float)) and value <= 0.0:
        raise ValueError(f"{name} must be positive, got {value!r}.")


def validate_beta(name: str, value) -> None:
    """utils.py:132-138."""
    if isinstance(value, (int, float)) and not 0.0 <= value < 1.0:
        raise ValueError(f"{name} must be in [0, 1), got {value!r}.")


def resolve_mask(mask, params) -> Any:
    """utils.py:155-170."""
    if mask is None:
        return None
    if callable(mask):
        return mask(params)
    return mask


# ---------------------------------------------------------------------------
# Combinators (optax._src.combine / wrappers)
# ---------------------------------------------------------------------------


def chain(*transforms: GradientTransformation) -> GradientTransformation:
    """optax.chain."""

    def init_fn(params):
        return tuple(t.init(params) for t in transforms)

    def update_fn(updates, state, params=None, **extra):
        new_state = []
        for t, s in zip(transforms, state):
            updates, s = t.update(updates, s, params, **extra)
            new_state.append(s)
        return updates, tuple(new_state)

    return GradientTransformation(init_fn, update_fn)


def _mask_tree(tree, mask):
    return tree_map(lambda x, m: x if m else MaskedNode(), tree, mask, is_leaf=is_aux_leaf)


def masked(inner: GradientTransformation, mask) -> GradientTransformation:
    """optax.masked: ``inner`` sees MaskedNode at leaves where mask is False."""

    def init_fn(params):
        m = mask(params) if callable(mask) else mask
        return MaskedState(inner.init(_mask_tree(params, m)))

    def update_fn(updates, state, params=None, **extra):
        m = mask(updates) if callable(mask) else mask
        mu = _mask_tree(updates, m)
        mp = None if params is None else _mask_tree(params, m)
        new_u, new_inner = inner.update(mu, state.inner_state, mp, **extra)
        merged = tree_map(lambda n, o, k: n if k else o, new_u, updates, m, is_leaf=is_aux_leaf)
        return merged, MaskedState(new_inner)

    return GradientTransformation(init_fn, update_fn)


def partition(transforms: dict, param_labels) -> GradientTransformation:
    """optax.partition (multi_transform)."""

    def labels_of(tree):
        return param_labels(tree) if callable(param_labels) else param_labels

    def make_mask(labels, group):
        return tree_map(lambda lab: lab == group, labels)

    def init_fn(params):
        labels = labels_of(params)
        used = set(x for x in tree_leaves(labels) if x is not None)
        missing = used - set(transforms)
        if missing:
            raise ValueError(f"Some parameters have no corresponding transformation: {sorted(missing)}")
        return PartitionState(
            {g: masked(t, make_mask(labels, g)).init(params) for g, t in transforms.items()}
        )

    def update_fn(updates, state, params=None, **extra):
        labels = labels_of(updates)
        new_inner = {}
        for g, t in transforms.items():
            updates, new_inner[g] = masked(t, make_mask(labels, g)).update(
                updates, state.inner_states[g], params, **extra
            )
        return updates, PartitionState(new_inner)

    return GradientTransformation(init_fn, update_fn)


# ---------------------------------------------------------------------------
# Elementwise transforms on the rf_muon_tail kernel:
#   out = -lr * (shape_scale * u + decay * p)
# ---------------------------------------------------------------------------


SIDE_CTAS_PER_SM = 2  # occupancy of HBM-bound kernels run beside the persistent GEMM kernel


def run_tail(items, lr: float, max_ctas_per_sm: int = 0) -> None:
    """items: list of (u, p_or_None, out, shape_scale, decay[, decay_in_f32])."""
    if not items:
        return
    lib = _lib.load()
    arr = (_lib.RfTailLeaf * len(items))()
    for i, item in enumerate(items):
        u, p, out, scale, decay = item[:5]
        arr[i].decay_in_f32 = int(bool(item[5])) if len(item) > 5 else 0
        arr[i].o = u.data_ptr()
        arr[i].param = p.data_ptr() if p is not None else None
        arr[i].out = out.data_ptr()
        arr[i].n = u.numel()
        arr[i].o_dtype = rf_dtype(u)
        arr[i].param_dtype = rf_dtype(p) if p is not None else _lib.RF_F32
        arr[i].out_dtype = rf_dtype(out)
        arr[i].shape_scale = scale
        arr[i].decay = decay
    _lib.check(lib.rf_muon_tail(arr, len(items), lr, int(max_ctas_per_sm),
                                torch.cuda.current_stream(items[0][0].device).cuda_stream))


def _array_leaves(tree):
    leaves, treedef = tree_flatten(tree, is_leaf=is_aux_leaf)
    return leaves, treedef


def scale_by_learning_rate(learning_rate: ScalarOrSchedule, *, flip_sign: bool = True) -> GradientTransformation:
    """optax.scale_by_learning_rate: multiplies by -lr (schedule-aware)."""
    sign = -1.0 if flip_sign else 1.0

    def init_fn(params):
        return ScaleByScheduleState(new_count(0)) if callable(learning_rate) else ScaleState()

    def update_fn(updates, state, params=None, **extra):
        if callable(learning_rate):
            c = host_count(state.count)
            lr = float(learning_rate(c))
            new_state = ScaleByScheduleState(safe_increment(state.count))
        else:
            lr = float(learning_rate)
            new_state = state
        leaves, treedef = _array_leaves(updates)
        items, outs = [], []
        for u in leaves:
            if is_aux_leaf(u):
                outs.append(u)
                continue
            require_cuda(u, "update")
            o = torch.empty_like(u)
            items.append((u.contiguous(), None, o, 1.0, 0.0))
            outs.append(o)
        run_tail(items, -sign * lr)
        return tree_unflatten(treedef, outs), new_state

    return GradientTransformation(init_fn, update_fn)


def add_decayed_weights(weight_decay: ScalarOrSchedule = 0.0, mask=None) -> GradientTransformation:
    """optax.add_decayed_weights: ``u + weight_decay * p``.  A constant (Python
    float) weight decay forms the product in the parameter dtype (JAX weak
    typing); a schedule is evaluated at the transform's own step count, kept
    in its state, and its product's dtype follows ``decay_at``."""
    scheduled = callable(weight_decay)

    def init_fn(params):
        return AddDecayedWeightsState(new_count(0)) if scheduled else AddDecayedWeightsState()

    def update_fn(updates, state, params=None, **extra):
        if params is None:
            raise ValueError(NO_PARAMS_MSG)
        wd, weak = decay_at(weight_decay, host_count(state.count) if scheduled else 0)
        leaves, treedef = _array_leaves(updates)
        pleaves = tree_flatten(params, is_leaf=is_aux_leaf)[0]
        items, outs = [], []
        for u, p in zip(leaves, pleaves):
            if is_aux_leaf(u) or is_aux_leaf(p):
                outs.append(u)
                continue
            require_cuda(u, "update")
            o = torch.empty(u.shape, dtype=torch.promote_types(u.dtype, p.dtype if weak else torch.float32),
                            device=u.device)
            items.append((u.contiguous(), p.contiguous(), o, 1.0, round_to_dtype(wd, p.dtype) if weak else wd,
                          not weak))
            outs.append(o)
        run_tail(items, -1.0)
        new_state = AddDecayedWeightsState(safe_increment(state.count)) if scheduled else state
        return tree_unflatten(treedef, outs), new_state

    tx = GradientTransformation(init_fn, update_fn)
    if mask is not None:
        return masked(tx, mask)
    return tx


def _splitmix64(x: int) -> int:
    """One SplitMix64 output for state ``x`` (Steele, Lea and Flood, 2014)."""
    m = (1 << 64) - 1
    z = (x + 0x9E3779B97F4A7C15) & m
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & m
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & m
    return z ^ (z >> 31)


def key_seed(key) -> int:
    """64-bit seed of a PRNG key: an int, or a 2-element tensor / sequence of
    32-bit words like ``jax.random.PRNGKey`` (``fresh_key`` layout)."""
    if isinstance(key, int):
        return key & ((1 << 64) - 1)
    words = [int(v) & 0xFFFFFFFF for v in (key.reshape(-1).tolist() if isinstance(key, torch.Tensor) else key)]
    if len(words) != 2:
        raise ValueError("a PRNG key is an int or two 32-bit words")
    return (words[0] << 32) | words[1]


def state_dtype(mu_dtype) -> torch.dtype:
    """Optimizer-state dtype for ``mu_dtype`` (muon.py:207-210, adam.py:98-106):
    float32 by default; bfloat16 state is stored with stochastic rounding."""
    if mu_dtype is None or mu_dtype in (torch.float32, "float32", "f32"):
        return torch.float32
    if mu_dtype in (torch.bfloat16, "bfloat16", "bf16"):
        return torch.bfloat16
    raise NotImplementedError(f"mu_dtype={mu_dtype!r}: float32 or bfloat16 optimizer state is supported")


def sr_step_seeds(key, n: int) -> tuple[list, torch.Tensor]:
    """Noise seeds for one step's stochastically rounded state (``n`` streams)
    and the advanced key.  The reference splits its PRNG key once per step
    (utils.py:545-562, adam.py:128-131) and draws Threefry bits; here the
    key's 64 bits seed SplitMix64 streams instead."""
    k = key_seed(key)
    step = _splitmix64(k ^ 0xD1B54A32D192ED03)
    seeds = [_splitmix64((step + i) & ((1 << 64) - 1)) for i in range(n)]
    nk = _splitmix64(k)
    return seeds, torch.tensor([(nk >> 32) & 0xFFFFFFFF, nk & 0xFFFFFFFF], dtype=torch.int64)


def advance_key(key) -> torch.Tensor:
    """The state key of the next step (the key sr_step_seeds returns)."""
    return sr_step_seeds(key, 0)[1]


_MAGMA_DOMAIN = 0x6A09E667F3BCC908


def magma_keeps(key, n: int, p: float) -> list[int]:
    """One Magma step's per-leaf Bernoulli(p) draws (magma.py:83, 122: a
    subkey per leaf, ``bernoulli(subkey, p)``).  The reference draws from
    JAX's Threefry stream; here each leaf's draw is a SplitMix64 output of a
    stream derived from the state key, ``keep = u < p`` with
    ``u = (x >> 11) * 2**-53`` uniform on [0, 1): the same distribution, a
    different sequence."""
    base = _splitmix64(key_seed(key) ^ _MAGMA_DOMAIN)
    m = (1 << 64) - 1
    return [int((_splitmix64((base + i) & m) >> 11) * (2.0 ** -53) < p) for i in range(n)]


def init_magma_state(params):
    """utils.py:64-69: a float32 score of 0.5 per (non-aux) leaf, on the
    leaf's device (meta for meta leaves)."""
    leaves, treedef = tree_flatten(params, is_leaf=is_aux_leaf)
    return tree_unflatten(treedef, [x if is_aux_leaf(x) else torch.full((), 0.5, dtype=torch.float32, device=x.device)
                                    for x in leaves])


def validate_magma_args(p: float, tau: float) -> None:
    """magma.py:8-13."""
    if not 0.0 <= p <= 1.0:
        raise ValueError(f"magma_p must be in [0, 1], got {p!r}.")
    if tau <= 0.0:
        raise ValueError(f"magma_tau must be positive, got {tau!r}.")


def apply_updates(params, updates, key=None, stochastic: bool = True):
    """rollfast.utils.apply_updates (utils.py:648-708) on the
    ``rf_apply_updates`` kernel: ``p + u`` in float32, cast to the parameter
    dtype; bfloat16 parameters round stochastically when ``stochastic``
    (utils.py:342-371).  Each leaf gets its own noise stream (the reference
    splits ``key`` per leaf); the bits differ from JAX's Threefry stream, so
    stochastic results agree with the reference in distribution only.
    Returns new parameter tensors."""
    if stochastic and key is None:
        raise ValueError(
            "apply_updates requires a PRNG `key` when stochastic=True. "
            "Pass stochastic=False for deterministic rounding."
        )
    seed = key_seed(key) if stochastic else 0
    leaves, treedef = tree_flatten(params, is_leaf=is_aux_leaf)
    ups = tree_flatten(updates, is_leaf=is_aux_leaf)[0]
    if len(ups) != len(leaves):
        raise ValueError("params and updates must have the same tree structure")
    items, outs = [], []
    for idx, (p, u) in enumerate(zip(leaves, ups)):
        if is_aux_leaf(p) or is_aux_leaf(u):
            outs.append(p)
            continue
        require_cuda(p, "param")
        require_cuda(u, "update")
        if p.shape != u.shape:
            raise ValueError(f"leaf {idx}: param shape {tuple(p.shape)} != update shape {tuple(u.shape)}")
        out = torch.empty_like(p, memory_format=torch.contiguous_format)
        items.append((p.contiguous(), u.contiguous(), out, _splitmix64(seed + idx) if stochastic else 0))
        outs.append(out)
    if items:
        lib = _lib.load()
        arr = (_lib.RfApplyLeaf * len(items))()
        for i, (p, u, out, sd) in enumerate(items):
            arr[i].param = p.data_ptr()
            arr[i].update = u.data_ptr()
            arr[i].out = out.data_ptr()
            arr[i].n = p.numel()
            arr[i].param_dtype = rf_dtype(p)
            arr[i].update_dtype = rf_dtype(u)
            arr[i].seed = sd
        _lib.check(lib.rf_apply_updates(arr, len(items), int(bool(stochastic)),
                                        torch.cuda.current_stream(items[0][0].device).cuda_stream))
    return tree_unflatten(treedef, outs)


def update_and_apply(tx: GradientTransformation, grads, state, params, key=None, stochastic: bool = True,
                     inplace: bool = False):
    """One optimizer step that returns new parameters: ``tx.update`` followed
    by ``apply_updates`` (utils.py:648-708), i.e.
    ``apply_updates(params, *tx.update(grads, state, params)[:1], key, stochastic)``
    together with the new state.

    For ``rollfast_b200.muon(...)`` on one GPU the apply is fused into the
    update kernels: the Newton-Schulz final epilogue and the AdamW kernel
    write ``p + u`` (rounded to the parameter dtype; bfloat16 stochastically
    when ``stochastic``, with the same noise streams ``apply_updates`` uses
    for ``key``) instead of the float32 update, which is never written to
    memory.  ``inplace``: write the new values into the parameter buffers
    (contiguous leaves in the reference's (batch, R, O) layout), as JAX would
    with donated parameters.  Other transforms (and the sharded multi-GPU
    update) run the two calls.  Returns ``(new_params, new_state)``."""
    if stochastic and key is None:
        raise ValueError(
            "apply_updates requires a PRNG `key` when stochastic=True. "
            "Pass stochastic=False for deterministic rounding."
        )
    if getattr(tx.update, "supports_fused_apply", False):
        return tx.update(grads, state, params, apply_updates=(key, stochastic, inplace))
    updates, state = tx.update(grads, state, params)
    return apply_updates(params, updates, key, stochastic), state
