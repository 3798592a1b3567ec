"""NumPy restatement of rollfast's Muon update path (test infrastructure only).

Every function names the reference file:line it restates.  Paths are relative
to the reference project root (RhizomeResearch/rollfast).

Precision modes:
  * ``np.float32`` -- "reference-equivalent": the reference casts the
    Newton-Schulz input to float32 (orthogonalization.py:227) and keeps the
    moments in float32 (utils.py:437-467).
  * ``np.float64`` -- "truth": the same algorithm in double precision.

Trees are nested ``dict`` / ``list`` / ``tuple`` containers of NumPy arrays,
with ``None`` and :class:`MaskedNode` as auxiliary leaves, matching the
reference's use of ``jax.tree.map(..., is_leaf=_is_aux_leaf)``.
"""

from __future__ import annotations

import math
from typing import Any, Callable, NamedTuple, Sequence

import numpy as np

__all__ = [
    "PRECONDITIONINGS",
    "apply_updates",
    "store_state",
    "noise16",
    "splitmix64",
    "stochastic_round_bf16",
    "MaskedNode",
    "MatrixDimensionNumbers",
    "MUON_NS_COEFFS",
    "DION_NS_COEFFS",
    "NS_COEFFS_PRESETS",
    "polar_express_coeffs",
    "resolve_ns_coeffs",
    "compute_matrix_reshape",
    "normalize_axes",
    "get_dimension_numbers",
    "make_matrix_partition_fns",
    "quintic_newton_schulz",
    "orthogonalize_via_newton_schulz",
    "momentum_runtime",
    "shape_scale_factor",
    "adam_leaf_update",
    "pow32",
    "magma_leaf",
    "decay_at",
    "decay_term",
    "in_transform_decay",
    "OracleMuon",
    "bf16_round",
    "f16_round",
    "tree_map",
    "tree_leaves_with_path",
]


# --------------------------------------------------------------------------
# Tree helpers (restating the jax.tree.map usage with aux-leaf handling,
# utils.py:13-22).
# --------------------------------------------------------------------------


class MaskedNode(NamedTuple):
    """Placeholder for a leaf routed to the other partition branch
    (optax.transforms._masking.MaskedNode, used at utils.py:13-14)."""


def is_aux_leaf(x: Any) -> bool:
    """utils.py:13-14: ``None`` and ``MaskedNode`` are auxiliary leaves."""
    return x is None or isinstance(x, MaskedNode)


def _is_container(x: Any) -> bool:
    return isinstance(x, (dict, list)) or (
        isinstance(x, tuple) and not isinstance(x, MaskedNode)
    )


def tree_map(fn: Callable, tree: Any, *rest: Any, is_leaf=None) -> Any:
    """Structural map over dict/list/tuple/NamedTuple trees."""
    if is_leaf is not None and is_leaf(tree):
        return fn(tree, *rest)
    if is_aux_leaf(tree):
        return fn(tree, *rest)
    if isinstance(tree, dict):
        return {k: tree_map(fn, tree[k], *[r[k] for r in rest], is_leaf=is_leaf) for k in tree}
    if isinstance(tree, tuple) and hasattr(tree, "_fields"):
        return type(tree)(
            *[tree_map(fn, v, *[r[i] for r in rest], is_leaf=is_leaf) for i, v in enumerate(tree)]
        )
    if isinstance(tree, (list, tuple)):
        out = [tree_map(fn, v, *[r[i] for r in rest], is_leaf=is_leaf) for i, v in enumerate(tree)]
        return type(tree)(out)
    return fn(tree, *rest)


def tree_leaves_with_path(tree: Any, prefix=()):
    """Flatten to (path, leaf) pairs in deterministic (insertion) order."""
    if is_aux_leaf(tree):
        return [(prefix, tree)]
    if isinstance(tree, dict):
        out = []
        for k in tree:
            out += tree_leaves_with_path(tree[k], prefix + (k,))
        return out
    if isinstance(tree, (list, tuple)) and not hasattr(tree, "_fields"):
        out = []
        for i, v in enumerate(tree):
            out += tree_leaves_with_path(v, prefix + (i,))
        return out
    return [(prefix, tree)]


# --------------------------------------------------------------------------
# 16-bit rounding helpers (used to model parameter dtypes).
# --------------------------------------------------------------------------


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), returned
    as float32.  NaN/Inf pass through."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).copy()
    bad = ~np.isfinite(x)
    out[bad] = x[bad]
    return out


def f16_round(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


# --------------------------------------------------------------------------
# Dimension numbers (dimension_numbers.py).
# --------------------------------------------------------------------------


class MatrixDimensionNumbers(NamedTuple):
    """dimension_numbers.py:15-24."""

    reduction_axis: Sequence[int] | int = 0
    output_axis: Sequence[int] | int = 1


def _is_dimension_numbers_leaf(x: Any) -> bool:
    """dimension_numbers.py:48-49."""
    return x is None or isinstance(x, (MatrixDimensionNumbers, MaskedNode))


def _has_matrix_spec(d: Any) -> bool:
    """dimension_numbers.py:56-57."""
    return d is not None and not isinstance(d, MaskedNode)


def _normalize_axis_group(ndim: int, axes, name: str) -> tuple[int, ...]:
    """dimension_numbers.py:288-309."""
    axes_tuple = (axes,) if isinstance(axes, int) else tuple(axes)
    if not axes_tuple:
        raise ValueError(f"{name} must not be empty.")
    norm = []
    for axis in axes_tuple:
        if axis < -ndim or axis >= ndim:
            raise ValueError(f"{name} axis {axis} is out of bounds for rank-{ndim} parameter.")
        norm.append(axis if axis >= 0 else axis + ndim)
    t = tuple(norm)
    if len(set(t)) != len(t):
        raise ValueError(f"{name} contains duplicate axes: {axes_tuple}.")
    return t


def normalize_axes(shape, dim_nums: MatrixDimensionNumbers):
    """dimension_numbers.py:279-285."""
    ndim = len(shape)
    return (
        _normalize_axis_group(ndim, dim_nums.reduction_axis, "reduction_axis"),
        _normalize_axis_group(ndim, dim_nums.output_axis, "output_axis"),
    )


def compute_matrix_reshape(shape, dim_nums: MatrixDimensionNumbers):
    """dimension_numbers.py:312-359: forward/inverse reshapes to the
    ``(batch, reduction, output)`` layout."""
    shape = tuple(shape)
    if len(shape) < 2:
        raise ValueError(f"Matrix-optimized parameters must have rank >= 2, got x.ndim={len(shape)}.")
    red, out = normalize_axes(shape, dim_nums)
    if set(red) & set(out):
        raise ValueError(f"Reduction and output axes must be disjoint. Got {red} and {out}.")
    batch = tuple(a for a in range(len(shape)) if a not in red and a not in out)
    perm = batch + red + out
    inv = [0] * len(shape)
    for o, i in enumerate(perm):
        inv[i] = o
    flat = (
        math.prod(shape[a] for a in batch),
        math.prod(shape[a] for a in red),
        math.prod(shape[a] for a in out),
    )
    unflat = tuple(shape[a] for a in batch) + tuple(shape[a] for a in red) + tuple(shape[a] for a in out)
    fwd = lambda x: np.transpose(x, perm).reshape(flat)
    bwd = lambda x: np.transpose(np.reshape(x, unflat), tuple(inv))
    return fwd, bwd


def get_dimension_numbers(weight_dimension_numbers, params):
    """dimension_numbers.py:82-116: default routes only rank-2 leaves."""
    if weight_dimension_numbers is None:
        return tree_map(
            lambda x: None
            if is_aux_leaf(x)
            else (MatrixDimensionNumbers() if getattr(x, "ndim", None) == 2 else None),
            params,
        )
    if callable(weight_dimension_numbers) and not isinstance(weight_dimension_numbers, MatrixDimensionNumbers):
        return weight_dimension_numbers(params)
    if isinstance(weight_dimension_numbers, MatrixDimensionNumbers):
        if hasattr(params, "shape") and hasattr(params, "dtype"):
            return weight_dimension_numbers
        raise ValueError(
            "A bare MatrixDimensionNumbers can only be used with a single array leaf."
        )
    return weight_dimension_numbers


def make_matrix_partition_fns(weight_dimension_numbers, matrix_label: str, fallback_label: str = "adam"):
    """dimension_numbers.py:137-215: labels / masked specs / default mask."""

    def resolve(params):
        return get_dimension_numbers(weight_dimension_numbers, params)

    def labels(params):
        return tree_map(
            lambda d, p: None if p is None else (matrix_label if _has_matrix_spec(d) else fallback_label),
            resolve(params),
            params,
            is_leaf=_is_dimension_numbers_leaf,
        )

    def masked_specs(params):
        return tree_map(
            lambda d: d if d is not None else MaskedNode(),
            resolve(params),
            is_leaf=_is_dimension_numbers_leaf,
        )

    def default_mask(params):
        return tree_map(
            lambda d, p: False if (p is None or isinstance(p, MaskedNode)) else _has_matrix_spec(d),
            resolve(params),
            params,
            is_leaf=_is_dimension_numbers_leaf,
        )

    return resolve, labels, masked_specs, default_mask


# --------------------------------------------------------------------------
# Newton-Schulz coefficients (orthogonalization.py:42-147).
# --------------------------------------------------------------------------

MUON_NS_COEFFS = (3.4445, -4.7750, 2.0315)  # orthogonalization.py:42
DION_NS_COEFFS = (  # orthogonalization.py:43-49
    (4.0848, -6.8946, 2.9270),
    (3.9505, -6.3029, 2.6377),
    (3.7418, -5.5913, 2.3037),
    (2.8769, -3.1427, 1.2046),
    (2.8366, -3.0525, 1.2012),
)
NS_COEFFS_PRESETS = {"standard": MUON_NS_COEFFS, "dion": DION_NS_COEFFS}


def _optimal_quintic(l: float, u: float):
    """orthogonalization.py:58-84: equi-oscillating odd quintic on [l, u]
    found by a Remez exchange (4x4 solve per sweep, <=1000 sweeps)."""
    if not 0 < l <= u:
        raise ValueError(f"l must satisfy 0 < l <= u, got l={l}, u={u}.")
    if l / u >= 1 - 1e-5:
        return (15 / 8) / u, (-10 / 8) / (u**3), (3 / 8) / (u**5)
    q = (3 * l + u) / 4
    r = (l + 3 * u) / 4
    err = np.inf
    old_err = None
    a = b = c = 0.0
    for _ in range(1000):
        if old_err is not None and abs(old_err - err) <= 1e-15:
            break
        old_err = err
        lhs = np.array(
            [[l, l**3, l**5, 1], [q, q**3, q**5, -1], [r, r**3, r**5, 1], [u, u**3, u**5, -1]]
        )
        a, b, c, err = np.linalg.solve(lhs, np.ones(4))
        q, r = np.sqrt((-3 * b + np.array([-1, 1]) * np.sqrt(9 * b**2 - 20 * a * c)) / (10 * c))
    return float(a), float(b), float(c)


def polar_express_coeffs(l: float = 1e-3, num_iters: int = 8, *, safety_factor_eps: float = 2e-2,
                         cushion: float = 0.02407327424182761):
    """orthogonalization.py:87-119."""
    u = 1.0
    if not 0 < l <= u:
        raise ValueError(f"l must satisfy 0 < l <= 1, got {l}.")
    if num_iters < 1:
        raise ValueError(f"num_iters must be >= 1, got {num_iters}.")
    sf = 1 + safety_factor_eps
    out = []
    for i in range(num_iters):
        a, b, c = _optimal_quintic(max(l, cushion * u), u)
        if cushion * u > l:
            pl = a * l + b * l**3 + c * l**5
            pu = a * u + b * u**3 + c * u**5
            rs = 2 / (pl + pu)
            a, b, c = a * rs, b * rs, c * rs
        if i < num_iters - 1:
            a /= sf
            b /= sf**3
            c /= sf**5
        out.append((a, b, c))
        l = a * l + b * l**3 + c * l**5
        u = 2 - l
    return out


def resolve_ns_coeffs(ns_coeffs, ns_steps) -> np.ndarray:
    """orthogonalization.py:122-147; returns float32 like ``jnp.asarray``."""
    n = int(ns_steps)
    if isinstance(ns_coeffs, str):
        if ns_coeffs == "polar_express":
            coeffs = polar_express_coeffs(num_iters=n)
        elif ns_coeffs in NS_COEFFS_PRESETS:
            coeffs = NS_COEFFS_PRESETS[ns_coeffs]
        else:
            raise ValueError(f"Unknown ns_coeff preset string: {ns_coeffs}")
    else:
        coeffs = ns_coeffs
    arr = np.asarray(coeffs, dtype=np.float32)
    if arr.ndim > 2 or arr.shape[-1] != 3:
        raise ValueError(f"ns_coeffs must have shape (3,) or (n, 3), got {arr.shape}")
    if arr.ndim == 2:
        if arr.shape[0] < n:
            raise ValueError(f"Not enough coeffs to perform {ns_steps} steps")
        arr = arr[:n]
    return arr


# --------------------------------------------------------------------------
# Quintic Newton-Schulz (orthogonalization.py:179-305).
# --------------------------------------------------------------------------


PRECONDITIONINGS = ("frobenius", "spectral", "aol", "schatten")


def _aol_first_iteration(m, a, b, c, dtype, clip=1e-8):
    """orthogonalization.py:153-163.  The reference calls it without an
    ``eps`` argument (189-192), so the clip is its default 1e-8."""
    A = np.matmul(m, np.swapaxes(m, -1, -2))
    rescaling = np.maximum(np.abs(A).sum(axis=-1), dtype(clip)).astype(dtype)
    s = (dtype(1.0) / np.sqrt(rescaling)).astype(dtype)[..., :, None]
    m = (m * s).astype(dtype)
    A = (A * s * np.swapaxes(s, -1, -2)).astype(dtype)
    B = b * A + c * np.matmul(A, A)
    return (a * m + np.matmul(B, m)).astype(dtype)


def _schatten_first_iteration(m, a, b, c, dtype, clip=1e-8):
    """orthogonalization.py:166-176 (clip: its default 1e-8, as called at 198-201)."""
    A = np.matmul(m, np.swapaxes(m, -1, -2))
    fro = np.sqrt(np.sum(A * A, axis=(-2, -1), keepdims=True, dtype=dtype)).astype(dtype)
    s = (dtype(1.0) / np.sqrt(np.maximum(fro, dtype(clip)))).astype(dtype)
    m = (m * s).astype(dtype)
    A = (A * s * s).astype(dtype)
    B = b * A + c * np.matmul(A, A)
    return (a * m + np.matmul(B, m)).astype(dtype)


def quintic_newton_schulz(x: np.ndarray, ns_coeffs, ns_steps: int = 5, eps: float = 1e-8,
                          dtype=np.float32, preconditioning: str = "frobenius") -> np.ndarray:
    """orthogonalization.py:211-273.

    Over the last two axes: cast (227), transpose when rows > cols (228-231),
    then by ``preconditioning`` (233-250): "frobenius" X / (||X||_F + eps),
    "spectral" X / (||X||_2 + eps), "aol" / "schatten" no pre-scaling but a
    rescaled first iteration (153-176, 189-201).  Each step is
    A = X X^T, B = b A + c A A, X = a X + B X (179-182), with a (3,) array
    repeated ``ns_steps`` times (253-260) or an (n,3) schedule scanned in
    order (262-269); untranspose (271-272).
    """
    coeffs = np.asarray(ns_coeffs, dtype=dtype)
    if coeffs.ndim > 2 or coeffs.shape[-1] != 3:
        raise ValueError("Newton-Schulz coefficients must have shape (3,) or (n, 3), got "
                         f"{coeffs.shape}.")
    if x.ndim < 2:
        raise ValueError(f"Input must have rank >= 2, got shape={x.shape}.")
    if preconditioning not in PRECONDITIONINGS:
        raise ValueError(f"Unknown preconditioning {preconditioning!r}.")
    m = np.asarray(x).astype(dtype)
    transposed = m.shape[-2] > m.shape[-1]
    if transposed:
        m = np.swapaxes(m, -1, -2)
    if preconditioning == "frobenius":
        norm = np.sqrt(np.sum(m.astype(dtype) * m, axis=(-2, -1), keepdims=True, dtype=dtype)).astype(dtype)
        m = (m / (norm + dtype(eps))).astype(dtype)
    elif preconditioning == "spectral":
        # ord=2 matrix norm: the largest singular value (computed in float64 here).
        sv = np.linalg.norm(m.astype(np.float64), ord=2, axis=(-2, -1), keepdims=True).astype(dtype)
        m = (m / (sv + dtype(eps))).astype(dtype)
    schedule = [coeffs] * int(ns_steps) if coeffs.ndim == 1 else list(coeffs)
    for i, (a, b, c) in enumerate(schedule):
        if i == 0 and preconditioning == "aol":
            m = _aol_first_iteration(m, a, b, c, dtype)
            continue
        if i == 0 and preconditioning == "schatten":
            m = _schatten_first_iteration(m, a, b, c, dtype)
            continue
        mt = np.swapaxes(m, -1, -2)
        A = np.matmul(m, mt)
        B = b * A + c * np.matmul(A, A)
        m = (a * m + np.matmul(B, m)).astype(dtype)
    if transposed:
        m = np.swapaxes(m, -1, -2)
    return np.ascontiguousarray(m)


def orthogonalize_via_newton_schulz(x, ns_coeffs, ns_steps=5, preconditioning="frobenius",
                                    eps=1e-8, dimension_numbers=None, dtype=np.float32):
    """orthogonalization.py:276-305."""
    if is_aux_leaf(x):
        return x
    if x.ndim != 2 and not isinstance(dimension_numbers, MatrixDimensionNumbers):
        raise ValueError("Input must have shape (m, n) or weight dimension numbers must be provided.")
    if x.ndim == 2:
        dimension_numbers = MatrixDimensionNumbers(0, 1)
    fwd, bwd = compute_matrix_reshape(x.shape, dimension_numbers)
    return bwd(quintic_newton_schulz(fwd(x), ns_coeffs, ns_steps, eps, dtype, preconditioning))


# --------------------------------------------------------------------------
# Parameter apply (utils.py:342-371, 648-708).
# --------------------------------------------------------------------------
_GAMMA = np.uint64(0x9E3779B97F4A7C15)


def splitmix64(state: np.ndarray) -> np.ndarray:
    """SplitMix64 output for each 64-bit state (Steele, Lea and Flood, 2014):
    z = state + gamma, then the two xor-shift-multiply rounds."""
    with np.errstate(over="ignore"):
        z = np.asarray(state, np.uint64) + _GAMMA
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def noise16(seed: int, n: int) -> np.ndarray:
    """The library's 16-bit rounding noise for elements 0..n-1 of a leaf:
    SplitMix64 output c (state seed + c * gamma) feeds elements 4c..4c+3,
    16 bits each from the low end.  (The reference uses JAX Threefry bits
    here, which cannot be reproduced without JAX.)"""
    c = np.arange((n + 3) // 4, dtype=np.uint64)
    with np.errstate(over="ignore"):
        r = splitmix64(np.uint64(seed) + c * _GAMMA)
    parts = [(r >> np.uint64(16 * k)) & np.uint64(0xFFFF) for k in range(4)]
    return np.stack(parts, axis=1).reshape(-1)[:n].astype(np.uint32)


def stochastic_round_bf16(x: np.ndarray, noise: np.ndarray) -> np.ndarray:
    """utils.py:342-371 with given 16-bit noise: add it to the float32 bits
    (none for +-Inf / NaN), clear the low 16 bits; returns float32 arrays
    holding bfloat16 values."""
    b = np.ascontiguousarray(np.asarray(x, np.float32)).view(np.uint32)
    special = (b & np.uint32(0x7FFFFFFF)) >= np.uint32(0x7F800000)
    n = np.where(special, np.uint32(0), np.asarray(noise, np.uint32) & np.uint32(0xFFFF))
    return ((b + n) & np.uint32(0xFFFF0000)).astype(np.uint32).view(np.float32)


def apply_updates(p: np.ndarray, u: np.ndarray, param_dtype: str, *, stochastic: bool = False,
                  seed: int = 0) -> np.ndarray:
    """utils.py:648-708 for one leaf (float32 arrays carrying the stored
    values): the sum in float32, then the parameter dtype; bfloat16 rounds
    stochastically (noise16(seed)) or to nearest even."""
    total = (np.asarray(p, np.float32) + np.asarray(u, np.float32)).astype(np.float32)
    if param_dtype == "bfloat16":
        if stochastic:
            return stochastic_round_bf16(total, noise16(seed, total.size).reshape(total.shape))
        return bf16_round(total)
    if param_dtype == "float16":
        return f16_round(total)
    return total


# --------------------------------------------------------------------------
# First-moment runtime (utils.py:327-645) and shape/decay/LR tail.
# --------------------------------------------------------------------------


def pow32(b, t: int, dtype=np.float32):
    """``b ** t`` for a float32 ``b``, correctly rounded to float32 (the power
    formed in float64).  JAX forms the bias-correction powers (utils.py:505,
    adam.py:137-141) in float32 with XLA's pow, whose last bit is not pinned;
    the CUDA host uses this same correctly rounded value.  The last bit
    matters: 1 - 0.999^t cancels, so one ulp of 0.999^9 is ~7e-6 relative in
    the AdamW second-moment correction."""
    return dtype(np.float64(dtype(b)) ** int(t))


def momentum_runtime(g: np.ndarray, mu: np.ndarray, count: int, beta: float, *, nesterov: bool,
                     accumulator: str = "ema", dtype=np.float32):
    """utils.py:565-645 as called by scale_by_muon (muon.py:240-253:
    bias_correction=True, nesterov_moment_count_offset=1).

    Returns (mu_new, direction) in ``dtype``.
      * mu_t = s*g + beta*mu   with s = 1-beta (ema) or 1 (heavy_ball)
        (utils.py:437-467, 327-339).
      * bias correction /(1-beta^k) for ema only (utils.py:496-506),
        k = t+1 for the moment under Nesterov, t for the gradient.
      * Nesterov lookahead beta*m + s*g (utils.py:509-530).
    """
    if accumulator not in ("ema", "heavy_ball"):
        raise ValueError(f"momentum_accumulator must be 'ema' or 'heavy_ball', got {accumulator!r}.")
    b = dtype(beta)
    s = dtype(1.0) - b if accumulator == "ema" else dtype(1.0)
    gf = np.asarray(g).astype(dtype)
    mu_new = (s * gf + b * np.asarray(mu).astype(dtype)).astype(dtype)
    t = count + 1
    if accumulator == "ema":
        k_mu = t + 1 if nesterov else t
        mu_t = mu_new / (dtype(1.0) - pow32(b, k_mu, dtype))
        g_t = gf / (dtype(1.0) - pow32(b, t, dtype)) if nesterov else gf
    else:
        mu_t = mu_new
        g_t = gf
    d = (b * mu_t + s * g_t) if nesterov else mu_t
    return mu_new, d.astype(dtype)


def store_state(x: np.ndarray, state_dtype: str, seed: int = 0) -> np.ndarray:
    """utils.py:412-425 / adam.py:219-225: the stored optimizer state.
    float32 is kept as is; bfloat16 rounds stochastically (utils.py:342-371)
    with the library's noise16 stream of ``seed`` over the flat index."""
    x = np.asarray(x, np.float32)
    if state_dtype == "bfloat16":
        return stochastic_round_bf16(x.reshape(-1), noise16(seed, x.size)).reshape(x.shape)
    return x


def shape_scale_factor(shape, dim_nums: MatrixDimensionNumbers, consistent_rms=None) -> np.float32:
    """muon.py:70-100: width-transfer sqrt(max(1, fan_out/fan_in)) or
    consistent-RMS sqrt(max(fan_in, fan_out)) * r."""
    red, out = normalize_axes(shape, dim_nums)
    fan_in = math.prod(shape[a] for a in red)
    fan_out = math.prod(shape[a] for a in out)
    if consistent_rms is None:
        return np.sqrt(np.float32(max(1.0, fan_out / fan_in)), dtype=np.float32)
    return np.float32(np.sqrt(np.float32(max(fan_in, fan_out)), dtype=np.float32) * np.float32(consistent_rms))


def decay_term(p: np.ndarray, wd: float, param_dtype: str) -> np.ndarray:
    """Optax add_decayed_weights ``g + weight_decay * p`` (muon.py:390-393,
    adam.py:398-401): the Python-float ``weight_decay`` is weakly typed, so
    the product is formed in the parameter dtype (bfloat16 for bf16 params)
    before it is promoted to float32 for the sum."""
    pf = np.asarray(p, dtype=np.float32)
    if param_dtype == "bfloat16":
        return bf16_round(bf16_round(np.full((), wd, np.float32)) * pf)
    if param_dtype == "float16":
        return f16_round(f16_round(np.full((), wd, np.float32)) * pf)
    return (np.float32(wd) * pf).astype(np.float32)


def decay_at(weight_decay, count: int):
    """(value, weak) of a scalar-or-schedule weight decay at ``count``
    (utils.py:93-102).  Under JAX's promotion rules a Python scalar is weakly
    typed (``weight_decay * p`` forms in the parameter dtype); a NumPy scalar
    or array value is strongly typed float32 (the product forms in float32)."""
    v = weight_decay(count) if callable(weight_decay) else weight_decay
    return float(v), type(v) in (int, float)


def in_transform_decay(u: np.ndarray, p: np.ndarray, wd_step: float, mask=True) -> np.ndarray:
    """utils.py:79-90: ``where(mask, u + wd * p.astype(u.dtype), u)`` with the
    float32 update (the product forms in float32); ``mask`` a boolean or an
    array broadcast against the leaf."""
    uf = np.asarray(u, np.float32)
    dec = (uf + (np.float32(wd_step) * np.asarray(p, np.float32)).astype(np.float32)).astype(np.float32)
    return np.where(np.asarray(mask, dtype=bool), dec, uf).astype(np.float32)


def magma_leaf(g, mu_new, delta, score_prev, keep, tau: float = 2.0):
    """magma.py:86-128 for one leaf, its Bernoulli draw ``keep`` given (the
    reference draws it from JAX's Threefry stream): the cosine between the
    raw gradient and the new first moment, the score EMA
    ``0.9 s + 0.1 sigmoid(cos / tau)``, and ``(keep * s_new) * delta``.
    The three inner products are summed in float64 and rounded to float32
    (JAX's float32 reduction order is not pinned).  Returns
    ``(masked delta, new score)``."""
    gf = np.asarray(g, np.float64).ravel()
    mf = np.asarray(mu_new, np.float32).astype(np.float64).ravel()
    dot = np.float32(np.dot(gf, mf))
    ng = np.float32(np.dot(gf, gf))
    nm = np.float32(np.dot(mf, mf))
    denom = np.maximum(np.float32(np.sqrt(ng)) * np.float32(np.sqrt(nm)), np.float32(1e-12))
    with np.errstate(invalid="ignore", divide="ignore"):
        cos = np.float32(dot / denom)
    cos = np.float32(np.clip(np.nan_to_num(cos, nan=0.0), -1.0, 1.0))
    s_tilde = np.float32(1.0 / (1.0 + np.exp(-np.float64(cos / np.float32(tau)))))
    s_new = np.float32(np.float32(0.9) * np.float32(score_prev) + np.float32(0.1) * s_tilde)
    fac = np.float32(np.float32(1.0 if keep else 0.0) * s_new)
    return (fac * np.asarray(delta, np.float32)).astype(np.float32), s_new


def adam_leaf_update(g, mu, nu, count: int, *, b1=0.9, b2=0.999, eps=1e-8, eps_root=0.0,
                     nesterov=False, dtype=np.float32):
    """adam.py:123-177 (no Magma, in-transform decay 0): returns
    (direction, mu_new, nu_new)."""
    gf = np.asarray(g).astype(dtype)
    b1f, b2f = dtype(b1), dtype(b2)
    mu_new = ((dtype(1.0) - b1f) * gf + b1f * np.asarray(mu, dtype)).astype(dtype)  # utils.py:437-467
    nu_new = (dtype(1.0 - b2) * np.square(gf) + b2f * np.asarray(nu, dtype)).astype(dtype)  # utils.py:470-493
    t = count + 1
    mu_bc = dtype(1.0) - pow32(b1f, t, dtype)
    nu_bc = dtype(1.0) - pow32(b2f, t, dtype)
    if nesterov:  # adam.py:140-159
        mu_bc_next = dtype(1.0) - pow32(b1f, t + 1, dtype)
        mu_hat = b1f * (mu_new / mu_bc_next) + dtype(1.0 - b1) * (gf / mu_bc)
    else:
        mu_hat = mu_new / mu_bc
    nu_hat = nu_new / nu_bc  # adam.py:166
    u = mu_hat / (np.sqrt(nu_hat + dtype(eps_root)) + dtype(eps))  # adam.py:168-177
    return u.astype(dtype), mu_new, nu_new


# --------------------------------------------------------------------------
# The full muon(...) transformation (muon.py:398-486).
# --------------------------------------------------------------------------


class OracleMuon:
    """CPU restatement of ``rollfast.muon(...)`` for the options on the hot
    path (no Magma, float32 state; any preconditioning; ``adaptive``).

    ``params`` / ``grads`` are trees of float32 NumPy arrays; ``param_dtypes``
    (a matching tree of dtype names) tells the decay term which weak-typed
    product the reference forms.
    """

    def __init__(self, learning_rate, ns_coeffs=MUON_NS_COEFFS, ns_steps=5, beta=0.95, eps=1e-8,
                 weight_decay=0.0, weight_decay_mask=None, *, nesterov=True, adam_b1=0.9,
                 adam_b2=0.999, adam_eps=None, adam_eps_root=0.0, adam_weight_decay=None,
                 adam_learning_rate=None, muon_weight_dimension_numbers=None, consistent_rms=None,
                 momentum_accumulator="ema", preconditioning="frobenius", adaptive=False, dtype=np.float32):
        self.lr = learning_rate
        self.preconditioning = preconditioning
        self.adaptive = adaptive
        self.ns_coeffs = ns_coeffs
        self.ns_steps = ns_steps
        self.beta = beta
        self.eps = eps
        self.wd = weight_decay
        self.wd_mask = weight_decay_mask
        self.nesterov = nesterov
        self.b1, self.b2 = adam_b1, adam_b2
        self.adam_eps = eps if adam_eps is None else adam_eps  # muon.py:430-431
        self.adam_eps_root = adam_eps_root
        self.adam_wd = weight_decay if adam_weight_decay is None else adam_weight_decay  # muon.py:432-434
        self.adam_lr = learning_rate if adam_learning_rate is None else adam_learning_rate  # muon.py:428-429
        self.wdn = muon_weight_dimension_numbers
        self.consistent_rms = consistent_rms
        self.acc = momentum_accumulator
        self.dtype = dtype

    def _labels_specs(self, params):
        resolve, labels, _, _ = make_matrix_partition_fns(self.wdn, "muon")
        return labels(params), resolve(params)

    def init(self, params):
        z = lambda p: None if p is None else np.zeros(np.shape(p), self.dtype)
        return {
            "count": 0,
            "mu": tree_map(z, params),
            "ns_coeffs": resolve_ns_coeffs(self.ns_coeffs, self.ns_steps),
            "adam_count": 0,
            "adam_mu": tree_map(z, params),
            "adam_nu": tree_map(z, params),
        }

    def update(self, grads, state, params, param_dtypes=None):
        labels, specs = self._labels_specs(params)
        if param_dtypes is None:
            param_dtypes = tree_map(lambda p: None if p is None else "float32", params)
        wd_mask = self.wd_mask(params) if callable(self.wd_mask) else self.wd_mask
        if wd_mask is None:
            wd_mask = tree_map(lambda p: True, params)
        count = state["count"]
        lr = self.lr(count) if callable(self.lr) else self.lr
        # add_decayed_weights of each branch, a constant or a schedule at the
        # branch's step count (every transform of a chain counts alike).
        mwd, mweak = decay_at(self.wd, count)
        awd, aweak = decay_at(self.adam_wd, state["adam_count"])
        adam_lr = self.adam_lr(state["adam_count"]) if callable(self.adam_lr) else self.adam_lr
        coeffs = state["ns_coeffs"]
        dt = self.dtype

        new_mu = {}
        new_am, new_an = {}, {}

        def leaf(path_label, g, p, mu, am, an, spec, pdt, msk, key):
            if g is None:
                return None
            if path_label == "muon":
                mu_new, d = momentum_runtime(g, mu, count, self.beta, nesterov=self.nesterov,
                                             accumulator=self.acc, dtype=dt)
                new_mu[key] = mu_new
                o = orthogonalize_via_newton_schulz(d, coeffs, self.ns_steps, self.preconditioning, self.eps,
                                                    spec, dtype=dt)
                if self.adaptive:  # muon.py:272-282: <mu_hat, O> O over the whole leaf
                    o = (np.sum(d.astype(dt) * o, dtype=dt) * o).astype(dt)
                u = (o * shape_scale_factor(np.shape(g), spec, self.consistent_rms)).astype(dt)
                if mwd != 0.0 and msk:
                    u = (u + decay_term(p, mwd, pdt if mweak else "float32")).astype(dt)
                return (dt(-lr) * u).astype(dt)
            u, am_new, an_new = adam_leaf_update(g, am, an, state["adam_count"], b1=self.b1,
                                                 b2=self.b2, eps=self.adam_eps,
                                                 eps_root=self.adam_eps_root,
                                                 nesterov=self.nesterov, dtype=dt)
            new_am[key], new_an[key] = am_new, an_new
            if awd != 0.0 and msk:
                u = (u + decay_term(p, awd, pdt if aweak else "float32")).astype(dt)
            return (dt(-adam_lr) * u).astype(dt)

        flat_g = tree_leaves_with_path(grads)
        get = lambda tree, path: _get_path(tree, path)
        updates_flat = {}
        for path, g in flat_g:
            lab = get(labels, path)
            updates_flat[path] = leaf(lab, g, get(params, path), get(state["mu"], path),
                                      get(state["adam_mu"], path), get(state["adam_nu"], path),
                                      get(specs, path), get(param_dtypes, path), bool(get(wd_mask, path)),
                                      path)
        updates = _rebuild(grads, updates_flat)
        mu_tree = _rebuild(state["mu"], {k: v for k, v in new_mu.items()}, keep_missing=True)
        am_tree = _rebuild(state["adam_mu"], new_am, keep_missing=True)
        an_tree = _rebuild(state["adam_nu"], new_an, keep_missing=True)
        return updates, {
            "count": count + 1,
            "mu": mu_tree,
            "ns_coeffs": coeffs,
            "adam_count": state["adam_count"] + 1,
            "adam_mu": am_tree,
            "adam_nu": an_tree,
        }


def _get_path(tree, path):
    for k in path:
        if tree is None or isinstance(tree, MaskedNode):
            return tree
        if isinstance(tree, (bool, np.bool_)):
            return tree
        tree = tree[k]
    return tree


def _rebuild(template, values: dict, prefix=(), keep_missing=False):
    if is_aux_leaf(template):
        return values.get(prefix, template) if keep_missing else values.get(prefix)
    if isinstance(template, dict):
        return {k: _rebuild(v, values, prefix + (k,), keep_missing) for k, v in template.items()}
    if isinstance(template, (list, tuple)) and not hasattr(template, "_fields"):
        return type(template)(_rebuild(v, values, prefix + (i,), keep_missing) for i, v in enumerate(template))
    if prefix in values:
        return values[prefix]
    return template if keep_missing else None
