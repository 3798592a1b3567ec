"""Matrix routing and reshapes (restates src/rollfast/optim/dimension_numbers.py).

Decides which leaves go to Muon and which to the AdamW fallback, and maps a
leaf to the ``(batch, reduction, output)`` matrix layout the kernels consume.
Host-side only.
"""

from __future__ import annotations

import math
from typing import Any, Callable, NamedTuple, Sequence

import torch

from .tree import MaskedNode, is_aux_leaf, tree_map


class MatrixDimensionNumbers(NamedTuple):
    """dimension_numbers.py:15-24."""

    reduction_axis: Sequence[int] | int = 0
    output_axis: Sequence[int] | int = 1


MuonDimensionNumbers = MatrixDimensionNumbers
WeightDimNumOrFn = Any


class MatrixPartitionFns(NamedTuple):
    """dimension_numbers.py:39-45."""

    resolve: Callable
    labels: Callable
    masked_specs: Callable
    default_mask: Callable


def _is_dimension_numbers_leaf(x: Any) -> bool:
    """dimension_numbers.py:48-49."""
    return x is None or isinstance(x, (MatrixDimensionNumbers, MaskedNode))


def _is_array_like_leaf(x: Any) -> bool:
    return hasattr(x, "shape") and hasattr(x, "dtype")


def _has_matrix_spec(d: Any) -> bool:
    return d is not None and not isinstance(d, MaskedNode)


def _validate_matrix_operand(x: Any, dim_nums, transform_name: str) -> None:
    """dimension_numbers.py:60-79."""
    if x is None or isinstance(x, MaskedNode):
        return
    if dim_nums is None or isinstance(dim_nums, MaskedNode):
        raise ValueError(
            f"`{transform_name}` only supports leaves with matrix dimension specs. "
            "Use the public wrapper for Adam fallback leaves, or pass a "
            "`weight_dimension_numbers` tree that marks every updated leaf."
        )
    if x.dtype.is_complex:
        raise ValueError(
            f"`{transform_name}` does not support complex matrix leaves. Route "
            "complex parameters to an Adam fallback branch or convert them to a "
            "real-valued representation before using matrix optimizers."
        )


def _get_dimension_numbers(weight_dimension_numbers, params):
    """dimension_numbers.py:82-116."""
    if weight_dimension_numbers is None:
        return tree_map(
            lambda x: None
            if is_aux_leaf(x)
            else (MatrixDimensionNumbers() if hasattr(x, "ndim") and x.ndim == 2 else None),
            params,
            is_leaf=is_aux_leaf,
        )
    if callable(weight_dimension_numbers) and not isinstance(weight_dimension_numbers, MatrixDimensionNumbers):
        return weight_dimension_numbers(params)
    if isinstance(weight_dimension_numbers, MatrixDimensionNumbers):
        if _is_array_like_leaf(params):
            return weight_dimension_numbers
        raise ValueError(
            "A bare MatrixDimensionNumbers can only be used with a single array "
            "leaf. For PyTree params, pass a matching PyTree of specs/None or a "
            "callable dimension-spec function; bare specs are not broadcast."
        )
    return weight_dimension_numbers


def _resolve_update_dimension_numbers(weight_dimension_numbers, *, params, updates, transform_name: str):
    """dimension_numbers.py:119-134."""
    if params is None:
        if callable(weight_dimension_numbers) and not isinstance(weight_dimension_numbers, MatrixDimensionNumbers):
            raise ValueError(
                f"`params` must be provided to `{transform_name}` when "
                "`weight_dimension_numbers` is callable."
            )
        return _get_dimension_numbers(weight_dimension_numbers, updates)
    return _get_dimension_numbers(weight_dimension_numbers, params)


def _mask_dimension_numbers(dim_nums_tree):
    """dimension_numbers.py:137-143."""
    return tree_map(lambda d: d if d is not None else MaskedNode(), dim_nums_tree,
                    is_leaf=_is_dimension_numbers_leaf)


def _make_matrix_labels(dim_nums_tree, params, matrix_label: str, fallback_label: str = "adam"):
    """dimension_numbers.py:146-162."""
    return tree_map(
        lambda d, p: None if p is None else (matrix_label if _has_matrix_spec(d) else fallback_label),
        dim_nums_tree,
        params,
        is_leaf=_is_dimension_numbers_leaf,
    )


def _make_dimension_numbers_mask(dim_nums_tree, params):
    """dimension_numbers.py:165-179."""
    return tree_map(
        lambda d, p: False if (p is None or isinstance(p, MaskedNode)) else _has_matrix_spec(d),
        dim_nums_tree,
        params,
        is_leaf=_is_dimension_numbers_leaf,
    )


def _make_matrix_partition_fns(weight_dimension_numbers, matrix_label: str, fallback_label: str = "adam"):
    """dimension_numbers.py:182-215."""

    def resolve(params):
        return _get_dimension_numbers(weight_dimension_numbers, params)

    def labels(params):
        return _make_matrix_labels(resolve(params), params, matrix_label, fallback_label)

    def masked_specs(params):
        return _mask_dimension_numbers(resolve(params))

    def default_mask(params):
        return _make_dimension_numbers_mask(resolve(params), params)

    return MatrixPartitionFns(resolve, labels, masked_specs, default_mask)


def _normalize_axis_group(ndim: int, axes, name: str) -> tuple[int, ...]:
    """dimension_numbers.py:288-309."""
    axes_tuple = (axes,) if isinstance(axes, int) else tuple(axes)
    if not axes_tuple:
        raise ValueError(f"{name} must not be empty.")
    out = []
    for axis in axes_tuple:
        if axis < -ndim or axis >= ndim:
            raise ValueError(f"{name} axis {axis} is out of bounds for rank-{ndim} parameter.")
        out.append(axis if axis >= 0 else axis + ndim)
    t = tuple(out)
    if len(set(t)) != len(t):
        raise ValueError(f"{name} contains duplicate axes: {axes_tuple}.")
    return t


def _normalize_axes(shape, dim_nums: MatrixDimensionNumbers):
    """dimension_numbers.py:279-285."""
    nd = len(shape)
    return (
        _normalize_axis_group(nd, dim_nums.reduction_axis, "reduction_axis"),
        _normalize_axis_group(nd, dim_nums.output_axis, "output_axis"),
    )


class MatrixLayout(NamedTuple):
    """A leaf's ``(batch, reduction, output)`` view (dimension_numbers.py:312-359)."""

    perm: tuple[int, ...]        # forward transpose
    inv_perm: tuple[int, ...]
    flat_shape: tuple[int, int, int]
    unflat_shape: tuple[int, ...]

    @property
    def is_identity(self) -> bool:
        return self.perm == tuple(range(len(self.perm)))


def _compute_matrix_layout(shape, dtype: torch.dtype, dim_nums: MatrixDimensionNumbers) -> MatrixLayout:
    """dimension_numbers.py:312-359."""
    if dtype.is_complex:
        raise ValueError(
            "Matrix optimizers do not support complex matrix leaves. Route complex "
            "parameters to an Adam fallback branch or convert them to a real-valued "
            "representation before using matrix optimizers."
        )
    shape = tuple(shape)
    if len(shape) < 2:
        raise ValueError(f"Matrix-optimized parameters must have rank >= 2, got x.ndim={len(shape)}.")
    red, out = _normalize_axes(shape, dim_nums)
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
    return MatrixLayout(perm, tuple(inv), flat, unflat)


def _compute_matrix_reshape(x: torch.Tensor, dim_nums: MatrixDimensionNumbers):
    """dimension_numbers.py:312-359: forward / inverse reshapes."""
    lay = _compute_matrix_layout(x.shape, x.dtype, dim_nums)
    fwd = lambda t: t.permute(lay.perm).reshape(lay.flat_shape)
    bwd = lambda t: t.reshape(lay.unflat_shape).permute(lay.inv_perm)
    return fwd, bwd


__all__ = [
    "MatrixDimensionNumbers",
    "MuonDimensionNumbers",
    "WeightDimNumOrFn",
]
