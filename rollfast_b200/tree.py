"""Minimal PyTree utilities with JAX semantics for the containers the
reference's trees use (dict, list, tuple, NamedTuple) and its auxiliary
leaves (``None`` and :class:`MaskedNode`, utils.py:13-22).

As in ``jax.tree``: ``None`` and ``MaskedNode()`` are nodes without children,
so ``tree_map`` passes them through unless ``is_leaf`` claims them.
"""

from __future__ import annotations

from typing import Any, Callable, NamedTuple


class MaskedNode(NamedTuple):
    """Stand-in for a leaf owned by another partition branch
    (optax.transforms._masking.MaskedNode)."""


def is_aux_leaf(x: Any) -> bool:
    """utils.py:13-14."""
    return x is None or isinstance(x, MaskedNode)


def _is_namedtuple(x: Any) -> bool:
    return isinstance(x, tuple) and hasattr(x, "_fields")


class _Node:
    __slots__ = ("kind", "meta", "children")

    def __init__(self, kind, meta, children):
        self.kind, self.meta, self.children = kind, meta, children


_LEAF = _Node("leaf", None, ())


def tree_flatten(tree: Any, is_leaf: Callable[[Any], bool] | None = None):
    leaves: list = []

    def rec(x):
        if is_leaf is not None and is_leaf(x):
            leaves.append(x)
            return _LEAF
        if x is None:
            return _Node("none", None, ())
        if isinstance(x, MaskedNode):
            return _Node("masked", None, ())
        if isinstance(x, dict):
            keys = list(x.keys())
            return _Node("dict", keys, [rec(x[k]) for k in keys])
        if _is_namedtuple(x):
            return _Node("namedtuple", type(x), [rec(v) for v in x])
        if isinstance(x, (list, tuple)):
            return _Node(type(x), None, [rec(v) for v in x])
        leaves.append(x)
        return _LEAF

    return leaves, rec(tree)


def tree_unflatten(treedef: _Node, leaves) -> Any:
    it = iter(leaves)

    def rec(n: _Node):
        if n is _LEAF or n.kind == "leaf":
            return next(it)
        if n.kind == "none":
            return None
        if n.kind == "masked":
            return MaskedNode()
        if n.kind == "dict":
            return {k: rec(c) for k, c in zip(n.meta, n.children)}
        if n.kind == "namedtuple":
            return n.meta(*[rec(c) for c in n.children])
        return n.kind(rec(c) for c in n.children)

    return rec(treedef)


def tree_leaves(tree: Any, is_leaf=None) -> list:
    return tree_flatten(tree, is_leaf)[0]


def tree_map(fn: Callable, tree: Any, *rest: Any, is_leaf=None) -> Any:
    """``jax.tree.map``: ``rest`` trees must have ``tree``'s structure (or be
    deeper at its leaves)."""
    leaves, treedef = tree_flatten(tree, is_leaf)
    others = [_flatten_up_to(treedef, r) for r in rest]
    return tree_unflatten(treedef, [fn(*xs) for xs in zip(leaves, *others)])


def _flatten_up_to(treedef: _Node, tree: Any) -> list:
    out: list = []

    def rec(n: _Node, x):
        if n is _LEAF or n.kind == "leaf":
            out.append(x)
            return
        if n.kind in ("none", "masked"):
            return
        if n.kind == "dict":
            if not isinstance(x, dict) or set(x.keys()) != set(n.meta):
                raise ValueError("tree structures do not match")
            for k, c in zip(n.meta, n.children):
                rec(c, x[k])
            return
        if not isinstance(x, (list, tuple)) or len(x) != len(n.children):
            raise ValueError("tree structures do not match")
        for c, v in zip(n.children, x):
            rec(c, v)

    rec(treedef, tree)
    return out


def tree_structure_equal(a: Any, b: Any) -> bool:
    try:
        _flatten_up_to(tree_flatten(a)[1], b)
        return True
    except ValueError:
        return False
