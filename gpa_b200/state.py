"""Constant-shape recurrent caches, layout-identical to fisalt/GPA's ``gpa.state``.

Field names, order and tensor shapes follow src/gpa/state.py:30-58 so a cache
produced by the b200 backend can be inspected, detached, moved and compared
exactly like a reference cache.  ``detach()`` is explicit, never automatic.
"""
from __future__ import annotations

from dataclasses import dataclass, fields, is_dataclass, replace

from torch import Tensor


def _flatten(node):
    """Split a cache tree into its tensors (depth first, fields in declaration order, the
    order of src/gpa/state.py:16-24) and a function that builds the same tree around a new
    sequence of tensors given in that order.  Ints, None and other leaves are kept."""
    if isinstance(node, Tensor):
        return [node], lambda it: next(it)
    if isinstance(node, tuple) or is_dataclass(node):
        names = None if isinstance(node, tuple) else [f.name for f in fields(node)]
        parts = [_flatten(x) for x in (node if names is None else
                                       (getattr(node, n) for n in names))]
        leaves = [t for sub, _ in parts for t in sub]

        def build(it):
            kids = [make(it) for _, make in parts]
            return tuple(kids) if names is None else replace(node, **dict(zip(names, kids)))
        return leaves, build
    return [], lambda it: node


def _map(value, fn):
    """The same tree with fn applied to every tensor."""
    leaves, build = _flatten(value)
    return build(iter([fn(t) for t in leaves]))


def tensors(value):
    """Every tensor of a cache in field order (src/gpa/state.py:16-24)."""
    return iter(_flatten(value)[0])


@dataclass(frozen=True)
class LevelState:
    inner: Tensor       # A: [B,H,Dk,M]
    outer: Tensor       # B: [B,H,M,Dv]
    count: Tensor       # [B,H,M] soft occurrence counts
    position: Tensor | None = None  # [B,H,Dk,M] additive positional moments (moments mode)


@dataclass(frozen=True)
class RelationState:
    source: int
    target: int
    memory: Tensor      # [B,H,M_source,M_target]


@dataclass(frozen=True)
class ResidualSnapshot:
    inner: Tensor
    outer: Tensor


@dataclass(frozen=True)
class GPAState:
    levels: tuple[LevelState, ...]
    relations: tuple[RelationState, ...]
    position: int = 0
    chunk_size: int = 1
    chunk_offset: int = 0
    frozen: tuple[ResidualSnapshot, ...] | None = None

    def detach(self) -> "GPAState":
        return _map(self, lambda x: x.detach())

    def to(self, *args, **kwargs) -> "GPAState":
        return _map(self, lambda x: x.to(*args, **kwargs))

    def numel(self) -> int:
        return sum(x.numel() for x in tensors(self))
