"""Constant-shape recurrent caches, layout-identical to fisalt/GPA's ``gpa.state``.

Field names, order and tensor shapes follow src/gpa/state.py:30-58 so a cache
produced by the b200 backend can be inspected, detached, moved and compared
exactly like a reference cache.  ``detach()`` is explicit, never automatic.
"""
from __future__ import annotations

from dataclasses import dataclass, fields, is_dataclass
from typing import Any

from torch import Tensor


def _map(value: Any, fn):
    if isinstance(value, Tensor):
        return fn(value)
    if isinstance(value, tuple):
        return tuple(_map(x, fn) for x in value)
    if is_dataclass(value):
        return type(value)(**{f.name: _map(getattr(value, f.name), fn) for f in fields(value)})
    return value


def tensors(value):
    """Every tensor of a cache in field order (src/gpa/state.py:16-24)."""
    if isinstance(value, Tensor):
        yield value
    elif isinstance(value, tuple):
        for x in value:
            yield from tensors(x)
    elif is_dataclass(value):
        for f in fields(value):
            yield from tensors(getattr(value, f.name))


@dataclass(frozen=True)
class LevelState:
    inner: Tensor       # A: [B,H,Dk,M]
    outer: Tensor       # B: [B,H,M,Dv]
    count: Tensor       # [B,H,M] soft occurrence counts
    position: Tensor | None = None  # positional moments (not used by the b200 backend)


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
