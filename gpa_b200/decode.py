"""In-place one-token decode of a DenseGPA cache on B200 (``gpa_b200_step``).

``DenseGPA.forward`` with a one-token input is the reference's decode call
(src/gpa/attention.py:347-414): it returns a new ``GPAState`` each time.  For
serving, :class:`DecodeSession` keeps the cache in fixed fp32 buffers that one
fused kernel per step (a single launch) updates in place, with the lag-block offset in device
memory, so a step allocates nothing, never synchronizes with the host and can be
captured once in a CUDA graph (:meth:`DecodeSession.capture`) and replayed.  Its
outputs and caches are those of the one-token ``forward`` calls it replaces
(lag-block caches, ``chunk_size >= 2``).
"""
from __future__ import annotations

import torch
from torch import Tensor

from . import _lib
from .core import DenseGPA, _Plan, _stream
from .state import GPAState, LevelState, RelationState, ResidualSnapshot


class DecodeSession:
    """One-token decode steps of ``model`` from ``state``, cache updated in place.

    ``state`` is copied into the session's own buffers (fp32, contiguous); the
    session's :attr:`state` is a ``GPAState`` view of them.  Inputs of every step
    are ``q, k [B, 1, H, Dk]`` and ``v [B, 1, H, Dv]`` in the dtype given here.
    """

    def __init__(self, model: DenseGPA, state: GPAState, dtype: torch.dtype = torch.bfloat16):
        cfg = model.config
        if cfg.chunk_size < 2:
            raise ValueError("DecodeSession needs lag-block caches (chunk_size >= 2)")
        self.model = model
        self.dtype = dtype
        dev = state.levels[0].inner.device
        B, H = state.levels[0].inner.shape[:2]
        D, Dv = model.config.key_dim, model.config.value_dim
        meta_q = torch.empty(B, 1, H, D, device="meta", dtype=dtype)
        meta_v = torch.empty(B, 1, H, Dv, device="meta", dtype=dtype)
        self._plan = _Plan(cfg, meta_q, meta_v, state)
        self._shape_q, self._shape_v = (B, 1, H, D), (B, 1, H, Dv)
        flat = []
        for lv in state.levels:
            flat += [lv.inner, lv.outer, lv.count]
        flat += [r.memory for r in state.relations]
        if self._plan.moments:
            flat += [lv.position for lv in state.levels]
        self._flat = [t.detach().to(dev, torch.float32).clone().contiguous() for t in flat]
        shapes = self._plan.state_shapes(True)
        base = len(self._flat)
        if state.frozen is not None and state.chunk_offset != 0:
            for snap in state.frozen:
                self._flat += [snap.inner.detach().to(dev, torch.float32).clone().contiguous(),
                               snap.outer.detach().to(dev, torch.float32).clone().contiguous()]
        else:  # written by the step that opens the next lag block
            self._flat += [torch.zeros(s, device=dev, dtype=torch.float32) for s in shapes[base:]]
        self._edges = model.edges
        # [chunk offset, completion counter of the step kernel (0 between steps), position]
        self._offset = torch.tensor([state.chunk_offset, 0, state.position], device=dev,
                                    dtype=torch.int32)
        self.offset = self._offset[:1]
        self.position = state.position
        self._graph = None

    # ------------------------------------------------------------------ steps
    def step(self, q: Tensor, k: Tensor, v: Tensor, out: Tensor | None = None) -> Tensor:
        """One token: returns ``out [B, 1, H, Dv]`` and advances the cache in place."""
        for x, shape in ((q, self._shape_q), (k, self._shape_q), (v, self._shape_v)):
            if tuple(x.shape) != shape or x.dtype != self.dtype or not x.is_cuda:
                raise ValueError(f"decode inputs must be CUDA {self.dtype} tensors of shape {shape}")
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        if out is None:
            out = torch.empty(self._shape_v, device=q.device, dtype=self.dtype)
        lib = _lib.load()
        plan = self._plan
        params = self.model._flat_params()
        with torch.cuda.device(q.device):
            rc = lib.gpa_b200_step(plan.dims, plan.params_ref(params), q.data_ptr(), k.data_ptr(),
                                   v.data_ptr(), plan.state_ref(self._flat, True),
                                   self._offset.data_ptr(), out.data_ptr(), _stream(q.device))
        _lib.check(rc, "gpa_b200_step")
        self.position += 1
        return out

    def capture(self, q: Tensor, k: Tensor, v: Tensor) -> Tensor:
        """Capture one step on the static inputs ``q, k, v`` in a CUDA graph; returns the
        static output.  :meth:`replay` then runs a step on whatever ``q, k, v`` hold."""
        self._static = (q, k, v, torch.empty(self._shape_v, device=q.device, dtype=self.dtype))
        rewind = [t.clone() for t in self._flat] + [self._offset.clone()]
        self.step(*self._static[:3], out=self._static[3])  # warm-up (library load, attributes)
        torch.cuda.synchronize(q.device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):  # recorded, not run
            self.step(*self._static[:3], out=self._static[3])
        for t, r in zip(self._flat + [self._offset], rewind):  # undo the warm-up step
            t.copy_(r)
        self.position -= 2
        self._graph = graph
        return self._static[3]

    def replay(self) -> Tensor:
        """One step through the captured graph (inputs: the static tensors given to capture)."""
        if self._graph is None:
            raise RuntimeError("capture() first")
        self._graph.replay()
        self.position += 1
        return self._static[3]

    # ------------------------------------------------------------------ state
    @property
    def state(self) -> GPAState:
        """The cache as a ``GPAState`` over the session's buffers (reads the device offset)."""
        L, E, nm = self._plan.L, self._plan.E, self._plan.n_mom
        f = self._flat
        levels = tuple(LevelState(f[3 * j], f[3 * j + 1], f[3 * j + 2],
                                  f[3 * L + E + j] if nm else None) for j in range(L))
        rel = tuple(RelationState(i, j, f[3 * L + e]) for e, (i, j) in enumerate(self._edges))
        off = int(self.offset.item())
        frozen = None
        if off != 0:
            base = 3 * L + E + nm
            frozen = tuple(ResidualSnapshot(f[base + 2 * j], f[base + 2 * j + 1]) for j in range(L))
        return GPAState(levels, rel, self.position, self.model.config.chunk_size, off, frozen)
