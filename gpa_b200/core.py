"""``DenseGPA`` on the b200 backend: the reference's module API over the C ABI.

Parameter names, shapes, initial values and their draw order are those of
fisalt/GPA's ``DenseGPA.__init__`` (src/gpa/attention.py:91-144), so
``state_dict`` files move between the two packages and a seeded model is the
same model.  ``forward`` keeps the reference's signature, argument checks and
return values (src/gpa/attention.py:347-414); the whole call -- every lag
block, level, edge and the reader -- runs as one native forward
(``gpa_b200_forward``) and one native backward (``gpa_b200_backward``).
"""
from __future__ import annotations

import math

import torch
from torch import Tensor, nn

from . import _lib
from .config import GPAConfig
from .state import GPAState, LevelState, RelationState, ResidualSnapshot

_DTYPES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
_LEVEL_NAMES = _lib._LEVEL_PARAMS
_SCALAR_NAMES = _lib._SCALAR_PARAMS


def _inverse_softplus(x: float) -> float:
    return math.log(math.expm1(x))


def edges_of(levels: int):
    """Ordered level pairs i != j, row-major (src/gpa/attention.py:122)."""
    return tuple((i, j) for i in range(levels) for j in range(levels) if i != j)


class _Plan:
    """Static description of one native call (shapes, flat tensor layout)."""

    def __init__(self, cfg: GPAConfig, q: Tensor, v: Tensor, state: GPAState):
        self.cfg = cfg
        self.L = len(cfg.slots)
        self.E = self.L * (self.L - 1)
        self.B, self.T, self.H, self.D = q.shape
        self.Dv = v.shape[-1]
        self.offset = state.chunk_offset
        self.new_offset = (state.chunk_offset + self.T) % cfg.chunk_size
        self.fz_in = state.frozen is not None and self.offset != 0
        self.fz_out = self.new_offset != 0
        self.moments = cfg.positional_mode == "moments"
        self.n_params = 7 * self.L + len(_SCALAR_NAMES)
        self.n_mom = self.L if self.moments else 0  # moment states, after the relations
        self.n_state_in = 3 * self.L + self.E + self.n_mom + (2 * self.L if self.fz_in else 0)
        d = _lib.GpaDims()
        d.batch, d.length, d.heads = self.B, self.T, self.H
        d.key_dim, d.value_dim, d.levels = self.D, self.Dv, self.L
        for j, m in enumerate(cfg.slots):
            d.slots[j] = m
        d.chunk_size, d.chunk_offset = cfg.chunk_size, self.offset
        d.input_dtype = _DTYPES[q.dtype]
        d.positional_none = int(cfg.positional_mode == "none")
        d.read_scale, d.query_scale, d.beta_max = cfg.read_scale, cfg.query_scale, cfg.beta_max
        d.reader_mode = (2 if cfg.relation_marginal else 1) if cfg.paper_product_read else 0
        d.positional_moments = int(self.moments)
        d.position = state.position
        self.dims = d

    def state_ref(self, flat, with_frozen: bool) -> _lib.GpaStateRef:
        """GpaStateRef over [A,B,n]*L + R*E (+ P*L with moments) (+ [fA, fB]*L)."""
        s = _lib.GpaStateRef()
        L, E = self.L, self.E
        for j in range(L):
            s.inner[j] = _lib.ptr(flat[3 * j])
            s.outer[j] = _lib.ptr(flat[3 * j + 1])
            s.count[j] = _lib.ptr(flat[3 * j + 2])
        for e in range(E):
            s.relation[e] = _lib.ptr(flat[3 * L + e])
        for j in range(self.n_mom):
            s.moment[j] = _lib.ptr(flat[3 * L + E + j])
        if with_frozen:
            base = 3 * L + E + self.n_mom
            for j in range(L):
                s.frozen_inner[j] = _lib.ptr(flat[base + 2 * j])
                s.frozen_outer[j] = _lib.ptr(flat[base + 2 * j + 1])
        return s

    def params_ref(self, params, cls=_lib.GpaParams):
        p = cls()
        L = self.L
        for j in range(L):
            for n, name in enumerate(_LEVEL_NAMES):
                getattr(p, name)[j] = _lib.ptr(params[7 * j + n])
        for n, name in enumerate(_SCALAR_NAMES):
            t = params[7 * L + n]
            setattr(p, name, _lib.ptr(t) if t.numel() else None)
        return p

    def state_shapes(self, with_frozen: bool):
        B, H, D, Dv = self.B, self.H, self.D, self.Dv
        shapes = []
        for m in self.cfg.slots:
            shapes += [(B, H, D, m), (B, H, m, Dv), (B, H, m)]
        for i, j in edges_of(self.L):
            shapes.append((B, H, self.cfg.slots[i], self.cfg.slots[j]))
        for m in self.cfg.slots[:self.n_mom]:
            shapes.append((B, H, D, m))
        if with_frozen:
            for m in self.cfg.slots:
                shapes += [(B, H, D, m), (B, H, m, Dv)]
        return shapes


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class _DenseGPACore(torch.autograd.Function):
    """One native forward / backward over a whole call (all lag blocks)."""

    @staticmethod
    def forward(ctx, plan: _Plan, q, k, v, *flat):
        lib = _lib.load()
        dev = q.device
        params = flat[:plan.n_params]
        state_in = flat[plan.n_params:]
        out = torch.empty(plan.B, plan.T, plan.H, plan.Dv, device=dev, dtype=v.dtype)
        state_out = [torch.empty(s, device=dev, dtype=torch.float32)
                     for s in plan.state_shapes(plan.fz_out)]
        nbytes = lib.gpa_b200_saved_bytes(plan.dims)
        if not nbytes:
            raise ValueError("gpa_b200_saved_bytes rejected the dimensions")
        saved = torch.empty(nbytes, device=dev, dtype=torch.uint8)
        with torch.cuda.device(dev):
            rc = lib.gpa_b200_forward(plan.dims, plan.params_ref(params), q.data_ptr(),
                                      k.data_ptr(), v.data_ptr(),
                                      plan.state_ref(state_in, plan.fz_in),
                                      plan.state_ref(state_out, plan.fz_out), out.data_ptr(),
                                      saved.data_ptr(), nbytes, _stream(dev))
        _lib.check(rc, "gpa_b200_forward")
        ctx.plan = plan
        ctx.saved_ws = saved
        ctx.in_dtype = q.dtype
        ctx.save_for_backward(*params, *state_in)
        # the workspace has no gradient, and unused outputs get None instead of a zero tensor
        # (a materialized zero gradient of the workspace would be as large as the workspace)
        ctx.mark_non_differentiable(saved)
        ctx.set_materialize_grads(False)
        return (out, *state_out, saved)

    @staticmethod
    def backward(ctx, dout, *dstate_and_ws):
        dstate = dstate_and_ws[:-1]
        lib = _lib.load()
        plan = ctx.plan
        tensors = ctx.saved_tensors
        params = tensors[:plan.n_params]
        state_in = tensors[plan.n_params:]
        dev = ctx.saved_ws.device
        if dout is None:
            dout = torch.zeros(plan.B, plan.T, plan.H, plan.Dv, device=dev, dtype=ctx.in_dtype)
        dout = dout.contiguous().to(ctx.in_dtype)
        dstate = [None if g is None else g.contiguous().float() for g in dstate]
        if plan.fz_out:  # frozen-snapshot gradients are consumed in (inner, outer) pairs
            base = 3 * plan.L + plan.E + plan.n_mom
            shapes = plan.state_shapes(True)
            for i in range(base, len(dstate)):
                if dstate[i] is None:
                    dstate[i] = torch.zeros(shapes[i], device=dev, dtype=torch.float32)
        dq = torch.empty(plan.B, plan.T, plan.H, plan.D, device=dev, dtype=ctx.in_dtype)
        dk = torch.empty_like(dq)
        dv = torch.empty(plan.B, plan.T, plan.H, plan.Dv, device=dev, dtype=ctx.in_dtype)
        dparams = [torch.zeros(p.shape, device=dev, dtype=torch.float32) for p in params]
        dstate_in = [torch.empty(s.shape, device=dev, dtype=torch.float32) for s in state_in]
        nbytes = lib.gpa_b200_scratch_bytes(plan.dims)
        scratch = torch.empty(nbytes, device=dev, dtype=torch.uint8)
        with torch.cuda.device(dev):
            rc = lib.gpa_b200_backward(plan.dims, plan.params_ref(params),
                                       plan.state_ref(state_in, plan.fz_in),
                                       ctx.saved_ws.data_ptr(), dout.data_ptr(),
                                       plan.state_ref(dstate, plan.fz_out), dq.data_ptr(),
                                       dk.data_ptr(), dv.data_ptr(),
                                       plan.state_ref(dstate_in, plan.fz_in),
                                       plan.params_ref(dparams, _lib.GpaParamGrads),
                                       scratch.data_ptr(), nbytes, _stream(dev))
        _lib.check(rc, "gpa_b200_backward")
        del scratch
        ctx.saved_ws = None
        dparams = [g.to(p.dtype) for g, p in zip(dparams, params)]
        if not plan.moments:  # moment_gain is unused without positional moments
            dparams[-1] = None
        return (None, dq, dk, dv, *dparams, *dstate_in)


class DenseGPA(nn.Module):
    """Projected Q/K/V -> output, cache.  Inputs [B,T,H,D], output [B,T,H,Dv].

    Drop-in for fisalt/GPA's ``gpa.DenseGPA`` (src/gpa/attention.py:82-414) on
    CUDA devices of compute capability 10.0 (B200).
    """

    def __init__(self, config: GPAConfig):
        super().__init__()
        self.config = config
        h, d, dv = config.heads, config.key_dim, config.value_dim
        for name in ("center", "inner_prefix", "outer_prefix", "route_weight", "query_weight",
                     "route_up", "route_down", "gate_weight", "gate_bias"):
            setattr(self, name, nn.ParameterList())
        gate_bias = torch.tensor([_inverse_softplus(config.decay_init),
                                  math.log(config.beta_init / (config.beta_max - config.beta_init))] * 2)
        for m in config.slots:
            # same draws, same order as the reference initialisation
            self.center.append(nn.Parameter(torch.randn(h, m, d) / math.sqrt(d)))
            self.inner_prefix.append(nn.Parameter(torch.randn(h, d, m) * .002))
            self.outer_prefix.append(nn.Parameter(torch.randn(h, m, dv) * .002))
            self.route_weight.append(nn.Parameter(torch.eye(m).repeat(h, 1, 1)))
            self.query_weight.append(nn.Parameter(torch.randn(h, d, m) / math.sqrt(d)))
            self.route_up.append(nn.Parameter(torch.randn(h, m, 2 * m) / math.sqrt(m)))
            self.route_down.append(nn.Parameter(torch.randn(h, 2 * m, m) * .002))
            self.gate_weight.append(nn.Parameter(torch.zeros(h, d, 4)))
            self.gate_bias.append(nn.Parameter(gate_bias.repeat(h, 1)))
        levels = len(config.slots)
        self.residual_raw = nn.Parameter(torch.zeros(levels, h, 2))
        self.count_gain_raw = nn.Parameter(torch.full((levels, h), _inverse_softplus(.1)))
        self.moment_gain = nn.Parameter(torch.full((levels, h), .1))
        self.route_mlp_gain = nn.Parameter(torch.full((levels, h), .1))
        self.output_logits = nn.Parameter(torch.zeros(levels, h))
        self.edges = edges_of(levels)
        self.register_buffer("_edge_source", torch.tensor([i for i, _ in self.edges], dtype=torch.long),
                             persistent=False)
        self.register_buffer("_edge_target", torch.tensor([j for _, j in self.edges], dtype=torch.long),
                             persistent=False)
        self.relation_prefix = nn.ParameterList([
            nn.Parameter(torch.zeros(h, config.slots[i], config.slots[j])) for i, j in self.edges])
        self.edge_logits = nn.Parameter(torch.zeros(len(self.edges), h))
        self.relation_gain = nn.Parameter(torch.full((levels, h), .1))
        self.relation_decay_raw = nn.Parameter(torch.full(
            (len(self.edges), h), _inverse_softplus(config.relation_decay_init)))
        rb = math.log(config.relation_beta_init / (1 - config.relation_beta_init))
        self.relation_beta_raw = nn.Parameter(torch.full((len(self.edges), h), rb))

    # ---------------------------------------------------------------- cache
    def initial_state(self, batch: int, *, device=None, dtype=None) -> GPAState:
        """Learned prefixes broadcast over the batch, zero counts (attention.py:146-159)."""
        ref = self.center[0]
        device = ref.device if device is None else device
        dtype = ref.dtype if dtype is None else dtype
        work = torch.float64 if dtype == torch.float64 else torch.float32
        expand = lambda p: p.to(device=device, dtype=work).unsqueeze(0).expand(batch, *p.shape)
        moments = self.config.positional_mode == "moments"
        h, d = self.config.heads, self.config.key_dim
        levels = tuple(LevelState(expand(a), expand(b),
                                  torch.zeros(batch, h, m, device=device, dtype=work),
                                  torch.zeros(batch, h, d, m, device=device, dtype=work)
                                  if moments else None)
                       for m, a, b in zip(self.config.slots, self.inner_prefix, self.outer_prefix))
        relations = tuple(RelationState(i, j, expand(p))
                          for (i, j), p in zip(self.edges, self.relation_prefix))
        return GPAState(levels, relations, chunk_size=self.config.chunk_size)

    def _flat_params(self):
        out = []
        for j in range(len(self.config.slots)):
            for name in _LEVEL_NAMES:
                out.append(getattr(self, name)[j])
        for name in _SCALAR_NAMES:
            out.append(getattr(self, name))
        return [p if p.dtype == torch.float32 and p.is_contiguous() else p.float().contiguous()
                for p in out]

    # -------------------------------------------------------------- forward
    def forward(self, q: Tensor, k: Tensor, v: Tensor, state: GPAState | None = None, *,
                position_ids: Tensor | None = None, return_diagnostics: bool = False,
                control_input=None):
        cfg = self.config
        if q.ndim != 4 or q.shape != k.shape or q.shape[:3] != v.shape[:3]:
            raise ValueError("expected Q,K [B,T,H,Dk], V [B,T,H,Dv]")
        if q.shape[2:] != (cfg.heads, cfg.key_dim) or v.shape[-1] != cfg.value_dim:
            raise ValueError("input heads/dimensions do not match GPAConfig")
        if q.device != k.device or q.device != v.device or q.dtype != k.dtype or q.dtype != v.dtype:
            raise ValueError("Q,K,V must share device and floating dtype")
        if control_input is not None:
            raise ValueError("full hidden controls need control_dim, which the b200 backend does not implement")
        if not q.is_cuda:
            raise ValueError("the b200 backend needs CUDA tensors (B200, sm_100a)")
        if q.dtype not in _DTYPES:
            raise ValueError("the b200 backend computes float32, bfloat16 or float16 inputs")
        if state is None:
            state = self.initial_state(q.shape[0], device=q.device, dtype=q.dtype)
        if state.chunk_size != cfg.chunk_size:
            raise ValueError("cannot switch cache between recurrent and lagged chunk semantics")
        if len(state.levels) != len(cfg.slots) or tuple((s.source, s.target) for s in state.relations) != self.edges:
            raise ValueError("cache topology does not match this model")
        default_ids = position_ids is None
        if position_ids is None:
            position_ids = torch.arange(state.position, state.position + q.shape[1], device=q.device)
        if position_ids.shape not in ((q.shape[1],), (q.shape[0], q.shape[1])):
            raise ValueError("position_ids must be [T] or [B,T]")
        if cfg.positional_mode == "moments" and not default_ids and not torch.equal(
                position_ids.to(torch.long).expand(q.shape[0], -1).cpu(),
                torch.arange(state.position, state.position + q.shape[1]).expand(q.shape[0], -1)):
            raise ValueError("positional moments on the b200 backend rotate by the cache position; "
                             "custom position_ids are not implemented")
        if q.shape[1] == 0:
            output = v.new_empty(v.shape)
            if return_diagnostics:
                routes = tuple(q.new_empty(q.shape[:3] + (m,)) for m in cfg.slots)
                return output, state, {"routes": routes, "edges": self.edges,
                                       "state_elements": state.numel(), "position": state.position}
            return output, state
        plan = _Plan(cfg, q, v, state)
        flat_state = []
        for lv in state.levels:
            flat_state += [lv.inner, lv.outer, lv.count]
        flat_state += [r.memory for r in state.relations]
        if plan.moments:
            if any(lv.position is None for lv in state.levels):
                raise ValueError("positional moments need the moment states of the cache")
            flat_state += [lv.position for lv in state.levels]
        if plan.fz_in:
            for snap in state.frozen:
                flat_state += [snap.inner, snap.outer]
        flat_state = [t.float().contiguous() for t in flat_state]
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        outs = _DenseGPACore.apply(plan, q, k, v, *self._flat_params(), *flat_state)
        output, st, saved = outs[0], outs[1:-1], outs[-1]
        L = plan.L
        moms = [st[3 * L + plan.E + j] if plan.moments else None for j in range(L)]
        levels = tuple(LevelState(st[3 * j], st[3 * j + 1], st[3 * j + 2], moms[j]) for j in range(L))
        relations = tuple(RelationState(i, j, st[3 * L + e]) for e, (i, j) in enumerate(self.edges))
        frozen = None
        if plan.fz_out:
            base = 3 * L + plan.E + plan.n_mom
            frozen = tuple(ResidualSnapshot(st[base + 2 * j], st[base + 2 * j + 1]) for j in range(L))
        new = GPAState(levels, relations, state.position + q.shape[1], cfg.chunk_size,
                       plan.new_offset, frozen)
        if return_diagnostics:
            routes = _routes(plan, saved, q.dtype)
            return output, new, {"routes": routes, "edges": self.edges,
                                 "state_elements": new.numel(), "position": new.position}
        return output, new


def _routes(plan: _Plan, saved: Tensor, dtype) -> tuple:
    """Per-level post-MLP routes [B,T,H,M] of a call (detached diagnostics)."""
    lib = _lib.load()
    outs = tuple(torch.empty(plan.B, plan.T, plan.H, m, device=saved.device, dtype=dtype)
                 for m in plan.cfg.slots)
    arr = (_lib.c_void_p * _lib.MAX_LEVELS)(*[o.data_ptr() for o in outs])
    with torch.cuda.device(saved.device):
        rc = lib.gpa_b200_routes(plan.dims, saved.data_ptr(), arr, _stream(saved.device))
    _lib.check(rc, "gpa_b200_routes")
    return outs
