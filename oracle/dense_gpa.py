"""CPU restatement of the fisalt/GPA DenseGPA attention core -- TEST INFRASTRUCTURE.

This module is the parity checker for the ``b200`` backend and nothing else.
Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it; the product package
``gpa_b200`` never does, and must fail loudly when its CUDA library is absent.

It restates the reference's ``backend="torch"`` algorithm (package
``gpa-attention`` v0.4.0) for the default flag set the b200 backend accepts:
``positional_mode`` in {"gated", "none", "moments"}, linear slot features, no RSA update,
no control input, no quadratic features, no balanced bridge, fixed read scale;
the reader in its centred-tanh form or the product form (``paper_product_read``,
optionally ``relation_marginal``).  Every function cites the reference lines it follows
(paths are relative to the reference project root).  Dtype handling follows
the reference exactly: states are float32 (float64 for float64 inputs) and the
activation dtype is rounded at the same points, so the restatement can be
pinned against golden vectors produced by the reference itself
(``tests/golden``).

Parameters are passed as a plain ``{name: tensor}`` mapping with the
reference's ``state_dict`` keys (``center.0``, ``inner_prefix.0``, ...,
``relation_prefix.<edge>``, ``edge_logits`` ...), so any model whose
``state_dict`` matches the reference can be checked.
"""
from __future__ import annotations

from dataclasses import dataclass
import math

import torch
import torch.nn.functional as F

__all__ = ["OracleConfig", "OracleState", "edges_of", "initial_state", "forward",
           "init_parameters", "unit", "gdn_scan", "tensors_of"]


@dataclass(frozen=True)
class OracleConfig:
    """The subset of ``GPAConfig`` (src/gpa/attention.py:17-43) the core uses."""
    heads: int
    key_dim: int
    value_dim: int
    slots: tuple
    chunk_size: int = 1
    positional_mode: str = "gated"
    query_scale: float = 1 / 16
    beta_init: float = .1
    beta_max: float = .9
    decay_init: float = .001
    relation_beta_init: float = .6
    relation_decay_init: float = .0001
    read_scale: float = 1.
    paper_product_read: bool = False
    relation_marginal: bool = False


@dataclass(frozen=True)
class OracleState:
    """Mirror of ``GPAState`` (src/gpa/state.py:30-58) with plain tuples.

    levels: tuple of (inner A [B,H,D,M], outer B [B,H,M,Dv], count [B,H,M][, moments
            P [B,H,D,M] when positional_mode is "moments"])
    relations: tuple of R [B,H,M_i,M_j] in edge order
    frozen: tuple of (A, B) snapshots or None
    """
    levels: tuple
    relations: tuple
    position: int = 0
    chunk_size: int = 1
    chunk_offset: int = 0
    frozen: tuple | None = None


def tensors_of(state: OracleState):
    """Flatten in the reference's ``tensors()`` order (src/gpa/state.py:16-24):
    per level inner, outer, count[, moments]; per relation memory; per frozen level inner,
    outer."""
    out = []
    for lv in state.levels:
        out += list(lv)
    out += list(state.relations)
    if state.frozen is not None:
        for a, b in state.frozen:
            out += [a, b]
    return out


def edges_of(levels: int):
    """Ordered level pairs i != j, row-major (src/gpa/attention.py:122)."""
    return tuple((i, j) for i in range(levels) for j in range(levels) if i != j)


def _work_dtype(x: torch.Tensor) -> torch.dtype:
    """src/gpa/ops.py:10-11."""
    return torch.float64 if x.dtype == torch.float64 else torch.float32


def unit(x: torch.Tensor) -> torch.Tensor:
    """x / max(||x||, 1e-6) in the work dtype, cast back (src/gpa/ops.py:14-17)."""
    w = x.to(_work_dtype(x))
    return (w / w.norm(dim=-1, keepdim=True).clamp_min(1e-6)).to(x.dtype)


def _softplus(x):
    return F.softplus(x)


def _inv_softplus(x: float) -> float:
    return math.log(math.expm1(x))


# --------------------------------------------------------------------------
# Parameters (src/gpa/attention.py:91-144)
# --------------------------------------------------------------------------

def init_parameters(cfg: OracleConfig, generator: torch.Generator | None = None) -> dict:
    """Draw parameters with the reference's shapes, initial values and draw order.

    The draw order matters only for reproducing a reference model from a seed:
    per level center, inner_prefix, outer_prefix, route_weight (identity),
    query_weight, route_up, route_down, gate_weight (zeros), gate_bias, then
    the level scalars, relation prefixes (zeros) and edge scalars
    (src/gpa/attention.py:104-135).
    """
    h, d, dv = cfg.heads, cfg.key_dim, cfg.value_dim
    levels = len(cfg.slots)
    rnd = lambda *s: torch.randn(*s, generator=generator)
    p = {}
    for j, m in enumerate(cfg.slots):
        p[f"center.{j}"] = rnd(h, m, d) / math.sqrt(d)
        p[f"inner_prefix.{j}"] = rnd(h, d, m) * .002
        p[f"outer_prefix.{j}"] = rnd(h, m, dv) * .002
        p[f"route_weight.{j}"] = torch.eye(m).repeat(h, 1, 1)
        p[f"query_weight.{j}"] = rnd(h, d, m) / math.sqrt(d)
        p[f"route_up.{j}"] = rnd(h, m, 2 * m) / math.sqrt(m)
        p[f"route_down.{j}"] = rnd(h, 2 * m, m) * .002
        p[f"gate_weight.{j}"] = torch.zeros(h, d, 4)
        bias = torch.tensor([_inv_softplus(cfg.decay_init),
                             math.log(cfg.beta_init / (cfg.beta_max - cfg.beta_init))] * 2)
        p[f"gate_bias.{j}"] = bias.repeat(h, 1)
    p["residual_raw"] = torch.zeros(levels, h, 2)
    p["count_gain_raw"] = torch.full((levels, h), _inv_softplus(.1))
    p["moment_gain"] = torch.full((levels, h), .1)
    p["route_mlp_gain"] = torch.full((levels, h), .1)
    p["output_logits"] = torch.zeros(levels, h)
    for e, (i, j) in enumerate(edges_of(levels)):
        p[f"relation_prefix.{e}"] = torch.zeros(h, cfg.slots[i], cfg.slots[j])
    ne = len(edges_of(levels))
    p["edge_logits"] = torch.zeros(ne, h)
    p["relation_gain"] = torch.full((levels, h), .1)
    p["relation_decay_raw"] = torch.full((ne, h), _inv_softplus(cfg.relation_decay_init))
    p["relation_beta_raw"] = torch.full(
        (ne, h), math.log(cfg.relation_beta_init / (1 - cfg.relation_beta_init)))
    return p


def initial_state(cfg: OracleConfig, p: dict, batch: int, dtype: torch.dtype) -> OracleState:
    """Learned prefixes broadcast over the batch, zero counts (src/gpa/attention.py:146-159)."""
    work = torch.float64 if dtype == torch.float64 else torch.float32
    levels = []
    for j, m in enumerate(cfg.slots):
        a = p[f"inner_prefix.{j}"].to(work).unsqueeze(0).expand(batch, -1, -1, -1)
        b = p[f"outer_prefix.{j}"].to(work).unsqueeze(0).expand(batch, -1, -1, -1)
        n = torch.zeros(batch, cfg.heads, m, dtype=work)
        if cfg.positional_mode == "moments":
            levels.append((a, b, n, torch.zeros(batch, cfg.heads, cfg.key_dim, m, dtype=work)))
        else:
            levels.append((a, b, n))
    rel = tuple(p[f"relation_prefix.{e}"].to(work).unsqueeze(0).expand(batch, -1, -1, -1)
                for e in range(len(edges_of(len(cfg.slots)))))
    return OracleState(tuple(levels), rel, 0, cfg.chunk_size, 0, None)


# --------------------------------------------------------------------------
# GDN primitive (src/gpa/ops.py:29-85, docs/EQUATIONS.md:7-28)
# --------------------------------------------------------------------------

def gdn_step(state, key, value, log_gate, beta):
    """One key-major gated delta update S <- a S + b u(k)(v - u(k)^T a S)^T (src/gpa/ops.py:29-42)."""
    k = unit(key).to(state.dtype)
    decayed = state * log_gate.to(state.dtype).exp()[..., None, None]
    pred = torch.einsum("bhk,bhkv->bhv", k, decayed)
    err = value.to(state.dtype) - pred
    return decayed + beta.to(state.dtype)[..., None, None] * k[..., :, None] * err[..., None, :]


def read(query, state):
    """y = u(q)^T S, cast to the query dtype (src/gpa/ops.py:45-46)."""
    return torch.einsum("bhk,bhkv->bhv", unit(query).to(state.dtype), state).to(query.dtype)


def gdn_scan(q, k, v, g, beta, state):
    """Causal token loop of ``gdn_step`` + ``read`` (src/gpa/ops.py:49-57,78-85)."""
    if q.shape[1] == 0:
        return v.new_empty(v.shape), state
    ys = []
    for t in range(q.shape[1]):
        state = gdn_step(state, k[:, t], v[:, t], g[:, t], beta[:, t])
        ys.append(read(q[:, t], state))
    return torch.stack(ys, 1), state


def rope(x, positions):
    """Adjacent-pair rotary embedding, base 10000 (src/gpa/ops.py:117-132): pair i of the last
    dimension turns by positions * 10000^(-2i/D); x [B,T,H,D] with positions [T], or [B,H,D] with
    one position."""
    d = x.shape[-1]
    work = x.to(_work_dtype(x))
    pos = torch.as_tensor(positions, dtype=work.dtype)
    if x.ndim == 4:
        pos = pos[None, :, None]
    freq = 10000. ** (-torch.arange(0, d, 2, dtype=work.dtype) / d)
    ang = pos[..., None] * freq
    ev, od = work[..., 0::2], work[..., 1::2]
    return torch.stack((ev * ang.cos() - od * ang.sin(), ev * ang.sin() + od * ang.cos()),
                       -1).flatten(-2).to(x.dtype)


def linear_scan(q, k, v, state):
    """Additive moments S += k v^T, read q^T S after each update (src/gpa/ops.py:86-114)."""
    outs = []
    for t in range(q.shape[1]):
        state = state + k[:, t].to(state.dtype)[..., :, None] * v[:, t].to(state.dtype)[..., None, :]
        outs.append(torch.einsum("bhd,bhdm->bhm", q[:, t].to(state.dtype), state).to(q.dtype))
    return torch.stack(outs, 1), state


# --------------------------------------------------------------------------
# Level pieces (src/gpa/attention.py:161-262)
# --------------------------------------------------------------------------

def _gates(cfg, p, j, key):
    """(gi, bi, go, bo) from u(k) (src/gpa/attention.py:161-174, default flags)."""
    w = p[f"gate_weight.{j}"]
    raw = torch.einsum("...hd,hdc->...hc", unit(key), w.to(key.dtype))
    raw = raw.to(_work_dtype(key)) + p[f"gate_bias.{j}"]
    gi, bi, go, bo = raw.unbind(-1)
    gi = -_softplus(gi).clamp(max=10.)
    go = -_softplus(go).clamp(max=10.)
    if cfg.positional_mode == "none":
        gi, go = gi * 0, go * 0
    return gi, cfg.beta_max * bi.sigmoid(), go, cfg.beta_max * bo.sigmoid()


def _slot(p, j, key):
    """Linear slot projection k C^T (src/gpa/attention.py:176-184)."""
    return torch.einsum("...hd,hmd->...hm", key, p[f"center.{j}"].to(key.dtype))


def _residual(p, j, key, value, rk, rv):
    """Bounded residual step sizes (src/gpa/attention.py:190-194)."""
    eta = 1 + .25 * p["residual_raw"][j].tanh()
    return ((key - eta[:, 0, None] * rk.to(key.dtype)).to(key.dtype),
            (value - eta[:, 1, None] * rv.to(value.dtype)).to(value.dtype))


def _base_logits(cfg, p, j, raw, count, moment=None):
    """read_scale * raw + softplus(c) log1p(n), plus g_m tanh(moment / (1 + n)) with positional
    moments (src/gpa/attention.py:196-204)."""
    gain = _softplus(p["count_gain_raw"][j])[..., None]
    logits = cfg.read_scale * raw.to(count.dtype) + gain * count.log1p()
    if moment is not None:
        logits = logits + p["moment_gain"][j][..., None] * torch.tanh(moment / (1 + count))
    return logits


def _relations(cfg, p, edges, local, writes, rel_states):
    """One GDN scan per ordered edge (src/gpa/attention.py:206-223, default flags)."""
    messages = [[] for _ in local]
    new = []
    for e, ((i, j), old) in enumerate(zip(edges, rel_states)):
        shape = writes[i].shape[:-1]
        g = -_softplus(p["relation_decay_raw"][e]).expand(shape)
        if cfg.positional_mode == "none":
            g = g * 0
        beta = p["relation_beta_raw"][e].sigmoid().expand(shape)
        msg, mem = gdn_scan(local[i], writes[i], writes[j], g, beta, old)
        messages[j].append((e, msg))
        new.append(mem)
    return messages, tuple(new)


def _bridge(cfg, p, edges, q, logits, messages, counts):
    """Dense reader: edge mix, then the centred tanh correction or the product read (each
    message times the norm of its source level's route softmax, added with gain
    M e^{clamp(g, -4, 4)}, minus e^{clamp(g)} log1p(counts) when marginal), route softmax +
    MLP, query projection (src/gpa/attention.py:225-262, flags rsa_update,
    shared_query_center and balanced_bridge off)."""
    routes, qouts = [], []
    for j, base in enumerate(logits):
        if messages[j]:
            ids = [e for e, _ in messages[j]]
            weights = p["edge_logits"][ids].softmax(0)
            if cfg.paper_product_read:
                gain = p["relation_gain"][j].clamp(-4, 4).exp()[..., None]
                incoming = sum(w[..., None] * msg
                               * logits[edges[e][0]].softmax(-1).norm(dim=-1, keepdim=True)
                               for w, (e, msg) in zip(weights, messages[j]))
                base = base + base.shape[-1] * gain * incoming
                if cfg.relation_marginal:
                    base = base - gain * counts[j].log1p()
            else:
                incoming = sum(w[..., None] * msg for w, (_, msg) in zip(weights, messages[j]))
                centered = incoming - incoming.mean(-1, keepdim=True)
                normalized = centered / (centered.square().mean(-1, keepdim=True) + 1e-5).sqrt()
                base = base + p["relation_gain"][j][..., None] * normalized.tanh()
        route = base.softmax(-1).to(q.dtype)
        hidden = F.gelu(torch.einsum("...hm,hmr->...hr", route, p[f"route_up.{j}"].to(q.dtype)))
        route = route + p["route_mlp_gain"][j][..., None] * torch.einsum(
            "...hr,hrm->...hm", hidden, p[f"route_down.{j}"].to(q.dtype))
        route = route.to(q.dtype)
        qo = torch.einsum("...hm,hmn->...hn", route, p[f"route_weight.{j}"].to(q.dtype))
        direct = cfg.query_scale * torch.einsum("...hd,hdm->...hm", q, p[f"query_weight.{j}"].to(q.dtype))
        qo = qo + direct
        routes.append(route)
        qouts.append(qo.to(q.dtype))
    return routes, qouts


def _token(cfg, p, edges, q, k, v, state):
    """Exact recurrence for one token, post-update writes (src/gpa/attention.py:264-297); with
    positional moments the query is rotated (RoPE at the cache position) and each level adds
    the moment read to its base logits."""
    moments = cfg.positional_mode == "moments"
    pos = state.position
    qr = rope(q, pos) if moments else q
    key, value = k, v
    levels, writes, logits = [], [], []
    for j, old in enumerate(state.levels):
        a_old, b_old, n_old = old[:3]
        slot = _slot(p, j, key)
        gi, bi, go, bo = _gates(cfg, p, j, key)
        a = gdn_step(a_old, key, slot, gi, bi)
        b = gdn_step(b_old, slot, value, go, bo)
        write = read(key, a).softmax(-1)
        count = n_old + write.to(n_old.dtype)
        corr = None
        if moments:
            kh = unit(key)
            delta = (rope(kh, pos) - kh).to(old[3].dtype)
            mom = old[3] + delta[..., :, None] * write.to(delta.dtype)[..., None, :]
            corr = read(qr, mom)
        raw = read(qr, a)
        logits.append(_base_logits(cfg, p, j, raw, count, corr))
        writes.append(write)
        levels.append((a, b, count, mom) if moments else (a, b, count))
        rk = torch.einsum("bhdm,bhm->bhd", a, write.to(a.dtype))
        rv = torch.einsum("bhm,bhmv->bhv", write.to(b.dtype), b)
        key, value = _residual(p, j, key, value, rk, rv)
    local = [x.softmax(-1).to(q.dtype).unsqueeze(1) for x in logits]
    messages, rel = _relations(cfg, p, edges, local, [x.unsqueeze(1) for x in writes], state.relations)
    messages = [[(e, m[:, 0]) for e, m in group] for group in messages]
    routes, qouts = _bridge(cfg, p, edges, qr, logits, messages, [lv[2] for lv in levels])
    weights = p["output_logits"].softmax(0)
    out = sum(weights[j][..., None] * read(qo, levels[j][1]) for j, qo in enumerate(qouts))
    new = OracleState(tuple(levels), rel, state.position + 1, cfg.chunk_size, 0, None)
    return out.to(v.dtype), new, routes


def _block(cfg, p, edges, q, k, v, state):
    """One lag block with frozen residual snapshots (src/gpa/attention.py:299-345); with
    positional moments the queries are rotated (RoPE at their positions) and each level adds
    the linear-scan moment read to its base logits."""
    moments = cfg.positional_mode == "moments"
    positions = torch.arange(state.position, state.position + q.shape[1])
    qr = rope(q, positions) if moments else q
    frozen = state.frozen or tuple((lv[0], lv[1]) for lv in state.levels)
    key, value = k, v
    finals, writes, logits, outer_in, history = [], [], [], [], []
    for j, (old, (fa, fb)) in enumerate(zip(state.levels, frozen)):
        a_old, n_old = old[0], old[2]
        slot = _slot(p, j, key)
        gi, bi, go, bo = _gates(cfg, p, j, key)
        raw, a = gdn_scan(qr, key, slot, gi, bi, a_old)
        write = torch.einsum("bthd,bhdm->bthm", unit(key).to(fa.dtype), fa).softmax(-1)
        write = write.to(q.dtype)
        counts = n_old[:, None] + write.to(n_old.dtype).cumsum(1)
        history.append(counts)
        corr, mom = None, None
        if moments:
            kh = unit(key)
            delta = rope(kh, positions) - kh
            corr, mom = linear_scan(unit(qr), delta, write, old[3])
        logits.append(_base_logits(cfg, p, j, raw, counts, corr))
        writes.append(write)
        finals.append((a, counts[:, -1], mom))
        outer_in.append((slot, value, go, bo))
        rk = torch.einsum("bhdm,bthm->bthd", fa, write.to(fa.dtype))
        rv = torch.einsum("bthm,bhmv->bthv", write.to(fb.dtype), fb)
        key, value = _residual(p, j, key, value, rk, rv)
    local = [x.softmax(-1).to(q.dtype) for x in logits]
    messages, rel = _relations(cfg, p, edges, local, writes, state.relations)
    routes, qouts = _bridge(cfg, p, edges, qr, logits, messages, history)
    outs, levels = [], []
    for j, qo in enumerate(qouts):
        slot, vl, go, bo = outer_in[j]
        y, b = gdn_scan(qo, slot, vl, go, bo, state.levels[j][1])
        a_f, n_f, mom = finals[j]
        levels.append((a_f, b, n_f, mom) if moments else (a_f, b, n_f))
        outs.append(y)
    weights = p["output_logits"].softmax(0)
    out = sum(weights[j][..., None] * y for j, y in enumerate(outs))
    offset = (state.chunk_offset + q.shape[1]) % cfg.chunk_size
    new = OracleState(tuple(levels), rel, state.position + q.shape[1], cfg.chunk_size,
                      offset, frozen if offset else None)
    return out.to(v.dtype), new, routes


def forward(cfg: OracleConfig, p: dict, q, k, v, state: OracleState | None = None,
            return_routes: bool = False):
    """Block loop of ``DenseGPA.forward`` (src/gpa/attention.py:347-414).

    Blocks never straddle ``chunk_size - chunk_offset`` (src/gpa/attention.py:396-405);
    ``chunk_size == 1`` uses the exact token recurrence (src/gpa/attention.py:387-395).
    Returns (out [B,T,H,Dv], OracleState[, routes per level [B,T,H,M]]).
    """
    if state is None:
        state = initial_state(cfg, p, q.shape[0], q.dtype)
    edges = edges_of(len(cfg.slots))
    outs, hist = [], [[] for _ in cfg.slots]
    start, t_total = 0, q.shape[1]
    while start < t_total:
        if cfg.chunk_size == 1:
            y, state, routes = _token(cfg, p, edges, q[:, start], k[:, start], v[:, start], state)
            outs.append(y.unsqueeze(1))
            routes = [r.unsqueeze(1) for r in routes]
            start += 1
        else:
            end = min(t_total, start + cfg.chunk_size - state.chunk_offset)
            y, state, routes = _block(cfg, p, edges, q[:, start:end], k[:, start:end],
                                      v[:, start:end], state)
            outs.append(y)
            start = end
        for h_, r in zip(hist, routes):
            h_.append(r)
    out = torch.cat(outs, 1) if outs else v.new_empty(v.shape)
    if return_routes:
        routes = tuple(torch.cat(x, 1) if x else q.new_empty(q.shape[:3] + (m,))
                       for x, m in zip(hist, cfg.slots))
        return out, state, routes
    return out, state
