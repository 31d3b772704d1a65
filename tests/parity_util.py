"""Helpers shared by the GPU parity tests: run the b200 path and the CPU oracle
on the same seeded model / inputs and report relative L2 errors.

The oracle (``oracle/``) is only the checker here; the path under test is
``gpa_b200.DenseGPA`` on CUDA, which calls the native library.
"""
from __future__ import annotations

import torch

import oracle
from gpa_b200 import DenseGPA, GPAConfig
from gpa_b200.state import tensors


def rel(a, b) -> float:
    """Relative L2 error of a against b; a gradient of None counts as zeros."""
    if a is None and b is None:
        return 0.0
    if a is None:
        a = torch.zeros_like(b)
    if b is None:
        b = torch.zeros_like(a)
    a = a.detach().double().cpu().reshape(-1)
    b = b.detach().double().cpu().reshape(-1)
    nb = b.norm()
    if nb == 0:
        return float(a.norm())
    return float((a - b).norm() / nb)


def ostate_to_flat(st: oracle.OracleState):
    return oracle.tensors_of(st)


def to_oracle_state(st, device="cpu", dtype=torch.float64):
    levels = tuple((lv.inner.detach().to(device, dtype), lv.outer.detach().to(device, dtype),
                    lv.count.detach().to(device, dtype))
                   + (() if lv.position is None else (lv.position.detach().to(device, dtype),))
                   for lv in st.levels)
    rel_ = tuple(r.memory.detach().to(device, dtype) for r in st.relations)
    fz = None if st.frozen is None else tuple((f.inner.detach().to(device, dtype),
                                                f.outer.detach().to(device, dtype)) for f in st.frozen)
    return oracle.OracleState(levels, rel_, st.position, st.chunk_size, st.chunk_offset, fz)


def make_model(cfg_kwargs: dict, seed: int = 0, prefix_std: float | None = None,
               perturb: float = 0.0) -> DenseGPA:
    """Seeded b200 model; optionally re-draw prefixes and perturb the zero-initialised
    parameters so every gradient path carries signal."""
    torch.manual_seed(seed)
    model = DenseGPA(GPAConfig(**cfg_kwargs))
    g = torch.Generator().manual_seed(seed + 77)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if prefix_std and name.startswith(("inner_prefix", "outer_prefix", "relation_prefix")):
                p.copy_(torch.randn(p.shape, generator=g) * prefix_std)
            if perturb and name.startswith(("gate_weight", "edge_logits", "residual_raw",
                                            "output_logits")):
                p.add_(torch.randn(p.shape, generator=g) * perturb)
    return model


def oracle_config(model: DenseGPA) -> oracle.OracleConfig:
    c = model.config
    return oracle.OracleConfig(heads=c.heads, key_dim=c.key_dim, value_dim=c.value_dim,
                               slots=tuple(c.slots), chunk_size=c.chunk_size,
                               positional_mode=c.positional_mode, query_scale=c.query_scale,
                               beta_init=c.beta_init, beta_max=c.beta_max,
                               decay_init=c.decay_init, relation_beta_init=c.relation_beta_init,
                               relation_decay_init=c.relation_decay_init, read_scale=c.read_scale,
                               paper_product_read=c.paper_product_read,
                               relation_marginal=c.relation_marginal)


def run_pair(model: DenseGPA, q, k, v, *, oracle_dtype=torch.float64, state_weights=True,
             device="cuda"):
    """Forward + backward of out-weighted loss (+ weighted state) on both paths.

    Returns {name: relative error}."""
    gpu = model.to(device)
    gen = torch.Generator().manual_seed(1234)
    dout = torch.randn(q.shape[:3] + (model.config.value_dim,), generator=gen)
    # ---- b200
    qg, kg, vg = (x.to(device).clone().requires_grad_() for x in (q, k, v))
    gpu.zero_grad(set_to_none=True)
    out, st = gpu(qg, kg, vg)
    ts = list(tensors(st))
    weights = [torch.randn(t.shape, generator=gen) * .1 for t in ts] if state_weights else []
    loss = (out.float() * dout.to(device)).sum()
    for t, w in zip(ts, weights):
        loss = loss + (t.float() * w.to(device)).sum()
    loss.backward()
    # ---- oracle
    p = {n: t.detach().cpu().to(torch.float64 if oracle_dtype == torch.float64 else torch.float32)
         .clone().requires_grad_() for n, t in gpu.state_dict().items()}
    ocfg = oracle_config(gpu)
    oq, ok, ov = (x.detach().cpu().to(oracle_dtype).clone().requires_grad_() for x in (q, k, v))
    oout, ost = oracle.forward(ocfg, p, oq, ok, ov)
    ots = oracle.tensors_of(ost)
    oloss = (oout.double() * dout.double()).sum()
    for t, w in zip(ots, weights):
        oloss = oloss + (t.double() * w.double()).sum()
    oloss.backward()
    err = {"out": rel(out, oout)}
    for nm, a, b in (("dq", qg, oq), ("dk", kg, ok), ("dv", vg, ov)):
        err[nm] = rel(a.grad, b.grad)
    for n, prm in gpu.named_parameters():
        og = p[n].grad
        if og is None:
            continue
        if prm.grad is None:
            err["d" + n] = float("inf")
            continue
        err["d" + n] = rel(prm.grad, og)
    for i, (a, b) in enumerate(zip(ts, ots)):
        err[f"state{i}"] = rel(a, b)
    assert st.position == ost.position and st.chunk_offset == ost.chunk_offset
    assert (st.frozen is None) == (ost.frozen is None)
    return err


def worst(err: dict):
    k = max(err, key=err.get)
    return k, err[k]
