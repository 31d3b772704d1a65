"""Run the oracle on one golden case and report the worst relative error per field.

Shared by ``tests/test_oracle_golden.py``; also runnable by hand:
    python tests/golden/check_oracle.py config1
"""
from __future__ import annotations

import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (ROOT, HERE):
    if p not in sys.path:
        sys.path.insert(0, p)

from cases import CASES, DTYPES, build, compare_summary, params_digest  # noqa: E402


def load(name):
    return torch.load(os.path.join(HERE, f"{name}.pt"), weights_only=False)


def oracle_errors(name: str) -> dict:
    """{field: relative error} of the oracle against the stored reference record."""
    import oracle
    rec = load(name)
    spec = CASES[name]
    cfg, params, inputs = build(name)
    assert params_digest(params) == rec["params_sha256"], "case parameters changed"
    ocfg = oracle.OracleConfig(**cfg)
    p = {k: v.clone().requires_grad_() for k, v in params.items()}
    q, k, v = (inputs[x].clone().requires_grad_() for x in ("q", "k", "v"))
    out, state = oracle.forward(ocfg, p, q, k, v)
    out.float().square().mean().backward()
    err = {"out": compare_summary(out, rec["out"])}
    for x, t in zip("qkv", (q, k, v)):
        err[f"d{x}"] = compare_summary(t.grad, rec["grad_inputs"][x])
    for n, g in rec["grad_params"].items():
        if p[n].grad is None:
            err[f"d{n}"] = float("inf")
        else:
            err[f"d{n}"] = compare_summary(p[n].grad, g)
    for i, (a, b) in enumerate(zip(oracle.tensors_of(state), rec["state"])):
        err[f"state[{i}]"] = compare_summary(a, b)
    meta = rec["state_meta"]
    assert state.position == meta["position"] and state.chunk_offset == meta["chunk_offset"]
    assert (state.frozen is not None) == meta["frozen"]
    assert len(oracle.tensors_of(state)) == len(rec["state"])
    with torch.no_grad():
        if spec.get("partitions"):
            running, pieces = None, []
            for lo, hi in spec["partitions"]:
                y, running = oracle.forward(ocfg, params, inputs["q"][:, lo:hi],
                                            inputs["k"][:, lo:hi], inputs["v"][:, lo:hi], running)
                pieces.append(y)
            err["partition_out"] = compare_summary(torch.cat(pieces, 1), rec["partition_out"])
            for i, (a, b) in enumerate(zip(oracle.tensors_of(running), rec["partition_state"])):
                err[f"partition_state[{i}]"] = compare_summary(a, b)
        dec = inputs["decode"]
        if dec:
            running = oracle.OracleState(*[_detach(x) for x in (state.levels, state.relations)],
                                         state.position, state.chunk_size, state.chunk_offset,
                                         _detach(state.frozen))
            outs = []
            for s in range(len(dec) // 3):
                y, running = oracle.forward(ocfg, params, dec[3 * s], dec[3 * s + 1],
                                            dec[3 * s + 2], running)
                outs.append(y)
            err["decode_out"] = compare_summary(torch.cat(outs, 1), rec["decode_out"])
            for i, (a, b) in enumerate(zip(oracle.tensors_of(running), rec["decode_state"])):
                err[f"decode_state[{i}]"] = compare_summary(a, b)
            dm = rec["decode_meta"]
            assert running.position == dm["position"] and running.chunk_offset == dm["chunk_offset"]
            assert (running.frozen is not None) == dm["frozen"]
    return err


def _detach(x):
    if x is None:
        return None
    if isinstance(x, torch.Tensor):
        return x.detach()
    return tuple(_detach(y) for y in x)


TOLERANCE = {"float64": 1e-10, "float32": 2e-5, "bfloat16": 2e-2}


if __name__ == "__main__":
    for name in (sys.argv[1:] or list(CASES)):
        e = oracle_errors(name)
        worst = max(e, key=e.get)
        print(f"{name:14s} dtype={CASES[name]['dtype']:9s} worst={e[worst]:.3g} ({worst}) "
              f"out={e['out']:.3g} dq={e['dq']:.3g} dk={e['dk']:.3g} dv={e['dv']:.3g}")
        _ = DTYPES
