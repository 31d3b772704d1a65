"""Generate golden vectors by running the REFERENCE DenseGPA (torch backend).

Run from the repository root, in a container that holds the reference sources:

    PYTHONPATH=<reference>/src:. python tests/golden/make_golden.py [--ref <reference>/src]

It imports ``gpa`` (fisalt/GPA v0.4.0), builds each case of ``cases.py``,
loads the case parameters into ``gpa.DenseGPA`` with ``load_state_dict``, and
stores under ``tests/golden/<case>.pt``:
  - the full-sequence output, the input gradients and every parameter gradient
    of ``out.float().square().mean()``;
  - the final cache tensors in ``GPAState`` order, plus position / chunk_offset
    and whether frozen snapshots are present;
  - outputs of the same sequence split into cached calls (``partitions``);
  - outputs of one-token recurrent decode steps continuing from the final cache.
Large tensors are stored as fixed Gaussian projections plus norm (cases.summarize).
The reference is not needed anywhere else: tests only read the ``.pt`` files.
"""
from __future__ import annotations

import argparse
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, HERE)

from cases import CASES, DTYPES, build, params_digest, summarize  # noqa: E402


def run_case(gpa, name):
    from gpa.state import tensors
    spec = CASES[name]
    cfg, params, inputs = build(name)
    dtype = DTYPES[spec["dtype"]]
    record = {"case": name, "spec": spec, "params_sha256": params_digest(params),
              "torch": torch.__version__, "reference": "gpa-attention " + gpa.__version__}
    if spec.get("reference_init"):
        torch.manual_seed(spec["seed"])
        fresh = gpa.DenseGPA(gpa.GPAConfig(**cfg))
        same = all(torch.equal(fresh.state_dict()[k], params[k]) for k in params)
        record["reference_init_matches"] = bool(same)
        assert same, "oracle.init_parameters does not reproduce the reference draw order"
    model = gpa.DenseGPA(gpa.GPAConfig(**cfg, execution=spec.get("execution", "reference")))
    if dtype == torch.float64:
        model = model.double()
    missing = model.load_state_dict(params, strict=True)
    assert not missing.missing_keys and not missing.unexpected_keys
    q, k, v = (inputs[x].clone().requires_grad_() for x in ("q", "k", "v"))
    out, state = model(q, k, v)
    loss = out.float().square().mean()
    loss.backward()
    record["out"] = summarize(out, 40000)
    record["loss"] = float(loss.detach())
    record["grad_inputs"] = {x: summarize(t.grad, 40000) for x, t in zip("qkv", (q, k, v))}
    record["grad_params"] = {n: summarize(p.grad) for n, p in model.named_parameters()
                             if p.grad is not None}
    record["state"] = [summarize(t) for t in tensors(state)]
    record["state_meta"] = {"position": state.position, "chunk_offset": state.chunk_offset,
                            "frozen": state.frozen is not None, "numel": state.numel()}
    with torch.no_grad():
        if spec.get("partitions"):
            running, pieces = None, []
            for lo, hi in spec["partitions"]:
                y, running = model(inputs["q"][:, lo:hi], inputs["k"][:, lo:hi],
                                   inputs["v"][:, lo:hi], running)
                pieces.append(y)
            record["partition_out"] = summarize(torch.cat(pieces, 1), 40000)
            record["partition_state"] = [summarize(t) for t in tensors(running)]
        dec = inputs["decode"]
        running, outs = state.detach(), []
        for s in range(len(dec) // 3):
            y, running = model(dec[3 * s], dec[3 * s + 1], dec[3 * s + 2], running)
            outs.append(y)
        if outs:
            record["decode_out"] = summarize(torch.cat(outs, 1), 40000)
            record["decode_state"] = [summarize(t) for t in tensors(running)]
            record["decode_meta"] = {"position": running.position,
                                     "chunk_offset": running.chunk_offset,
                                     "frozen": running.frozen is not None}
    return record


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=None, help="path to the reference's src/ directory")
    ap.add_argument("--cases", default=",".join(CASES))
    args = ap.parse_args()
    if args.ref:
        sys.path.insert(0, args.ref)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    import gpa
    for name in args.cases.split(","):
        rec = run_case(gpa, name)
        path = os.path.join(HERE, f"{name}.pt")
        torch.save(rec, path)
        print(f"{name}: loss={rec['loss']:.6g} -> {os.path.relpath(path)} "
              f"({os.path.getsize(path) / 1024:.0f} KiB)")


if __name__ == "__main__":
    main()
