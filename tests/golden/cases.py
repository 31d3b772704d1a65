"""Seeded golden-vector cases shared by the fixture generator and the tests.

Each case fixes a configuration, the parameters (the reference's initial
values drawn from a seed, optionally with prefixes re-drawn at N(0, std)) and
the inputs.  ``make_golden.py`` runs the reference ``gpa.DenseGPA`` (torch
backend) on them and stores outputs; the tests rebuild the same parameters
and inputs here and compare.
"""
from __future__ import annotations

import hashlib

import torch

# name -> spec.  dims: heads, key_dim, value_dim, slots, chunk_size.  ``execution`` (default
# "reference") selects the reference's schedule: "packed" (src/gpa/packed.py, taken for uniform
# slots) or "staged" (src/gpa/staged.py, taken for uniform slots with key_dim == slots[0] on
# runs of >= 4 whole chunks starting at a block boundary).
CASES = {
    # fp32, chunk 1, B=2, T=16, H=4, 32/48, slots (64,64,64,128): the reference's CPU-runnable case
    "config1": dict(cfg=dict(heads=4, key_dim=32, value_dim=48, slots=(64, 64, 64, 128),
                             chunk_size=1), batch=2, length=16, dtype="float32", seed=0,
                    reference_init=True, decode=1),
    # small lagged blocks with partial blocks, float64, unequal slots
    "chunk4_f64": dict(cfg=dict(heads=2, key_dim=8, value_dim=6, slots=(4, 8), chunk_size=4),
                       batch=2, length=13, dtype="float64", seed=3,
                       partitions=((0, 5), (5, 6), (6, 10), (10, 13)), decode=2),
    # three levels, chunk 3, positional_mode none, float64
    "none_f64": dict(cfg=dict(heads=2, key_dim=4, value_dim=3, slots=(3, 2, 4), chunk_size=3,
                              positional_mode="none"), batch=2, length=9, dtype="float64", seed=11,
                     partitions=((0, 2), (2, 3), (3, 7), (7, 9)), decode=1),
    # chunk 1 exact recurrence, float64, tiny
    "token_f64": dict(cfg=dict(heads=2, key_dim=4, value_dim=3, slots=(3, 2), chunk_size=1),
                      batch=2, length=7, dtype="float64", seed=12,
                      partitions=((0, 3), (3, 7)), decode=1),
    # 64-token blocks with a partial tail, unequal slots, fp32
    "chunk64_f32": dict(cfg=dict(heads=2, key_dim=32, value_dim=32, slots=(16, 16, 16, 32),
                                 chunk_size=64), batch=1, length=130, dtype="float32", seed=5,
                        prefix_std=.02, partitions=((0, 47), (47, 65), (65, 130)), decode=1),
    # the benched head shape (D=Dv=128, slots (64,64,64,128)), bf16 activations, fp32 state
    "c2head_bf16": dict(cfg=dict(heads=2, key_dim=128, value_dim=128, slots=(64, 64, 64, 128),
                                 chunk_size=64), batch=1, length=80, dtype="bfloat16", seed=7,
                        prefix_std=.02, unit_qk=True, decode=1),
    # uniform slots through the reference's packed schedule (src/gpa/attention.py:301-303)
    "packed_uniform": dict(cfg=dict(heads=2, key_dim=16, value_dim=12, slots=(16, 16, 16),
                                    chunk_size=8), execution="packed", batch=2, length=37,
                           dtype="float32", seed=21, prefix_std=.02,
                           partitions=((0, 11), (11, 12), (12, 37)), decode=2),
    # uniform slots with key_dim == slots[0]: the reference's staged schedule runs the first
    # 256 tokens (src/gpa/attention.py:370-373), its lag-block path the 44-token tail
    "staged_uniform": dict(cfg=dict(heads=2, key_dim=32, value_dim=24, slots=(32, 32, 32, 32),
                                    chunk_size=64), execution="staged", batch=1, length=300,
                           dtype="float32", seed=22, prefix_std=.02, decode=1),
    # the staged schedule in bf16 rounds at other points than the lag-block schedule that the
    # oracle restates: token-summed scalar parameter gradients (edge_logits) differ by ~2.3e-2
    "staged_bf16": dict(cfg=dict(heads=2, key_dim=64, value_dim=64, slots=(64, 64, 64, 64),
                                 chunk_size=64), execution="staged", batch=1, length=320,
                        dtype="bfloat16", seed=23, prefix_std=.02, unit_qk=True, decode=1,
                        oracle_param_tol=5e-2),
    # the product reader (paper_product_read, src/gpa/attention.py:231-236): messages times the
    # norm of the source level's route softmax, gain M e^{clamp(g)}; lag blocks, float64
    "product_f64": dict(cfg=dict(heads=2, key_dim=8, value_dim=6, slots=(4, 8, 6), chunk_size=4,
                                 paper_product_read=True),
                        batch=2, length=13, dtype="float64", seed=31,
                        partitions=((0, 5), (5, 6), (6, 13)), decode=2),
    # product reader with the marginal count term, exact token recurrence, float64
    "marginal_token_f64": dict(cfg=dict(heads=2, key_dim=4, value_dim=3, slots=(3, 2, 4),
                                        chunk_size=1, paper_product_read=True,
                                        relation_marginal=True),
                               batch=2, length=7, dtype="float64", seed=32,
                               partitions=((0, 3), (3, 7)), decode=1),
    # product + marginal at 64-token blocks with a partial tail, fp32
    "marginal_c64_f32": dict(cfg=dict(heads=2, key_dim=32, value_dim=32, slots=(16, 16, 16, 32),
                                      chunk_size=64, paper_product_read=True,
                                      relation_marginal=True),
                             batch=1, length=130, dtype="float32", seed=33, prefix_std=.02,
                             partitions=((0, 47), (47, 65), (65, 130)), decode=1),
    # positional moments (src/gpa/attention.py:277-283, 318-322; src/gpa/ops.py:86-132): rotated
    # queries and the per-level additive moment state read into the base logits
    "moments_f64": dict(cfg=dict(heads=2, key_dim=8, value_dim=6, slots=(4, 8, 6), chunk_size=4,
                                 positional_mode="moments"),
                        batch=2, length=13, dtype="float64", seed=41,
                        partitions=((0, 5), (5, 6), (6, 13)), decode=2),
    "moments_token_f64": dict(cfg=dict(heads=2, key_dim=4, value_dim=3, slots=(3, 2, 4),
                                       chunk_size=1, positional_mode="moments"),
                              batch=2, length=7, dtype="float64", seed=42,
                              partitions=((0, 3), (3, 7)), decode=1),
    "moments_c64_f32": dict(cfg=dict(heads=2, key_dim=32, value_dim=32, slots=(16, 16, 16, 32),
                                     chunk_size=64, positional_mode="moments"),
                            batch=1, length=130, dtype="float32", seed=43, prefix_std=.02,
                            partitions=((0, 47), (47, 65), (65, 130)), decode=1),
}

DTYPES = {"float32": torch.float32, "float64": torch.float64, "bfloat16": torch.bfloat16}


def build(name: str):
    """Return (cfg dict, params {name: fp32/fp64 tensor}, inputs dict) for a case.

    Parameters come from ``oracle.init_parameters`` under ``torch.manual_seed(seed)``
    (the reference's own draw order), then prefixes re-drawn at N(0, prefix_std)
    with a separate generator when the case asks for it.
    """
    from oracle import OracleConfig, init_parameters
    spec = CASES[name]
    cfg = dict(spec["cfg"])
    dtype = DTYPES[spec["dtype"]]
    torch.manual_seed(spec["seed"])
    params = init_parameters(OracleConfig(**cfg))
    gen = torch.Generator().manual_seed(1000 + spec["seed"])
    std = spec.get("prefix_std")
    if std:
        for key in sorted(params):
            if key.startswith(("inner_prefix.", "outer_prefix.", "relation_prefix.")):
                params[key] = torch.randn(params[key].shape, generator=gen) * std
    if dtype == torch.float64:
        params = {k: v.double() for k, v in params.items()}
    b, t, h = spec["batch"], spec["length"], cfg["heads"]
    d, dv = cfg["key_dim"], cfg["value_dim"]
    if spec.get("reference_init"):
        # the reference's CPU-runnable case draws q, k, v right after the model under seed 0
        q = torch.randn(b, t, h, d)
        k = torch.randn(b, t, h, d)
        v = torch.randn(b, t, h, dv)
    else:
        q = torch.randn(b, t, h, d, generator=gen)
        k = torch.randn(b, t, h, d, generator=gen)
        v = torch.randn(b, t, h, dv, generator=gen)
    if spec.get("unit_qk"):
        q = q / q.norm(dim=-1, keepdim=True)
        k = k / k.norm(dim=-1, keepdim=True)
    n_dec = spec.get("decode", 0)
    dec = [torch.randn(b, 1, h, x, generator=gen) for _ in range(n_dec) for x in (d, d, dv)]
    inputs = {"q": q.to(dtype), "k": k.to(dtype), "v": v.to(dtype),
              "decode": [x.to(dtype) for x in dec]}
    return cfg, params, inputs


def params_digest(params: dict) -> str:
    """sha256 over the parameters in key order (bytes of the fp32/fp64 tensors)."""
    h = hashlib.sha256()
    for key in sorted(params):
        h.update(key.encode())
        h.update(params[key].detach().contiguous().cpu().numpy().tobytes())
    return h.hexdigest()


def projection(x: torch.Tensor, n: int = 8) -> torch.Tensor:
    """n fixed Gaussian projections of a tensor (float64), for large tensors."""
    g = torch.Generator().manual_seed(x.numel())
    r = torch.randn(n, x.numel(), generator=g, dtype=torch.float64)
    return r @ x.detach().reshape(-1).to(torch.float64)


def summarize(x: torch.Tensor, full_limit: int = 2048):
    """Full tensor when small, else {'proj', 'norm'} (float64)."""
    x = x.detach().cpu()
    if x.numel() <= full_limit:
        return x.clone()
    return {"proj": projection(x), "norm": x.to(torch.float64).norm()}


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.detach().to(torch.float64).reshape(-1)
    b = b.detach().to(torch.float64).reshape(-1)
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def compare_summary(actual: torch.Tensor, stored) -> float:
    """Relative error of ``actual`` against a stored summary (full or projected)."""
    if isinstance(stored, dict):
        p = projection(actual)
        err_p = float((p - stored["proj"]).norm() / stored["proj"].norm().clamp_min(1e-30))
        err_n = abs(float(actual.detach().to(torch.float64).norm()) - float(stored["norm"])) / max(
            float(stored["norm"]), 1e-30)
        return max(err_p, err_n)
    return rel_l2(actual, stored)


__all__ = ["CASES", "DTYPES", "build", "params_digest", "summarize", "compare_summary",
           "rel_l2", "projection"]

