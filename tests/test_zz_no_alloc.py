"""The no-allocation forward (gpa_b200_forward_noalloc) against gpa_b200_forward.

Some callers of this library cannot allocate device memory: code that runs
inside another runtime's stream capture or fixed memory pool, or a decode loop
whose memory is reserved up front.  For them the library keeps its forward
workspace in a file-scope device array and exposes a forward that takes only
inputs and outputs.  This test calls both entry points through the C ABI on
the same seeded decode-style calls -- a short prefill, then a one-token step
that continues from the first call's cache -- and requires the same output and
cache from both, call after call.  It also checks that a call too large for the
array is refused with a clear error.  It is collected last (file name) so that
a run stopping at the first failure has run every other test before it.
"""
from __future__ import annotations

import pytest
import torch

from gpa_b200 import DenseGPA, GPAConfig, _lib
from gpa_b200.core import _Plan, _stream

pytestmark = pytest.mark.gpu

TOL = 1e-6  # same kernels, same order: results agree to rounding noise


def _flat_state(state, plan):
    flat = []
    for lv in state.levels:
        flat += [lv.inner, lv.outer, lv.count]
    flat += [r.memory for r in state.relations]
    if plan.fz_in:
        for f in state.frozen:
            flat += [f.inner, f.outer]
    return [t.float().contiguous() for t in flat]


def _call(lib, model, q, k, v, state, noalloc: bool):
    """One forward through the C ABI; returns (out, flat output cache, plan)."""
    plan = _Plan(model.config, q, v, state)
    params = model._flat_params()
    st_in = _flat_state(state, plan)
    out = torch.empty(plan.B, plan.T, plan.H, plan.Dv, device=q.device, dtype=v.dtype)
    st_out = [torch.empty(s, device=q.device) for s in plan.state_shapes(plan.fz_out)]
    args = (plan.dims, plan.params_ref(params), q.data_ptr(), k.data_ptr(), v.data_ptr(),
            plan.state_ref(st_in, plan.fz_in), plan.state_ref(st_out, plan.fz_out), out.data_ptr())
    if noalloc:
        rc = lib.gpa_b200_forward_noalloc(*args, _stream(q.device))
        _lib.check(rc, "gpa_b200_forward_noalloc")
    else:
        nbytes = lib.gpa_b200_saved_bytes(plan.dims)
        # all bytes 0xFF (an fp32 NaN): a read of any region this call did not write first
        # would poison the compared outputs
        saved = torch.full((nbytes,), 255, device=q.device, dtype=torch.uint8)
        rc = lib.gpa_b200_forward(*args, saved.data_ptr(), nbytes, _stream(q.device))
        _lib.check(rc, "gpa_b200_forward")
    torch.cuda.synchronize()
    return out, st_out, plan


def _to_state(model, flat, plan, position):
    from gpa_b200.state import GPAState, LevelState, RelationState, ResidualSnapshot
    L = plan.L
    levels = tuple(LevelState(flat[3 * j], flat[3 * j + 1], flat[3 * j + 2]) for j in range(L))
    rels = tuple(RelationState(i, j, flat[3 * L + e]) for e, (i, j) in enumerate(model.edges))
    fz = None
    if plan.fz_out:
        b = 3 * L + plan.E
        fz = tuple(ResidualSnapshot(flat[b + 2 * j], flat[b + 2 * j + 1]) for j in range(L))
    return GPAState(levels, rels, position, model.config.chunk_size, plan.new_offset, fz)


def _rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_forward_matches_caller_buffer_forward(dtype):
    lib = _lib.load()
    torch.manual_seed(0)
    cfg = GPAConfig(heads=4, key_dim=32, value_dim=32, slots=(16, 32), chunk_size=64)
    model = DenseGPA(cfg).cuda()
    g = torch.Generator().manual_seed(1)
    prefill = [torch.randn(1, 9, 4, 32, generator=g).to("cuda", dtype) for _ in range(3)]
    step = [torch.randn(1, 1, 4, 32, generator=g).to("cuda", dtype) for _ in range(3)]
    with torch.no_grad():
        # a larger call first leaves unrelated values all over the shared array, so the
        # compared calls below only match if they write every part of it that they read
        big = [torch.randn(2, 48, 4, 32, generator=g).to("cuda", dtype) for _ in range(3)]
        _call(lib, model, *big, model.initial_state(2, device="cuda", dtype=dtype), noalloc=True)
        state = model.initial_state(1, device="cuda", dtype=dtype)
        ref_state = new_state = state
        for xs in (prefill, step):  # two calls in a row, the second continuing the cache
            ref_out, ref_flat, plan = _call(lib, model, *xs, ref_state, noalloc=False)
            out, flat, plan2 = _call(lib, model, *xs, new_state, noalloc=True)
            assert _rel(out.float(), ref_out.float()) <= TOL
            for a, b in zip(flat, ref_flat):
                assert _rel(a, b) <= TOL
            position = ref_state.position + xs[0].shape[1]
            ref_state = _to_state(model, ref_flat, plan, position)
            new_state = _to_state(model, flat, plan2, position)
        assert new_state.chunk_offset == 10 and new_state.frozen is not None


def test_noalloc_refuses_calls_larger_than_its_array():
    lib = _lib.load()
    cap = lib.gpa_b200_noalloc_capacity()
    assert cap == 64 << 20
    cfg = GPAConfig(heads=16, key_dim=128, value_dim=128, slots=(64, 64, 64, 128), chunk_size=64)
    model = DenseGPA(cfg).cuda()
    q = torch.zeros(2, 512, 16, 128, device="cuda", dtype=torch.bfloat16)
    state = model.initial_state(2, device="cuda", dtype=q.dtype)
    plan = _Plan(cfg, q, q, state)
    assert lib.gpa_b200_saved_bytes(plan.dims) > cap
    with pytest.raises(ValueError, match="no-allocation entry point holds"):
        _call(lib, model, q, q, q, state, noalloc=True)
