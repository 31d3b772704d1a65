"""The fused one-token decode step (gpa_b200_step, DecodeSession) against the oracle.

A prefill through ``DenseGPA.forward`` leaves the cache inside a lag block; then
one-token steps of a DecodeSession (cache in place, offset on the device) run
across several block boundaries, and each step's output and the final cache are
compared with the oracle's one-token ``forward`` calls from the same prefix
(src/gpa/attention.py:347-414).  The same steps replayed from a captured CUDA
graph must reproduce the eager session exactly.
"""
from __future__ import annotations

import pytest
import torch

import oracle
from parity_util import make_model, oracle_config, rel, to_oracle_state
from gpa_b200.decode import DecodeSession
from gpa_b200.state import tensors

pytestmark = pytest.mark.gpu

CFG = dict(heads=2, key_dim=32, value_dim=24, slots=(16, 32, 8), chunk_size=4)


def _inputs(gen, B, T, H, D, Dv, dtype):
    q = torch.randn(B, T, H, D, generator=gen)
    k = torch.randn(B, T, H, D, generator=gen)
    v = torch.randn(B, T, H, Dv, generator=gen)
    return [x.to(dtype) for x in (q, k, v)]


# a second shape: three levels with equal outer states and narrower values
CFG_SPLIT = dict(heads=2, key_dim=32, value_dim=16, slots=(16, 8, 16), chunk_size=4)
# the product reader (paper_product_read) with its marginal count term
CFG_PRODUCT = dict(CFG, paper_product_read=True, relation_marginal=True)
# positional moments: rotated queries and the per-level moment state
CFG_MOMENTS = dict(CFG, positional_mode="moments")


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-4), (torch.bfloat16, 2e-2),
                                       (torch.float16, 2e-2)])
@pytest.mark.parametrize("prefill,cfg", [(6, CFG), (8, CFG), (6, CFG_SPLIT), (6, CFG_PRODUCT),
                                         (6, CFG_MOMENTS)])
def test_decode_steps_match_oracle(dtype, tol, prefill, cfg, cpu_threads):
    model = make_model(cfg, seed=3, prefix_std=0.02, perturb=0.1).cuda()
    gen = torch.Generator().manual_seed(7)
    B, H, D, Dv = 2, cfg["heads"], cfg["key_dim"], cfg["value_dim"]
    pre = _inputs(gen, B, prefill, H, D, Dv, dtype)
    steps = [_inputs(gen, B, 1, H, D, Dv, dtype) for _ in range(9)]
    p = {n: t.detach().cpu().double() for n, t in model.state_dict().items()}
    ocfg = oracle_config(model)
    with torch.no_grad():
        _, st = model(*(x.cuda() for x in pre))
        sess = DecodeSession(model, st, dtype)
        _, ost = oracle.forward(ocfg, p, *(x.double() for x in pre))
        for i, xs in enumerate(steps):
            y = sess.step(*(x.cuda() for x in xs))
            oy, ost = oracle.forward(ocfg, p, *(x.double() for x in xs), ost)
            assert rel(y.float(), oy) <= tol, (i, rel(y.float(), oy))
        final = sess.state
    assert final.position == ost.position and final.chunk_offset == ost.chunk_offset
    assert (final.frozen is None) == (ost.frozen is None)
    for a, b in zip(tensors(final), oracle.tensors_of(ost)):
        assert rel(a, b) <= tol


def test_decode_graph_replay_matches_eager_steps():
    model = make_model(CFG, seed=4, prefix_std=0.02, perturb=0.1).cuda()
    gen = torch.Generator().manual_seed(8)
    B, H, D, Dv = 3, CFG["heads"], CFG["key_dim"], CFG["value_dim"]
    dtype = torch.bfloat16
    pre = _inputs(gen, B, 5, H, D, Dv, dtype)
    steps = [[x.cuda() for x in _inputs(gen, B, 1, H, D, Dv, dtype)] for _ in range(7)]
    with torch.no_grad():
        _, st = model(*(x.cuda() for x in pre))
        eager = DecodeSession(model, st, dtype)
        graph = DecodeSession(model, st, dtype)
        sq, sk, sv = (torch.empty_like(x) for x in steps[0])
        out = graph.capture(sq, sk, sv)
        for xs in steps:
            ye = eager.step(*xs)
            for s_, x in zip((sq, sk, sv), xs):
                s_.copy_(x)
            yg = graph.replay()
            assert torch.equal(ye, yg)
        torch.cuda.synchronize()
    a, b = eager.state, graph.state
    assert a.chunk_offset == b.chunk_offset and a.position == b.position
    for x, y in zip(tensors(a), tensors(b)):
        assert torch.equal(x, y)
    assert out.data_ptr() == yg.data_ptr()


def test_decode_session_rejects_token_mode_and_bad_inputs():
    model = make_model(dict(CFG, chunk_size=1), seed=1).cuda()
    st = model.initial_state(1, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="chunk_size >= 2"):
        DecodeSession(model, st)
    model = make_model(CFG, seed=1).cuda()
    sess = DecodeSession(model, model.initial_state(1, device="cuda", dtype=torch.bfloat16))
    x = torch.zeros(1, 2, CFG["heads"], CFG["key_dim"], device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="decode inputs"):
        sess.step(x, x, x)
