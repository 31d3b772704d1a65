"""A whole b200 training step (forward + backward) captured once with GradientGraph.

Mirrors the reference's own graph tests (tests/test_training_graph.py:5-55 of fisalt/GPA): a
replay must give the gradients of an eager forward + backward on the same inputs, overwrite
rather than accumulate them, and follow new input values.  As with the reference's
GradientGraph, the captured model must not have run an eager backward on the default stream
before the capture: its parameters' gradient accumulators would then belong to that stream.
"""
from __future__ import annotations

import copy

import pytest
import torch

from parity_util import make_model, rel
from gpa_b200.training_graph import GradientGraph

pytestmark = pytest.mark.gpu

CFG = dict(heads=4, key_dim=64, value_dim=64, slots=(32, 32, 64), chunk_size=64)


def _loss_fn(model):
    def fn(q, k, v):
        out, _ = model(q, k, v)
        return out.float().square().mean(), out
    return fn


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_graph_replay_matches_eager_step(dtype):
    model = make_model(CFG, seed=5, prefix_std=.02, perturb=.3).cuda()
    g = torch.Generator(device="cuda").manual_seed(3)
    xs = [torch.randn(2, 200, 4, 64, device="cuda", generator=g).to(dtype).requires_grad_()
          for _ in range(3)]
    fn = _loss_fn(model)
    # eager reference step on a copy of the model: its parameters are other leaves, so the
    # captured model's gradient accumulators are first created inside GradientGraph's
    # side-stream warm-up, as the graph needs
    twin = copy.deepcopy(model)
    xe = [x.detach().clone().requires_grad_() for x in xs]
    loss_e, out_e = _loss_fn(twin)(*xe)
    loss_e.backward()
    eager = {n: p.grad.clone() for n, p in twin.named_parameters() if p.grad is not None}
    eager_in = [x.grad.clone() for x in xe]
    captured = GradientGraph(model, xs, fn)
    for _ in range(2):  # a second replay overwrites, it does not accumulate
        loss, out = captured.replay(*xs)
        torch.cuda.synchronize()
        assert rel(out, out_e) <= 1e-6 and rel(loss, loss_e) <= 1e-6
        for n, p in model.named_parameters():
            if n in eager:
                assert rel(p.grad, eager[n]) <= 1e-5, n
        for a, b in zip(captured.inputs, eager_in):
            assert rel(a.grad, b) <= 1e-5
    # new input values change the gradients (the replay is not a recorded constant)
    once = {n: p.grad.clone() for n, p in model.named_parameters() if p.grad is not None}
    captured.replay(*(x.detach() * 1.5 for x in xs))
    torch.cuda.synchronize()
    assert any(not torch.allclose(p.grad, once[n]) for n, p in model.named_parameters() if n in once)


def test_graph_rejects_other_shapes():
    model = make_model(CFG, seed=6).cuda()
    xs = [torch.randn(1, 64, 4, 64, device="cuda", dtype=torch.bfloat16, requires_grad=True)
          for _ in range(3)]
    captured = GradientGraph(model, xs, _loss_fn(model), warmups=1)
    with pytest.raises(ValueError):
        captured.replay(*(x[:, :32] for x in xs))
