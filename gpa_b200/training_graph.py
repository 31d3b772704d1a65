"""Forward + backward of a static-shape training step captured once in a CUDA graph.

Counterpart of fisalt/GPA's ``gpa.training_graph.GradientGraph``
(src/gpa/training_graph.py:10-38), with the same constructor, ``replay`` and
semantics:

* ``GradientGraph(model, inputs, loss_fn, warmups=3)`` clones ``inputs`` into
  static buffers (keeping each one's ``requires_grad``), runs ``warmups`` eager
  forward + backward passes on a side stream (they allocate the library's
  workspaces in the caching allocator and do not touch the parameters), clears
  every gradient, then records ``loss, output = loss_fn(*inputs)`` and
  ``loss.backward()`` in one graph.
* ``replay(*inputs)`` copies the new values into the static buffers (shapes and
  dtypes must match the captured ones) and replays the graph, which overwrites
  the captured gradient buffers of the parameters and of the static inputs;
  the optimizer step stays outside the graph.  Gradients are overwritten, not
  accumulated, and the ``.grad`` tensors must not be replaced (``zero_grad(
  set_to_none=True)``) while the graph is reused.

With the b200 backend the captured region is the native forward and backward
of every ``DenseGPA`` in ``loss_fn``: a fixed sequence of kernel launches on
the caller's stream with no host synchronisation, so a replay costs one graph
launch instead of several hundred kernel launches.
"""
from __future__ import annotations

import torch


class GradientGraph:
    def __init__(self, model: torch.nn.Module, inputs, loss_fn, warmups: int = 3):
        self.model = model
        self.inputs = tuple(x.detach().clone().requires_grad_(x.requires_grad) for x in inputs)
        caller = torch.cuda.current_stream()
        side = torch.cuda.Stream()
        side.wait_stream(caller)
        with torch.cuda.stream(side):
            for _ in range(warmups):
                self._clear_grads()
                loss, _ = loss_fn(*self.inputs)
                loss.backward()
        caller.wait_stream(side)
        self._clear_grads()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.loss, self.output = loss_fn(*self.inputs)
            self.loss.backward()

    def _clear_grads(self):
        self.model.zero_grad(set_to_none=True)
        for x in self.inputs:
            x.grad = None

    def replay(self, *inputs):
        """Run the captured step on ``inputs``; returns the static ``(loss, output)``."""
        with torch.no_grad():
            for static, value in zip(self.inputs, inputs):
                if static.shape != value.shape or static.dtype != value.dtype:
                    raise ValueError("the CUDA graph was captured for other input shapes/dtypes")
                static.copy_(value)
        self.graph.replay()
        return self.loss, self.output
