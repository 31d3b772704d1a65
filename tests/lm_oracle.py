"""Test infrastructure: GPALM with the CPU oracle in place of each b200 DenseGPA core.

``oracle_lm(model)`` returns a copy of a GPALM whose attention cores call the oracle
(``oracle.forward``) with the same parameters; everything around the core (projections,
convolution, norms, MLP, loss, cache) is the product's own code, so the pair checks the b200
core inside the model it serves.
"""
from __future__ import annotations

import copy

import torch
from torch import nn

import oracle
from parity_util import oracle_config


class OracleCore(nn.Module):
    def __init__(self, gpa):
        super().__init__()
        self.inner = gpa
        self.ocfg = oracle_config(gpa)

    def forward(self, q, k, v, state=None):
        p = dict(self.inner.named_parameters())
        return oracle.forward(self.ocfg, p, q, k, v, state)


def oracle_lm(model, device="cpu", dtype=torch.float64):
    twin = copy.deepcopy(model).to(device)
    for blk in twin.blocks:
        blk.attn.gpa = OracleCore(blk.attn.gpa)
    if dtype is not None:
        twin = twin.to(dtype)
    return twin
