"""The b200 cores inside the all-GPA causal LM (gpa_b200.lm) against the oracle.

A two-layer model (GQA 4/2 heads of 32, slots 16/16/32, chunk 64, 130-token sequences, the
loss in 48-token chunks) runs with per-layer checkpointing on the GPU; its twin replaces each
core by the CPU oracle (tests/lm_oracle.py) and keeps every other module.
  * fp32 end to end: loss within 1e-5 and every parameter gradient within 1e-3 (relative L2) of
    the fp32 twin;
  * bf16 autocast, the training mode: loss within 1e-2 of the fp32 twin;
  * greedy generation: the fused decode (one DecodeSession kernel per layer and token) and the
    one-token forward calls agree on the tokens.
"""
from __future__ import annotations

import pytest
import torch

from gpa_b200.lm import GPALM, GPALMConfig
from lm_oracle import oracle_lm
from parity_util import rel

pytestmark = pytest.mark.gpu

CFG = GPALMConfig(vocab_size=500, hidden_size=128, num_layers=2, num_heads=4, num_kv_heads=2,
                  head_dim=32, intermediate_size=256, slots=(16, 16, 32), chunk_size=64,
                  loss_chunk_size=48)


def _model(seed=0):
    torch.manual_seed(seed)
    m = GPALM(CFG)
    with torch.no_grad():
        for blk in m.blocks:
            blk.attn.conv.normal_(0., .3)
            for w in blk.attn.gpa.query_weight:
                w.normal_(0., .2)
            for name, p in blk.attn.gpa.named_parameters():
                if name.startswith(("inner_prefix", "outer_prefix", "relation_prefix")):
                    p.normal_(0., .02)
    return m


def _grads(m):
    return {n: p.grad.detach().double().cpu() for n, p in m.named_parameters() if p.grad is not None}


def test_lm_training_step_matches_oracle_cores(cpu_threads):
    m = _model()
    twin = oracle_lm(m, dtype=torch.float32)
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, CFG.vocab_size, (2, 130), generator=g)
    twin.train()
    ref, _ = twin(ids, labels=ids)
    ref.backward()
    ref_g = _grads(twin)
    gpu = m.cuda().train()
    gpu.gradient_checkpointing = True
    gpu.autocast = False
    loss, _ = gpu(ids.cuda(), labels=ids.cuda())
    loss.backward()
    got = _grads(gpu)
    assert rel(loss, ref) <= 1e-5
    twin_names = {n.replace("gpa.inner.", "gpa."): n for n in ref_g}
    bad = {n: rel(got[n], ref_g[twin_names[n]]) for n in got
           if not rel(got[n], ref_g[twin_names[n]]) <= 1e-3}
    assert not bad, bad
    gpu.zero_grad(set_to_none=True)
    gpu.autocast = True
    loss16, _ = gpu(ids.cuda(), labels=ids.cuda())
    loss16.backward()
    assert rel(loss16, ref) <= 1e-2


def test_fused_and_stepwise_generation_agree():
    m = _model(seed=2).cuda().eval()
    ids = torch.randint(0, CFG.vocab_size, (3, 70), generator=torch.Generator().manual_seed(3)).cuda()
    a = m.generate(ids, 6, fused_decode=True)
    b = m.generate(ids, 6, fused_decode=False)
    assert a.shape == (3, 6)
    assert torch.equal(a, b)
