"""The all-GPA causal LM (gpa_b200.lm) on the CPU: cache, beam reorder and chunked loss.

The b200 core needs a GPU, so these tests run the model with the oracle in place of its
cores (tests/lm_oracle.py); they check the model's own logic: cached calls partition a
sequence exactly, ``reorder_cache`` / ``batch_repeat_interleave`` move every layer's
GPAState and convolution tail with its batch row (src/gpa/hf_qwen.py:92-115), and the
chunked next-token loss equals the unchunked one.  tests/test_gpu_lm.py checks the b200
cores inside the same model.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from gpa_b200.lm import GPALM, GPALMConfig, num_parameters
from lm_oracle import oracle_lm

SMALL = GPALMConfig(vocab_size=97, hidden_size=32, num_layers=2, num_heads=2, num_kv_heads=1,
                    head_dim=8, intermediate_size=48, slots=(4, 8), chunk_size=4,
                    loss_chunk_size=5)


def _model(cfg=SMALL, seed=0):
    torch.manual_seed(seed)
    m = GPALM(cfg)
    with torch.no_grad():  # non-trivial convolutions and query weights
        for blk in m.blocks:
            blk.attn.conv.normal_(0., .3)
            for w in blk.attn.gpa.query_weight:
                w.normal_(0., .2)
    return oracle_lm(m)


def _hidden_logits(m, ids, cache=None):
    logits, cache = m(ids, cache=cache, use_cache=True)
    return logits, cache


def test_cached_calls_partition_the_sequence():
    m = _model().eval()
    ids = torch.randint(0, SMALL.vocab_size, (2, 11), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        full, _ = m(ids, use_cache=True)
        _, cache = m(ids[:, :6], use_cache=True)
        _, cache = m(ids[:, 6:9], cache=cache, use_cache=True)
        part, cache = m(ids[:, 9:], cache=cache, use_cache=True)
    assert cache.seen_tokens == 11
    assert torch.allclose(part, full, atol=1e-10)


def test_reorder_and_repeat_move_every_cache_row():
    m = _model(seed=2).eval()
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, SMALL.vocab_size, (3, 7), generator=g)
    nxt = torch.randint(0, SMALL.vocab_size, (3, 1), generator=g)
    with torch.no_grad():
        _, cache = m(ids, use_cache=True)
        ref, _ = m(nxt, cache=cache.detach(), use_cache=True)
        perm = torch.tensor([2, 0, 1])
        cache.reorder_cache(perm)
        got, _ = m(nxt[perm], cache=cache, use_cache=True)
        assert torch.allclose(got, ref[perm], atol=1e-10)
        _, cache = m(ids, use_cache=True)
        cache.batch_repeat_interleave(2)
        rep, _ = m(nxt.repeat_interleave(2, 0), cache=cache, use_cache=True)
        assert torch.allclose(rep, ref.repeat_interleave(2, 0), atol=1e-10)


def test_chunked_loss_equals_full_cross_entropy():
    m = _model(seed=4)
    ids = torch.randint(0, SMALL.vocab_size, (2, 13), generator=torch.Generator().manual_seed(5))
    labels = ids.clone()
    labels[0, 4] = -100
    m.train()
    loss, _ = m(ids, labels=labels)
    m.eval()
    with torch.no_grad():
        x = m.embed(ids)
        for blk in m.blocks:
            x, _ = blk(x)
        logits = m.lm_head(m.norm(x))[:, :-1]
        ref = F.cross_entropy(logits.reshape(-1, SMALL.vocab_size), labels[:, 1:].reshape(-1),
                              ignore_index=-100)
    assert torch.allclose(loss.detach(), ref, atol=1e-10)


def test_greedy_generation_matches_stepwise_argmax():
    m = _model(seed=6).eval()
    ids = torch.randint(0, SMALL.vocab_size, (2, 5), generator=torch.Generator().manual_seed(7))
    out = m.generate(ids, 4, fused_decode=False)
    seq = ids
    with torch.no_grad():
        for i in range(4):
            logits, _ = m(seq, use_cache=True)
            tok = logits[:, -1].argmax(-1)
            assert torch.equal(tok, out[:, i])
            seq = torch.cat((seq, tok[:, None]), 1)


def test_qwen_shaped_parameter_count():
    """28 layers, hidden 1024, 16 x 128 query heads (8 key/value), SwiGLU 3072, vocab 151,936,
    tied head, DenseGPA slots 64/64/64/128 per layer: counted on the meta device."""
    with torch.device("meta"):
        m = GPALM(GPALMConfig())
    n = num_parameters(m)
    gpa = num_parameters(m.blocks[0].attn.gpa)
    assert gpa == 6_128_896
    assert 700e6 < n < 800e6, n
