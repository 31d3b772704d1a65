"""All-GPA causal language model shaped like Qwen3-0.6B, on the b200 DenseGPA core.

The caller of the attention core in fisalt/GPA is its Qwen wrapper
(src/gpa/hf_qwen.py:132-407): every self-attention of a Qwen decoder is replaced by a
DenseGPA layer fed by the native q/k/v projections.  This module rebuilds that model
without Hugging Face Transformers, with the same data flow per layer:

* ``q, k, v`` projections (GQA: ``num_kv_heads`` key/value heads), a depthwise short
  causal convolution over the concatenated projections whose last ``conv_width - 1``
  inputs are carried in the cache (src/gpa/hf_qwen.py:117-123, 169-171), per-head RMSNorm
  of q and k, key/value heads repeated to the query heads (:183), the DenseGPA core, and
  the output projection (:192);
* pre-norm residual blocks with a SwiGLU MLP and RMSNorm, a final RMSNorm and a head tied
  to the embedding;
* the training loss summed over 512-token chunks of next-token cross entropy, each chunk
  recomputed in the backward (:388-401), and per-layer activation checkpointing
  (:379-381), which keeps one layer's core workspace alive at a time;
* a cache of per-layer ``GPAState`` plus convolution tails that reorders along the batch
  for beam search (``reorder_cache``, ``batch_repeat_interleave``: :92-115).

The GPA layers use the default flag set of the b200 backend (no control input, product
reader or RSA update), as the hot-path scope allows; query weights start at zero like the
wrapper's "aligned direct query" (:158-160).  Master weights are fp32; ``forward`` runs
the projections and the core in bf16 under autocast.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F
from torch import Tensor, nn
from torch.utils.checkpoint import checkpoint

from .config import GPAConfig
from .core import DenseGPA
from .state import GPAState, _map


@dataclass(frozen=True)
class GPALMConfig:
    vocab_size: int = 151936
    hidden_size: int = 1024
    num_layers: int = 28
    num_heads: int = 16
    num_kv_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 3072
    rms_eps: float = 1e-6
    conv_width: int = 4
    loss_chunk_size: int = 512
    slots: tuple = (64, 64, 64, 128)
    chunk_size: int = 64
    initializer_range: float = 0.02
    tie_embeddings: bool = True

    def __post_init__(self):
        if self.num_heads % self.num_kv_heads:
            raise ValueError("query heads must be divisible by key/value heads")
        if self.conv_width < 1 or self.loss_chunk_size < 1:
            raise ValueError("conv_width and loss_chunk_size must be positive")


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x: Tensor) -> Tensor:
        w = x.float()
        w = w * torch.rsqrt(w.square().mean(-1, keepdim=True) + self.eps)
        return (w * self.weight.float()).to(x.dtype)


def causal_conv(x: Tensor, weight: Tensor, tail: Tensor | None):
    """Depthwise causal convolution over time of x [B,T,C] with weight [C,1,W]; `tail`
    [B,C,W-1] holds the previous inputs (zeros when None).  Returns (y [B,T,C], new tail)."""
    width = weight.shape[-1] - 1
    prefix = x.new_zeros(x.shape[0], x.shape[-1], width) if tail is None else tail.to(x.dtype)
    joined = torch.cat((prefix, x.transpose(1, 2)), -1)
    y = F.conv1d(joined, weight.to(x.dtype), groups=x.shape[-1]).transpose(1, 2)
    return y, joined[:, :, joined.shape[-1] - width:]


@dataclass
class LayerMemory:
    """Per-layer recurrent memory: the GPA cache and the convolution tail."""
    state: GPAState
    tail: Tensor


@dataclass
class GPALMCache:
    """No growing key/value tensors: a GPAState and a short convolution tail per layer."""
    layers: list = field(default_factory=list)
    seen_tokens: int = 0

    def reorder_cache(self, beam_idx: Tensor):
        """Select batch rows (beam search): every cache tensor indexed along dim 0."""
        self.layers = [None if m is None else LayerMemory(
            _map(m.state, lambda x: x.index_select(0, beam_idx.to(x.device))),
            m.tail.index_select(0, beam_idx.to(m.tail.device))) for m in self.layers]

    def batch_repeat_interleave(self, repeats: int):
        """Repeat every batch row `repeats` times (expansion to beams)."""
        self.layers = [None if m is None else LayerMemory(
            _map(m.state, lambda x: x.repeat_interleave(repeats, dim=0)),
            m.tail.repeat_interleave(repeats, dim=0)) for m in self.layers]

    def detach(self) -> "GPALMCache":
        return GPALMCache([None if m is None else LayerMemory(_map(m.state, lambda x: x.detach()),
                                                              m.tail.detach())
                           for m in self.layers], self.seen_tokens)


class GPAAttention(nn.Module):
    def __init__(self, cfg: GPALMConfig):
        super().__init__()
        h, kv, d = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
        self.cfg = cfg
        self.q_proj = nn.Linear(cfg.hidden_size, h * d, bias=False)
        self.k_proj = nn.Linear(cfg.hidden_size, kv * d, bias=False)
        self.v_proj = nn.Linear(cfg.hidden_size, kv * d, bias=False)
        self.o_proj = nn.Linear(h * d, cfg.hidden_size, bias=False)
        self.q_norm = RMSNorm(d, cfg.rms_eps)
        self.k_norm = RMSNorm(d, cfg.rms_eps)
        channels = (h + 2 * kv) * d
        conv = torch.zeros(channels, 1, cfg.conv_width)
        conv[:, :, -1] = 1.  # identity at initialisation
        self.conv = nn.Parameter(conv)
        self.gpa = DenseGPA(GPAConfig(heads=h, key_dim=d, value_dim=d, slots=tuple(cfg.slots),
                                      chunk_size=cfg.chunk_size))
        with torch.no_grad():
            for w in self.gpa.query_weight:
                w.zero_()

    def forward(self, x: Tensor, memory: LayerMemory | None = None):
        cfg = self.cfg
        b, t, _ = x.shape
        h, kv, d = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
        proj = torch.cat((self.q_proj(x), self.k_proj(x), self.v_proj(x)), -1)
        proj, tail = causal_conv(proj, self.conv, None if memory is None else memory.tail)
        q, k, v = proj.split((h * d, kv * d, kv * d), -1)
        q = self.q_norm(q.reshape(b, t, h, d))
        k = self.k_norm(k.reshape(b, t, kv, d))
        v = v.reshape(b, t, kv, d)
        k, v = (y.repeat_interleave(h // kv, dim=2) for y in (k, v))
        # under autocast the projections, hence q, k, v, are bf16
        q, k, v = (y.contiguous() for y in (q, k, v))
        out, state = self.gpa(q, k, v, None if memory is None else memory.state)
        return self.o_proj(out.reshape(b, t, h * d).to(x.dtype)), LayerMemory(state, tail)


class SwiGLU(nn.Module):
    def __init__(self, cfg: GPALMConfig):
        super().__init__()
        self.gate_proj = nn.Linear(cfg.hidden_size, cfg.intermediate_size, bias=False)
        self.up_proj = nn.Linear(cfg.hidden_size, cfg.intermediate_size, bias=False)
        self.down_proj = nn.Linear(cfg.intermediate_size, cfg.hidden_size, bias=False)

    def forward(self, x: Tensor) -> Tensor:
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class GPABlock(nn.Module):
    def __init__(self, cfg: GPALMConfig):
        super().__init__()
        self.input_norm = RMSNorm(cfg.hidden_size, cfg.rms_eps)
        self.attn = GPAAttention(cfg)
        self.post_norm = RMSNorm(cfg.hidden_size, cfg.rms_eps)
        self.mlp = SwiGLU(cfg)

    def forward(self, x: Tensor, memory: LayerMemory | None = None):
        y, memory = self.attn(self.input_norm(x), memory)
        x = x + y
        return x + self.mlp(self.post_norm(x)), memory


class GPALM(nn.Module):
    """Causal LM: ``forward(ids, labels=None, cache=None)`` -> (loss or last logits, cache)."""

    def __init__(self, cfg: GPALMConfig):
        super().__init__()
        self.cfg = cfg
        self.embed = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.blocks = nn.ModuleList(GPABlock(cfg) for _ in range(cfg.num_layers))
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_eps)
        self.lm_head = nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False)
        std = cfg.initializer_range
        with torch.no_grad():
            self.embed.weight.normal_(0., std)
            for blk in self.blocks:
                for lin in (blk.attn.q_proj, blk.attn.k_proj, blk.attn.v_proj, blk.attn.o_proj,
                            blk.mlp.gate_proj, blk.mlp.up_proj, blk.mlp.down_proj):
                    lin.weight.normal_(0., std)
        if cfg.tie_embeddings:
            self.lm_head.weight = self.embed.weight
        else:
            with torch.no_grad():
                self.lm_head.weight.normal_(0., std)
        self.gradient_checkpointing = False
        self.autocast = True  # bf16 projections and core on CUDA; False: fp32 end to end

    def forward(self, ids: Tensor, labels: Tensor | None = None,
                cache: GPALMCache | None = None, use_cache: bool = False):
        cfg = self.cfg
        if ids.ndim != 2 or ids.shape[1] < 1:
            raise ValueError("expected token ids [B, T] with T >= 1")
        if cache is not None and self.training and self.gradient_checkpointing:
            raise ValueError("checkpointed training requires a fresh stream")
        if use_cache and cache is None:
            cache = GPALMCache([None] * cfg.num_layers)
        x = self.embed(ids)
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=x.is_cuda and self.autocast):
            for i, blk in enumerate(self.blocks):
                old = None if cache is None else cache.layers[i]
                if self.training and self.gradient_checkpointing:
                    # reentrant: the layer's forward runs without a graph, so the core's
                    # forward workspace is freed at once and rebuilt in the backward
                    x = checkpoint(lambda y, blk=blk: blk(y)[0], x, use_reentrant=True)
                else:
                    x, mem = blk(x, old)
                    if cache is not None:
                        cache.layers[i] = mem
            x = self.norm(x)
            if cache is not None:
                cache.seen_tokens += ids.shape[1]
            if labels is None:
                return self.lm_head(x[:, -1:]).float(), cache
            if labels.shape != ids.shape:
                raise ValueError("labels must match ids")
            return self._loss(x, labels), cache

    def _loss(self, x: Tensor, labels: Tensor) -> Tensor:
        """Mean next-token cross entropy over labels[:, 1:] != -100, in recomputed chunks."""
        t = x.shape[1]
        count = (labels[:, 1:] != -100).sum().clamp_min(1)
        step = self.cfg.loss_chunk_size

        def ce(h, y):
            logits = self.lm_head(h).float()
            return F.cross_entropy(logits.reshape(-1, logits.shape[-1]), y.reshape(-1),
                                   reduction="sum", ignore_index=-100)

        loss = x.sum() * 0.
        for start in range(0, t - 1, step):
            stop = min(t - 1, start + step)
            h, y = x[:, start:stop], labels[:, start + 1:stop + 1]
            part = checkpoint(ce, h, y, use_reentrant=False) if self.training else ce(h, y)
            loss = loss + part / count
        return loss

    @torch.no_grad()
    def generate(self, ids: Tensor, max_new_tokens: int, fused_decode: bool = True):
        """Greedy continuation of `ids` [B, T]: returns [B, max_new_tokens] token ids.

        The prompt runs as one cached call per layer; each new token then runs every layer
        once: with ``fused_decode`` through a DecodeSession per layer (one kernel per layer
        and token, the cache in fixed buffers), the whole token step replayed from one CUDA
        graph; else through one-token DenseGPA calls."""
        logits, cache = self.forward(ids, use_cache=True)
        nxt = logits[:, -1].argmax(-1)
        out = [nxt]
        if max_new_tokens <= 1:
            return torch.stack(out, 1)
        if not fused_decode:
            for _ in range(max_new_tokens - 1):
                logits, cache = self.forward(nxt[:, None], cache=cache, use_cache=True)
                nxt = logits[:, -1].argmax(-1)
                out.append(nxt)
            return torch.stack(out, 1)
        from .decode import DecodeSession
        sessions = [DecodeSession(blk.attn.gpa, m.state, torch.bfloat16)
                    for blk, m in zip(self.blocks, cache.layers)]
        tails = [m.tail.clone() for m in cache.layers]  # updated in place by every step
        cfg = self.cfg
        h, kv, d = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
        tok = nxt.clone()  # the token fed to the next step; the step overwrites it

        def one_token():
            b = tok.shape[0]
            x = self.embed(tok[:, None])
            with torch.autocast("cuda", dtype=torch.bfloat16):
                for i, (blk, sess) in enumerate(zip(self.blocks, sessions)):
                    a = blk.attn
                    y = blk.input_norm(x)
                    proj = torch.cat((a.q_proj(y), a.k_proj(y), a.v_proj(y)), -1)
                    proj, tail = causal_conv(proj, a.conv, tails[i])
                    tails[i].copy_(tail)
                    q, k, v = proj.split((h * d, kv * d, kv * d), -1)
                    q = a.q_norm(q.reshape(b, 1, h, d))
                    k = a.k_norm(k.reshape(b, 1, kv, d))
                    v = v.reshape(b, 1, kv, d)
                    k, v = (z.repeat_interleave(h // kv, dim=2) for z in (k, v))
                    o = sess.step(*(z.to(torch.bfloat16).contiguous() for z in (q, k, v)))
                    x = x + a.o_proj(o.reshape(b, 1, h * d).to(x.dtype))
                    x = x + blk.mlp(blk.post_norm(x))
                x = self.norm(x)
                tok.copy_(self.lm_head(x[:, -1]).float().argmax(-1))

        # every decode step is the same sequence of launches on fixed buffers: record one in a
        # CUDA graph (after an eager warm-up whose cache updates are undone) and replay it
        live = [t for sess in sessions for t in sess._flat + [sess._offset]] + tails + [tok]
        saved = [t.clone() for t in live]
        one_token()
        torch.cuda.synchronize()
        for t, r in zip(live, saved):
            t.copy_(r)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            one_token()
        for _ in range(max_new_tokens - 1):
            graph.replay()
            out.append(tok.clone())
        return torch.stack(out, 1)


def num_parameters(model: nn.Module) -> int:
    return sum(p.numel() for p in {id(p): p for p in model.parameters()}.values())


__all__ = ["GPALMConfig", "GPALM", "GPALMCache", "LayerMemory", "causal_conv", "num_parameters"]
