"""Multi-GPU plumbing for the DenseGPA core: one process per GPU.

Every (batch, head) unit is an independent recurrence (no cross-unit term in
fisalt/GPA's src/gpa/attention.py:161-345), so the work shards over units with
no communication in the forward.  Two layouts are supported:

* data parallel (the default of bench.py): every rank owns whole batch rows
  and all heads; parameters are replicated and their gradients are averaged
  once per step with one bucketed all-reduce (NCCL over NVLink on B200);
* head parallel: a rank owns a contiguous head slice of every parameter (see
  ``head_slice`` and ``head_parallel_state_dict``); parameter gradients are then
  disjoint and need no reduction.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def batch_shard(batch: int, world: int, rank: int) -> slice:
    """Contiguous batch rows owned by `rank` (sizes differ by at most one)."""
    base, extra = divmod(batch, world)
    lo = rank * base + min(rank, extra)
    return slice(lo, lo + base + (1 if rank < extra else 0))


def head_slice(heads: int, world: int, rank: int) -> slice:
    """Contiguous heads owned by `rank` under head parallelism."""
    return batch_shard(heads, world, rank)


# parameters whose head axis is dim 1 ([levels or edges, H, ...]); every other DenseGPA
# parameter (per-level lists and relation prefixes) is [H, ...]
_HEAD_DIM1 = ("residual_raw", "count_gain_raw", "moment_gain", "route_mlp_gain", "output_logits",
              "edge_logits", "relation_gain", "relation_decay_raw", "relation_beta_raw")


def head_axis(name: str) -> int:
    """Axis of the head index in the DenseGPA parameter `name` (src/gpa/attention.py:104-135)."""
    return 1 if name.split(".")[0] in _HEAD_DIM1 else 0


def head_parallel_state_dict(state_dict: dict, heads: slice) -> dict:
    """The parameters of a DenseGPA restricted to the head slice `heads`: load it into a
    DenseGPA whose config has ``heads = heads.stop - heads.start`` (all else unchanged).  The
    heads never interact, so that model computes exactly those heads of the full one."""
    out = {}
    for name, t in state_dict.items():
        ax = head_axis(name)
        out[name] = t.narrow(ax, heads.start, heads.stop - heads.start).contiguous()
    return out


def allreduce_gradients(module: torch.nn.Module, group=None, average: bool = True,
                        bucket_bytes: int = 256 << 20) -> int:
    """All-reduce the gradients of `module`'s parameters in flat buckets.

    Returns the number of collectives issued.  Every rank must call this with
    the same set of parameters holding gradients (the same collective order on
    all ranks).
    """
    if not dist.is_available() or not dist.is_initialized():
        return 0
    world = dist.get_world_size(group)
    if world == 1:
        return 0
    grads = [p.grad for p in module.parameters() if p.grad is not None]
    calls = 0
    bucket, size = [], 0
    for g in grads + [None]:
        if g is not None and (not bucket or size + g.numel() * g.element_size() <= bucket_bytes):
            bucket.append(g)
            size += g.numel() * g.element_size()
            continue
        if bucket:
            flat = torch.cat([x.reshape(-1) for x in bucket])
            dist.all_reduce(flat, group=group)
            if average:
                flat /= world
            off = 0
            for x in bucket:
                n = x.numel()
                x.copy_(flat[off:off + n].view_as(x))
                off += n
            calls += 1
        bucket, size = ([g], g.numel() * g.element_size()) if g is not None else ([], 0)
    return calls
