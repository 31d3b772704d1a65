"""Multi-process host logic on CPU: two `gloo` ranks.

bench.py runs one process per GPU, each on its own batch rows, and averages the
parameter gradients with ``gpa_b200.dist.allreduce_gradients``.  These tests
check the sharding and the reduction with the CPU oracle as the per-rank
compute: the averaged gradients of two half-batch ranks must equal the
gradients of the whole batch on one process (the loss is a mean, shards are
equal), whatever the bucket size.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from gpa_b200.dist import (allreduce_gradients, batch_shard, head_axis, head_parallel_state_dict,
                           head_slice)

CFG = oracle.OracleConfig(heads=2, key_dim=8, value_dim=8, slots=(4, 8), chunk_size=4)


class _Params(torch.nn.Module):
    """The oracle's parameter dict as module parameters ('.' is not allowed in names)."""

    def __init__(self, p: dict):
        super().__init__()
        self.p = torch.nn.ParameterDict({k.replace(".", "__"): torch.nn.Parameter(v.clone())
                                         for k, v in p.items()})

    def as_oracle(self) -> dict:
        return {k.replace("__", "."): v for k, v in self.p.items()}


def _inputs(batch=4, length=7):
    g = torch.Generator().manual_seed(3)
    q = oracle.unit(torch.randn(batch, length, CFG.heads, CFG.key_dim, generator=g, dtype=torch.float64))
    k = oracle.unit(torch.randn(batch, length, CFG.heads, CFG.key_dim, generator=g, dtype=torch.float64))
    v = torch.randn(batch, length, CFG.heads, CFG.value_dim, generator=g, dtype=torch.float64)
    return q, k, v


def _params():
    p = oracle.init_parameters(CFG, torch.Generator().manual_seed(0))
    g = torch.Generator().manual_seed(5)
    return {k: (v.double() + 0.02 * torch.randn(v.shape, generator=g, dtype=torch.float64))
            for k, v in p.items()}


def _grads(module, q, k, v):
    module.zero_grad(set_to_none=True)
    out, _ = oracle.forward(CFG, module.as_oracle(), q, k, v)
    out.square().mean().backward()
    return {n: p.grad.clone() for n, p in module.p.items() if p.grad is not None}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, bucket_bytes, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _check(rank, world, bucket_bytes, q)
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, None, repr(e)))
    finally:
        dist.destroy_process_group()


def _check(rank, world, bucket_bytes, q):
    xs = _inputs()
    module = _Params(_params())
    full = _grads(module, *xs)
    rows = batch_shard(xs[0].shape[0], world, rank)
    _grads(module, *(x[rows] for x in xs))
    calls = allreduce_gradients(module, average=True, bucket_bytes=bucket_bytes)
    worst = max(float((module.p[n].grad - full[n]).abs().max() /
                      full[n].abs().max().clamp_min(1e-300)) for n in full)
    q.put((rank, calls, worst))


@pytest.mark.parametrize("bucket_bytes", [256 << 20, 512])
def test_data_parallel_gradients_match_full_batch(bucket_bytes):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, bucket_bytes, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    n_params = len(oracle.init_parameters(CFG))
    assert len(results) == world
    for rank, calls, worst in results:
        assert calls is not None, (rank, worst)
        assert worst < 1e-12, (rank, worst)
        if bucket_bytes >= 1 << 20:
            assert calls == 1
        else:
            assert 1 < calls <= n_params


def test_shards_cover_rows_once():
    for total in (0, 1, 7, 8, 13):
        for world in (1, 2, 3, 8):
            rows = [batch_shard(total, world, r) for r in range(world)]
            seen = [i for s in rows for i in range(total)[s]]
            assert seen == list(range(total))
            sizes = [s.stop - s.start for s in rows]
            assert max(sizes) - min(sizes) <= 1
    assert head_slice(16, 4, 3) == slice(12, 16)


def test_allreduce_without_process_group_is_a_no_op():
    m = torch.nn.Linear(2, 2)
    m(torch.ones(1, 2)).sum().backward()
    before = m.weight.grad.clone()
    assert allreduce_gradients(m) == 0
    assert torch.equal(m.weight.grad, before)


def _head_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        xs = _inputs()
        params = _params()
        full = _Params(params)
        full.zero_grad(set_to_none=True)
        out_full, _ = oracle.forward(CFG, full.as_oracle(), *xs)
        (out_full * out_full).sum().backward()
        hs = head_slice(CFG.heads, world, rank)
        local_cfg = oracle.OracleConfig(**{**CFG.__dict__, "heads": hs.stop - hs.start})
        local = _Params(head_parallel_state_dict(params, hs))
        out, _ = oracle.forward(local_cfg, local.as_oracle(), *(x[:, :, hs] for x in xs))
        (out * out).sum().backward()
        # outputs of all ranks, gathered along heads, are the full model's output
        parts = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(parts, out.contiguous())
        err_out = float((torch.cat(parts, 2) - out_full).abs().max())
        # local gradients are the full gradients' head slice: no reduction needed
        err_grad = 0.0
        for n, p in local.p.items():
            name = n.replace("__", ".")
            if full.p[n].grad is None:  # a parameter the default flags never read
                assert p.grad is None
                continue
            ref = full.p[n].grad.narrow(head_axis(name), hs.start, hs.stop - hs.start)
            err_grad = max(err_grad, float((p.grad - ref).abs().max()))
        q.put((rank, err_out, err_grad))
    except Exception as e:
        q.put((rank, None, repr(e)))
    finally:
        dist.destroy_process_group()


def test_head_parallel_ranks_compute_the_full_model():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_head_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err_out, err_grad in results:
        assert err_out is not None, (rank, err_grad)
        assert err_out < 1e-12 and err_grad < 1e-12, (rank, err_out, err_grad)


def test_head_slices_load_into_a_narrower_model():
    """bench.py --scaling strong builds each rank's model this way: every parameter of the
    full model sliced along its head axis loads strictly into DenseGPA(heads = slice size)."""
    from gpa_b200 import DenseGPA, GPAConfig
    full = DenseGPA(GPAConfig(heads=8, key_dim=16, value_dim=16, slots=(8, 16), chunk_size=4))
    sd = full.state_dict()
    for r in range(4):
        hs = head_slice(8, 4, r)
        part = DenseGPA(GPAConfig(heads=hs.stop - hs.start, key_dim=16, value_dim=16,
                                  slots=(8, 16), chunk_size=4))
        part.load_state_dict(head_parallel_state_dict(sd, hs), strict=True)
        assert torch.equal(part.edge_logits, full.edge_logits[:, hs])
        assert torch.equal(part.center[1], full.center[1][hs])
