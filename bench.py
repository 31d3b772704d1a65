#!/usr/bin/env python
"""DenseGPA fwd+bwd throughput on B200, one process per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--scaling weak|strong] [--workload train|decode]
    torchrun --nproc-per-node N bench.py --gpus N ...   (N > 1)

Training workload: one DenseGPA layer with H=16, Dk=Dv=128, slots (64,64,64,128),
chunk 64, T=8192, bf16 activations, fp32 state; q, k ~ N(0,1) L2-normalised per
head, v ~ N(0,1), learnable prefixes re-drawn at N(0,0.02); seed 0.  One step =
forward, out.float().square().mean(), backward (every parameter, input and prefix
gradient).
  * weak scaling (default): every rank runs B=8 (data seeded 1000 + rank) and the
    parameter gradients are all-reduced over NCCL once per step (data parallel),
    the only cross-GPU exchange the path has; the all-reduce is timed separately;
  * strong scaling: one global B=8 x H=16 problem, each rank owning a contiguous
    head slice of every parameter and of the inputs (16/N heads, all 8 batch
    rows); head slices never interact, so the step has no collective at all.

Prints one JSON line (rank 0).  ``value`` is the device-timed tokens/s of the
whole job with inputs resident in HBM (inputs are 805 MB per B=8 rank, larger than
the 126 MB L2, and each step streams tens of GB of activations, so no L2 flush is
needed); ``e2e`` is the same step through the public API with the inputs copied
from pinned host memory and the loss read back every step.  ``--impl reference``
times the reference algorithm's CPU implementation (the test oracle, a
restatement of the reference torch backend) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "DenseGPA fwd+bwd tokens/s at 1/2/4/8 B200 (T=8192) + % of roofline"
CFG = dict(heads=16, key_dim=128, value_dim=128, slots=(64, 64, 64, 128), chunk_size=64)
BATCH, LENGTH = 8, 8192
CPU_SAMPLE = dict(batch=2, length=64)  # bounded CPU sample of the same layer
# DRAM bytes per algorithmic byte of tc_bwd_chunk, from an ncu capture of a small case of the
# same kernel (B=1, T=2048 of the same layer); a full launch's traffic is its algorithmic
# bytes times this ratio.
TRAFFIC_RATIO = {"tc_bwd_chunk": 1.00}
# kernels of the chunked GDN scans: tensor-core bound by their algorithmic FLOPs
CHUNK_KERNELS = ("tc_fwd_chunk", "tc5_fwd_chunk", "tc_fwd_state", "tc5_fwd_state", "tc_fwd_out",
                 "tc5_fwd_out", "tc_bwd_local", "tc_bwd_state", "tc5_bwd_state", "tc_bwd_chunk")


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained", p["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


# ------------------------------------------------------------- algorithmic work

def gdn_g(K, V, C):
    """Chunked GDN forward FLOPs per token (A, UT solve, W, U, W S, Q S, QK^T V, K^T U)."""
    return 2 * (3 * K * V + 3 * C * K + 2 * C * V + C * C / 3)


def layer_flops_per_token_head(cfg):
    """Forward FLOPs per token-head; fwd+bwd counts 3x (backward = 2x forward)."""
    D, Dv, C, M = cfg["key_dim"], cfg["value_dim"], cfg["chunk_size"], cfg["slots"]
    f = sum(gdn_g(D, m, C) + gdn_g(m, Dv, C) for m in M)
    f += sum(gdn_g(M[i], M[j], C) for i in range(len(M)) for j in range(len(M)) if i != j)
    f += 2 * sum(4 * D * m + m * Dv + 5 * m * m + 4 * D for m in M)
    return f


def gdn_scans(cfg):
    """(K, V) of every GDN scan of the layer: inner, outer, relations."""
    D, Dv, M = cfg["key_dim"], cfg["value_dim"], cfg["slots"]
    inner = [(D, m) for m in M]
    outer = [(m, Dv) for m in M]
    rel = [(M[i], M[j]) for i in range(len(M)) for j in range(len(M)) if i != j]
    return inner, outer, rel


def kernel_flops(cfg, units, length):
    """Algorithmic FLOPs per training step of each GDN scan kernel (whole step).

    Per block of c tokens with key width K and value width V:
      fwd_chunk   c^2 (2K + V)              (K K^T lower half, UT solve of [V | K])
      fwd_state   4 c K V                   (W = U - Wk S, S += K^T W)
      fwd_out     c^2 K + 2 c K V + c^2 V   (Q K^T, Q S, P W)
      bwd_local   3 c^2 K + 2 c^2 V + 4 c K V
      bwd_state   6 c K V
      bwd_chunk_v c^2 K + 4 c K V + 2 c^2 V
      bwd_chunk_k 5 c^2 K
    """
    c = cfg["chunk_size"]
    nb = -(-length // c)
    inner, outer, rel = gdn_scans(cfg)
    per = {
        "gdn_fwd_chunk": lambda K, V: c * c * (2 * K + V),
        "gdn_fwd_state": lambda K, V: 4 * c * K * V,
        "gdn_fwd_out": lambda K, V: c * c * K + 2 * c * K * V + c * c * V,
        "gdn_bwd_local": lambda K, V: 3 * c * c * K + 2 * c * c * V + 4 * c * K * V,
        "gdn_bwd_state": lambda K, V: 6 * c * K * V,
        "gdn_bwd_chunk_v": lambda K, V: c * c * K + 4 * c * K * V + 2 * c * c * V,
        "gdn_bwd_chunk_k": lambda K, V: 5 * c * c * K,
    }
    allscans = inner + outer + rel
    use = {
        # forward: chunk + state for all scans; out for inner, outer reads, relations
        "gdn_fwd_chunk": allscans + allscans,   # SIMT path: forward + backward recompute
        "gdn_fwd_state": allscans,
        "gdn_fwd_out": allscans,
        "gdn_bwd_local": allscans,
        "gdn_bwd_state": allscans,
        "gdn_bwd_chunk_v": allscans,
        "gdn_bwd_chunk_k": allscans,
    }
    out = {k: units * nb * sum(per[k](K, V) for K, V in use[k]) for k in per}
    # tensor-core variants (bf16 path): the forward keeps U and Wk, so the backward does not
    # recompute fwd_chunk, and one fused kernel does both chunk phases of the backward
    for tk, sk in (("tc_fwd_state", "gdn_fwd_state"), ("tc_fwd_out", "gdn_fwd_out"),
                   ("tc_bwd_local", "gdn_bwd_local"), ("tc_bwd_state", "gdn_bwd_state")):
        out[tk] = out[sk]
    out["tc5_fwd_state"] = out["gdn_fwd_state"]  # the tcgen05 forward sweep
    out["tc5_bwd_state"] = out["gdn_bwd_state"]  # the tcgen05 backward sweep
    out["tc_fwd_chunk"] = out["gdn_fwd_chunk"] // 2
    out["tc5_fwd_chunk"] = out["tc_fwd_chunk"]  # the tcgen05 WY / UT transform
    out["tc5_fwd_out"] = out["tc_fwd_out"]  # the tcgen05 block outputs
    out["tc_bwd_chunk"] = out["gdn_bwd_chunk_v"] + out["gdn_bwd_chunk_k"]
    return out


def kernel_bytes(cfg, units, length):
    """HBM bytes per training step of the intermediates that tc_bwd_chunk streams (this
    design's own fp32 terms, not the layer's algorithmic I/O).

    Per block of c tokens of a (K, V) scan: reads k, Wk, the dk partial and the
    accumulated dk (c K each, fp32), dW, U, v and the accumulated dv (c V each, fp32), W (c V,
    bf16), the state snapshot S and its gradient D (K V each, fp32), T (c^2, fp32; A is formed
    again from k), and the gates and the dG partial (3 c); writes dk (c K), dv (c V), dg and
    dbeta (2 c).
    """
    c = cfg["chunk_size"]
    nb = -(-length // c)
    inner, outer, rel = gdn_scans(cfg)
    per = sum(4 * (2 * K * V + c * c + 5 * c * K + 5 * c * V + 5 * c) + 2 * c * V
              for K, V in inner + outer + rel)
    return {"tc_bwd_chunk": units * nb * per}


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------- b200 arm

def make_model(device, cfg=CFG):
    from gpa_b200 import DenseGPA, GPAConfig
    torch.manual_seed(0)
    model = DenseGPA(GPAConfig(**cfg))
    g = torch.Generator().manual_seed(0)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.startswith(("inner_prefix", "outer_prefix", "relation_prefix")):
                p.copy_(torch.randn(p.shape, generator=g) * .02)
    return model.to(device)


def make_inputs(batch, length, seed, device="cpu", dtype=torch.bfloat16, cfg=CFG):
    g = torch.Generator().manual_seed(seed)
    H, D, Dv = cfg["heads"], cfg["key_dim"], cfg["value_dim"]
    q = torch.randn(batch, length, H, D, generator=g)
    k = torch.randn(batch, length, H, D, generator=g)
    v = torch.randn(batch, length, H, Dv, generator=g)
    q = q / q.norm(dim=-1, keepdim=True)
    k = k / k.norm(dim=-1, keepdim=True)
    return [x.to(dtype).to(device) for x in (q, k, v)]


def reader_bytes_per_token_head(cfg):
    """Standalone dense reader, per (token, head): read the base logits (sum_i M_i), the
    incoming messages (sum_j (L-1) M_j), write the routes (sum_i M_i), all fp32."""
    M, L = cfg["slots"], len(cfg["slots"])
    return 4 * (2 * sum(M) + (L - 1) * sum(M))


def build_rank_model(args, rank, world, device):
    """(model, heads on this rank, batch on this rank) for the scaling mode."""
    from gpa_b200 import DenseGPA, GPAConfig
    from gpa_b200.dist import head_parallel_state_dict, head_slice
    if args.scaling == "weak" or world == 1:
        return make_model(device), CFG["heads"], BATCH
    hs = head_slice(CFG["heads"], world, rank)
    full = make_model("cpu")
    cfg = dict(CFG, heads=hs.stop - hs.start)
    model = DenseGPA(GPAConfig(**cfg))
    model.load_state_dict(head_parallel_state_dict(full.state_dict(), hs))
    return model.to(device), cfg["heads"], BATCH


def run_b200(args, rank, world, local):
    from gpa_b200 import _lib
    from gpa_b200.dist import allreduce_gradients
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    model, heads, batch = build_rank_model(args, rank, world, device)
    cfg = dict(CFG, heads=heads)
    reduce_grads = args.scaling == "weak" and world > 1
    q, k, v = make_inputs(batch, LENGTH, 1000 + rank, device, cfg=cfg)
    for x in (q, k, v):
        x.requires_grad_(True)
    stream = torch.cuda.current_stream()
    ar_events = []  # (start, end) of each timed step's all-reduce

    def step(timed=False):
        model.zero_grad(set_to_none=True)
        for x in (q, k, v):
            x.grad = None
        out, _ = model(q, k, v)
        loss = out.float().square().mean()
        loss.backward()
        if reduce_grads:
            e = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            e[0].record(stream)
            allreduce_gradients(model)
            e[1].record(stream)
            if timed:
                ar_events.append(e)
        return loss

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    launches0 = _lib.launch_count()
    _lib.profile_start()
    with ClockSampler(local) as clocks:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for _ in range(args.steps):
            step(timed=True)
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    prof = _lib.profile_stop()
    launches = _lib.launch_count() - launches0
    ms = ev0.elapsed_time(ev1) / args.steps
    ar_ms = sum(a.elapsed_time(b) for a, b in ar_events) / args.steps if ar_events else 0.0
    ms_all = torch.tensor([ms, ar_ms], device=device)
    if world > 1:
        dist.all_reduce(ms_all, op=dist.ReduceOp.MAX)
    ms, ar_ms = float(ms_all[0].item()), float(ms_all[1].item())

    # end-to-end through the public API with pinned host inputs: every step's q, k, v are
    # copied host -> device (double-buffered, on a copy stream, while the previous step
    # computes, as a training loop's prefetching loader does) and its loss is read back
    hq, hk, hv = (x.detach().cpu().pin_memory() for x in (q, k, v))
    del q, k, v
    h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv))
    copy_stream = torch.cuda.Stream(device)
    bufs = [[torch.empty(x.shape, dtype=x.dtype, device=device) for x in (hq, hk, hv)]
            for _ in range(2)]
    ready = [torch.cuda.Event() for _ in range(2)]

    def issue_copy(i):
        # buffer i % 2 was last read by step i - 2, which the loss read-back has finished
        with torch.cuda.stream(copy_stream):
            for d, h_ in zip(bufs[i % 2], (hq, hk, hv)):
                d.copy_(h_, non_blocking=True)
            ready[i % 2].record(copy_stream)

    def e2e_step(i):
        model.zero_grad(set_to_none=True)
        stream.wait_event(ready[i % 2])
        issue_copy(i + 1)
        xs = [x.detach().requires_grad_() for x in bufs[i % 2]]
        out, _ = model(*xs)
        loss = out.float().square().mean()
        loss.backward()
        if reduce_grads:
            allreduce_gradients(model)
        return loss.item()

    issue_copy(0)
    n_warm = max(1, args.warmup // 2)
    for i in range(n_warm):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier()
    e2e_steps = max(1, args.steps // 2)
    t0 = time.perf_counter()
    ev2, ev3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev2.record(stream)
    for i in range(n_warm, n_warm + e2e_steps):
        e2e_step(i)
    ev3.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max(ev2.elapsed_time(ev3), (time.perf_counter() - t0) * 1e3) / e2e_steps
    e2e_all = torch.tensor([e2e_ms], device=device)
    if world > 1:
        dist.all_reduce(e2e_all, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_all.item())

    strong = args.scaling == "strong"
    tokens = batch * LENGTH * (1 if strong else world)
    value = tokens / (ms / 1e3)
    pk = peaks()
    units = batch * heads
    kf = kernel_flops(cfg, units, LENGTH)
    kb = kernel_bytes(cfg, units, LENGTH)
    per_step_ms = {n: round(t / args.steps, 3) for n, (c, t) in prof.items()}
    # dominant kernel by device time; the chunked-scan kernels are tensor-core bound on their
    # algorithmic FLOPs, timed inside a long step: the sustained bf16 peak is the denominator
    top = max(prof, key=lambda n: prof[n][1])
    n_launch, tot_ms = prof[top]
    step_s = tot_ms / args.steps / 1e3
    lps = n_launch / args.steps
    if top in CHUNK_KERNELS:
        peak = pk["bf16_tflops_sustained"]
        achieved = kf[top] / step_s / 1e12
        roof = {"bound": "tensor", "achieved": round(achieved, 3), "peak": peak,
                "unit": "TFLOP/s", "frac": round(achieved / peak, 5),
                "traffic": round(kb[top] / lps * TRAFFIC_RATIO[top]) if top in TRAFFIC_RATIO else None,
                "traffic_unit": "DRAM bytes per launch",
                "traffic_source": "algorithmic intermediate bytes per launch x the DRAM/algorithmic "
                                  "ratio of an ncu capture of a small case of the same kernel",
                "kernel": top, "launches_per_step": round(lps),
                "avg_launch_ms": round(tot_ms / n_launch, 4), "flops_per_step": kf[top],
                "flops_per_launch": round(kf[top] / lps),
                "peak_which": "bf16_tflops_sustained (kernel timed inside a long step)",
                "peak_source": pk["source"]}
        if top in kb:
            gbs = kb[top] / step_s / 1e9
            roof["intermediates_hbm"] = {
                "bytes_per_step": kb[top], "achieved": round(gbs, 1), "peak": pk["hbm_gbs"],
                "unit": "GB/s", "frac": round(gbs / pk["hbm_gbs"], 4),
                "note": "bytes of this design's own fp32 intermediates (k, Wk, U, dW, S and D "
                        "snapshots, T) that the kernel streams, not the layer's algorithmic I/O"}
    else:
        roof = {"bound": "tensor", "achieved": None, "peak": pk["bf16_tflops_sustained"],
                "unit": "TFLOP/s", "frac": None, "traffic": None, "kernel": top,
                "peak_source": pk["source"]}
    reader = None
    if "tc_bridge" in prof:
        rb = reader_bytes_per_token_head(cfg) * units * LENGTH
        r_s = prof["tc_bridge"][1] / args.steps / 1e3
        reader = {"bound": "hbm", "kernel": "tc_bridge", "bytes_per_step": rb,
                  "bytes_per_token_head": reader_bytes_per_token_head(cfg),
                  "ms_per_step": round(r_s * 1e3, 3), "achieved": round(rb / r_s / 1e9, 1),
                  "peak": pk["hbm_gbs"], "unit": "GB/s",
                  "frac": round(rb / r_s / 1e9 / pk["hbm_gbs"], 4),
                  "note": "forward dense reader (edge mix, centred tanh, route softmax, route MLP "
                          "and query projection of every level) against the standalone reader's "
                          "bytes: base logits and messages read, routes written, fp32"}
    step_flops = 3 * layer_flops_per_token_head(cfg) * heads * batch * LENGTH
    result = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": args.scaling if world > 1 else "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1), q/k L2-normalised; random-init weights, prefixes N(0,0.02))",
        "config": {"workload": "DenseGPA layer fwd+bwd, H=16, Dk=Dv=128, slots 64/64/64/128, "
                               "chunk 64, B=8, T=8192" + (" (global, head-sharded)" if strong else
                                                          " per rank"),
                   "model": "DenseGPA", "global_batch": batch * (1 if strong else world),
                   "seq_len": LENGTH, "heads": CFG["heads"], "heads_per_rank": heads,
                   "key_dim": CFG["key_dim"], "value_dim": CFG["value_dim"],
                   "slots": list(CFG["slots"]), "chunk_size": CFG["chunk_size"],
                   "state_dtype": "fp32",
                   "parallelism": (f"head-parallel {world} (16/{world} heads x all batch rows per "
                                   "rank, no collective)") if strong else
                                  f"dp{world} (batch rows per rank, gradient all-reduce)",
                   "l2": f"inputs {h2d / 1e6:.0f} MB/rank > 126 MB L2; no flush"},
        "e2e": {"value": round(tokens / (e2e_ms / 1e3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
                "note": "each step's inputs copied from pinned host memory on a copy stream "
                        "during the previous step (double buffer); loss read back every step"},
        "gpu_launches": launches,
        "roofline": roof,
        "reader_roofline": reader,
        "step_roofline": {"flops_per_step": step_flops,
                          "achieved_tflops": round(step_flops / (ms / 1e3) / 1e12, 3),
                          "frac_of_bf16_peak": round(step_flops / (ms / 1e3) / 1e12 / pk["bf16_tflops_sustained"], 5)},
        "allreduce_ms_per_step": round(ar_ms, 3) if reduce_grads else None,
        "kernel_ms_per_step": per_step_ms,
        "clocks": clocks.summary(),
    }
    return result


# --------------------------------------------------------------- decode

DECODE_BATCHES = (1, 64, 256)
DECODE_PREFILL = 4096


def decode_bytes_per_unit(cfg):
    """Algorithmic HBM bytes of one decode step per (batch, head) unit: the cache read and
    written once (2 x 4 x S), one read of the frozen snapshots, q/k/v/out in bf16."""
    D, Dv, M = cfg["key_dim"], cfg["value_dim"], cfg["slots"]
    S = sum(D * m + m * Dv + m for m in M) + sum(M[i] * M[j] for i in range(len(M))
                                                  for j in range(len(M)) if i != j)
    frozen = sum(D * m + m * Dv for m in M)
    return 2 * 4 * S + 4 * frozen + 2 * (3 * D + Dv)


def decode_param_bytes(cfg):
    """Per-head parameters read once per step (every unit of a head shares them in L2)."""
    D, M = cfg["key_dim"], cfg["slots"]
    return cfg["heads"] * 4 * sum(2 * D * m + 5 * m * m + 4 * D for m in M)


def run_decode(args):
    """The training layer decoding: prefill 4096 tokens, then one-token steps replayed from a
    CUDA graph at each batch size."""
    from gpa_b200 import _lib
    from gpa_b200.decode import DecodeSession
    dev = torch.device("cuda", 0)
    model = make_model(dev)
    H, D, Dv = CFG["heads"], CFG["key_dim"], CFG["value_dim"]
    per_unit, pbytes = decode_bytes_per_unit(CFG), decode_param_bytes(CFG)
    pk = peaks()
    rows = {}
    batches = tuple(int(b) for b in args.decode_batches.split(","))
    for B in batches:
        g = torch.Generator(device=dev).manual_seed(1000 + B)
        seg = 512 if B <= 64 else 64  # prefill in segments: the forward's workspace scales with B*T
        seg = min(seg, args.prefill)
        with torch.no_grad():
            state = model.initial_state(B, device=dev, dtype=torch.bfloat16)
            for _ in range(args.prefill // seg):
                xs = [torch.randn(B, seg, H, w, device=dev, generator=g) for w in (D, D, Dv)]
                xs[0] = xs[0] / xs[0].norm(dim=-1, keepdim=True)
                xs[1] = xs[1] / xs[1].norm(dim=-1, keepdim=True)
                _, state = model(*(x.bfloat16() for x in xs), state)
            sess = DecodeSession(model, state, torch.bfloat16)
            del state
            torch.cuda.empty_cache()
            steps = max(args.steps, 64)
            host = [[x.cpu().pin_memory() for x in make_inputs(B, 1, 7 + i)] for i in range(8)]
            static = [x.to(dev) for x in host[0]]
            out = sess.capture(*static)
            for i in range(max(args.warmup, 3)):
                sess.replay()
            torch.cuda.synchronize()
            launches0 = _lib.launch_count()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with ClockSampler(0) as clocks:
                e0.record()
                for _ in range(steps):
                    sess.replay()
                e1.record()
                torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / steps
            # end to end: pinned host inputs in, output back, every step
            hout = torch.empty(out.shape, dtype=out.dtype).pin_memory()
            t0 = time.perf_counter()
            e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e2.record()
            for i in range(steps):
                for s_, h_ in zip(static, host[i % len(host)]):
                    s_.copy_(h_, non_blocking=True)
                sess.replay()
                hout.copy_(out, non_blocking=True)
            e3.record()
            torch.cuda.synchronize()
            e2e_ms = max(e2.elapsed_time(e3), (time.perf_counter() - t0) * 1e3) / steps
            U = B * H
            byts = U * per_unit + pbytes
            rows[B] = {"us_per_step": round(ms * 1e3, 2), "tokens_per_s": round(B / ms * 1e3, 1),
                       "e2e_tokens_per_s": round(B / e2e_ms * 1e3, 1),
                       "achieved_gbs": round(byts / (ms / 1e3) / 1e9, 1),
                       "frac": round(byts / (ms / 1e3) / 1e9 / pk["hbm_gbs"], 4),
                       "bytes_per_step": byts, "clocks": clocks.summary()}
            del sess, out, static
            torch.cuda.empty_cache()
    top = rows[batches[-1]]
    Bt = batches[-1]
    h2d = 2 * Bt * H * (2 * D + Dv)
    result = {
        "metric": "DenseGPA decode tokens/s (H=16, Dk=Dv=128, slots 64/64/64/128, prefill 4096, CUDA graph)",
        "value": top["tokens_per_s"], "unit": "tokens/s", "n_gpus": 1, "steps": max(args.steps, 64),
        "warmup": max(args.warmup, 3), "ms_per_step": round(top["us_per_step"] / 1e3, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) q/k/v, random-init weights)",
        "config": {"workload": f"one-token decode steps, B={Bt}", "model": "DenseGPA", "global_batch": Bt,
                   "seq_len": 1, "prefill": args.prefill, "state_dtype": "fp32",
                   "l2": f"cache {Bt * H * per_unit / 1e9:.2f} GB per step > 126 MB L2; no flush"},
        "e2e": {"value": top["e2e_tokens_per_s"], "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": Bt * H * Dv * 2},
        "gpu_launches": 1,
        "roofline": {"bound": "hbm", "achieved": top["achieved_gbs"], "peak": pk["hbm_gbs"],
                     "unit": "GB/s", "frac": top["frac"], "traffic": None, "kernel": "decode_step",
                     "bytes_per_step": top["bytes_per_step"], "peak_source": pk["source"]},
        "by_batch": rows,
        "clocks": top["clocks"],
    }
    return result


# --------------------------------------------------------------- all-GPA LM

def run_lm(args, rank, world, local):
    """Qwen3-0.6B-shaped all-GPA LM: a training step (fwd + bwd, per-layer checkpointing,
    chunked loss; gradients all-reduced over the ranks) at B=8, T=8192 per rank on uniform
    random token ids, then greedy generation of 256 tokens after a 512-token prompt."""
    from gpa_b200 import _lib
    from gpa_b200.dist import allreduce_gradients
    from gpa_b200.lm import GPALM, GPALMConfig, num_parameters
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    torch.manual_seed(0)
    cfg = GPALMConfig()
    model = GPALM(cfg).to(device)
    model.gradient_checkpointing = True
    g = torch.Generator(device=device).manual_seed(1000 + rank)
    ids = torch.randint(0, cfg.vocab_size, (BATCH, LENGTH), device=device, generator=g)
    stream = torch.cuda.current_stream()

    def step():
        model.train()
        model.zero_grad(set_to_none=True)
        loss, _ = model(ids, labels=ids)
        loss.backward()
        allreduce_gradients(model)
        return loss

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    launches0 = _lib.launch_count()
    with ClockSampler(local) as clocks:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            loss = step()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    launches = _lib.launch_count() - launches0
    ms_t = torch.tensor([ms], device=device)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    # end to end: the step's token ids copied from pinned host memory, the loss read back
    host_ids = ids.cpu().pin_memory()
    t0 = time.perf_counter()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    ids.copy_(host_ids, non_blocking=True)
    loss_v = step().item()
    e3.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max(e2.elapsed_time(e3), (time.perf_counter() - t0) * 1e3)
    peak_gb = torch.cuda.max_memory_allocated(device) / 1e9
    # greedy generation: 512-token prompt, 256 new tokens, fused one-kernel decode per layer
    model.eval()
    gen_b, prompt, new = BATCH, 512, 256
    with torch.no_grad():
        p_ids = ids[:gen_b, :prompt].contiguous()
        model.generate(p_ids, 4)
        torch.cuda.synchronize()
        e4, e5 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e4.record(stream)
        model.generate(p_ids, new)
        e5.record(stream)
        torch.cuda.synchronize()
    gen_ms = e4.elapsed_time(e5)
    tokens = BATCH * LENGTH * world
    return {
        "metric": "all-GPA Qwen3-0.6B-shaped LM train-step tokens/s (28 DenseGPA layers, T=8192)",
        "value": round(tokens / (ms / 1e3), 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (uniform random token ids; random-init weights)",
        "config": {"workload": "all-GPA LM train step (fwd+bwd, per-layer checkpointing, chunked CE)",
                   "model": "GPALM 28 x (hidden 1024, 16 heads x 128, 8 KV heads, SwiGLU 3072), "
                            "vocab 151936, DenseGPA slots 64/64/64/128",
                   "parameters": num_parameters(model), "global_batch": BATCH * world,
                   "seq_len": LENGTH, "parallelism": f"dp{world}",
                   "l2": "activations of tens of GB per step > 126 MB L2; no flush"},
        "loss": round(loss_v, 4), "peak_memory_gb": round(peak_gb, 1),
        "e2e": {"value": round(tokens / (e2e_ms / 1e3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": host_ids.numel() * host_ids.element_size(),
                "d2h_bytes_per_step": 4},
        "gpu_launches": launches // max(1, args.steps),
        "generation": {"batch": gen_b, "prompt": prompt, "new_tokens": new,
                       "ms": round(gen_ms, 1),
                       "tokens_per_s": round(gen_b * new / (gen_ms / 1e3), 1),
                       "note": "prompt prefill plus 255 fused decode steps (one DecodeSession "
                               "kernel per layer and token) and the torch projections / MLP"},
        "clocks": clocks.summary(),
    }


# --------------------------------------------------------------- CPU (oracle) arm

def _oracle_cfg(cfg):
    import oracle
    return oracle.OracleConfig(heads=cfg["heads"], key_dim=cfg["key_dim"],
                               value_dim=cfg["value_dim"], slots=cfg["slots"],
                               chunk_size=cfg["chunk_size"])


def cpu_sample_step(threads, dtype=torch.bfloat16, batch=None, length=None):
    """One fwd+bwd of the reference algorithm (oracle) on a bounded CPU sample of the layer."""
    import oracle
    torch.set_num_threads(threads)
    model = make_model("cpu")
    p = {n: t.detach().clone().requires_grad_() for n, t in model.state_dict().items()}
    ocfg = _oracle_cfg(CFG)
    xs = [x.requires_grad_() for x in make_inputs(batch or CPU_SAMPLE["batch"],
                                                   length or CPU_SAMPLE["length"], 1000,
                                                   dtype=dtype)]

    def step():
        for t in list(p.values()) + xs:
            t.grad = None
        out, _ = oracle.forward(ocfg, p, *xs)
        out.float().square().mean().backward()

    return step


def _timed(fn, reps=1):
    fn()
    t0 = time.perf_counter()
    for _ in range(reps):
        fn()
    return (time.perf_counter() - t0) / reps


def cpu_legs(threads):
    """Further CPU legs of the same reference algorithm, each a bounded sample."""
    import oracle
    torch.set_num_threads(threads)
    legs = []
    b, t = CPU_SAMPLE["batch"], CPU_SAMPLE["length"]
    dt = _timed(cpu_sample_step(threads, torch.float32))
    legs.append({"workload": f"training layer fwd+bwd, fp32 activations, B={b}, T={t}",
                 "tokens_per_s": round(b * t / dt, 3), "seconds": round(dt, 3)})
    # the reference's CPU-runnable case: H=4, Dk=32, Dv=48, slots (64,64,64,128), chunk 1,
    # B=2, T=16, fp32; fwd, out.square().mean() bwd, then a one-token decode
    torch.manual_seed(0)
    c1 = oracle.OracleConfig(heads=4, key_dim=32, value_dim=48, slots=(64, 64, 64, 128))
    p1 = {n: v.requires_grad_() for n, v in oracle.init_parameters(c1).items()}
    x1 = [torch.randn(2, 16, 4, d).requires_grad_() for d in (32, 32, 48)]
    x1d = [torch.randn(2, 1, 4, d) for d in (32, 32, 48)]

    def c1_step():
        out, st = oracle.forward(c1, p1, *x1)
        out.square().mean().backward()
        with torch.no_grad():
            oracle.forward(c1, p1, *x1d, oracle.OracleState(
                tuple(tuple(z.detach() for z in lv) for lv in st.levels),
                tuple(z.detach() for z in st.relations), st.position, st.chunk_size,
                st.chunk_offset, None))
    dt = _timed(c1_step)
    legs.append({"workload": "H=4, Dk=32, Dv=48, slots 64/64/64/128, chunk 1, B=2, T=16, fp32: "
                             "fwd+bwd and a one-token decode", "tokens_per_s": round(32 / dt, 3),
                 "seconds": round(dt, 3)})
    # one decode step of the training layer (B=1) after a 64-token prefill, fp32 state
    model = make_model("cpu")
    p = {n: v.detach() for n, v in model.state_dict().items()}
    ocfg = _oracle_cfg(CFG)
    with torch.no_grad():
        _, st = oracle.forward(ocfg, p, *make_inputs(1, 64, 7))
        xs = make_inputs(1, 1, 8)
        dt = _timed(lambda: oracle.forward(ocfg, p, *xs, st), reps=3)
    legs.append({"workload": "training layer, one-token decode step, B=1, after a 64-token "
                             "prefill, bf16 activations / fp32 state",
                 "tokens_per_s": round(1 / dt, 3), "seconds": round(dt, 4)})
    return legs


def cpu_baseline(threads):
    dt = _timed(cpu_sample_step(threads))
    toks = CPU_SAMPLE["batch"] * CPU_SAMPLE["length"]
    return {"value": round(toks / dt, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"oracle (restated reference torch backend) fwd+bwd of the training layer, "
                      f"B={CPU_SAMPLE['batch']}, T={CPU_SAMPLE['length']}, bf16 activations, "
                      f"{dt:.2f} s",
            "legs": cpu_legs(threads)}


def run_reference(args, rank):
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    step = cpu_sample_step(threads)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    toks = CPU_SAMPLE["batch"] * CPU_SAMPLE["length"]
    value = toks / dt
    return {"metric": METRIC, "value": round(value, 3), "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": "DenseGPA layer fwd+bwd, H=16, Dk=Dv=128, slots 64/64/64/128, "
                                   "chunk 64 (bounded CPU sample)",
                       "model": "DenseGPA", "global_batch": CPU_SAMPLE["batch"],
                       "seq_len": CPU_SAMPLE["length"], "parallelism": "cpu"},
            "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": threads,
                             "kind": "port",
                             "sample": f"B={CPU_SAMPLE['batch']}, T={CPU_SAMPLE['length']}"},
            "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def main():
    global BATCH, LENGTH
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=["train", "decode", "lm"], default="train",
                    help="train: layer fwd+bwd at B=8, T=8192 (the headline); decode: one-token "
                         "steps; lm: the all-GPA Qwen-shaped LM train step and generation")
    ap.add_argument("--decode-batches", default=",".join(str(b) for b in DECODE_BATCHES),
                    help="decode: batch sizes (the last one is the headline line)")
    ap.add_argument("--prefill", type=int, default=DECODE_PREFILL,
                    help="decode: prefill length before the steps (default 4096)")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="weak",
                    help="weak: B=8 per rank, data parallel; strong: global B=8 x 16 heads "
                         "split by heads over the ranks")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true",
                    help="train workload on one GPU: skip the decode leg (one-token steps of the "
                         "same layer at B=1/64/256, reported under \"decode\")")
    ap.add_argument("--batch", type=int, default=BATCH,
                    help="per-rank batch (default 8); smaller values are for profiling")
    ap.add_argument("--length", type=int, default=LENGTH,
                    help="sequence length (default 8192); smaller values are for profiling")
    args = ap.parse_args()
    BATCH, LENGTH = args.batch, args.length
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.workload == "decode" and args.impl == "b200":
        if rank == 0:
            print(json.dumps(run_decode(args)), flush=True)
        return
    if args.impl == "reference":
        res = run_reference(args, rank)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(minutes=3),
                                device_id=torch.device("cuda", local))
    if args.workload == "lm":
        res = run_lm(args, rank, world, local)
        if rank == 0:
            print(json.dumps(res), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    res = run_b200(args, rank, world, local)
    if rank == 0:
        if world == 1 and not args.no_decode and (BATCH, LENGTH) == (8, 8192):
            # the decode workload of the same layer (4096-token prefill, one-token steps at
            # B = 1, 64, 256), timed after the training step: CUDA-graph replays of the
            # one-kernel step at each batch size
            torch.cuda.empty_cache()
            dec = run_decode(args)
            res["decode"] = {k: dec[k] for k in ("metric", "value", "unit", "ms_per_step", "e2e",
                                                 "gpu_launches", "roofline", "by_batch", "config")}
        if not args.no_cpu_baseline:
            res["cpu_baseline"] = cpu_baseline(os.cpu_count() or 1)
        print(json.dumps(res), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
