"""Draft-training throughput: the reference's headline draft-phase benchmark on B200.

Workload (reference: experiments/overlap.py and VALIDATION.md:22-36): the 5-layer
1.75 B-parameter DSPark draft ("qwen" config) with the frozen 248,320 x 5120 target
embedding and LM head, bf16 with fp32 masters, one row of S=128 tokens and 8 anchors
per training rank, fixed synthetic teacher tensors (random hidden states; the
verifier is excluded, as in the reference's measurement), full forward, CE+KL head,
backward, and AdamW every step. Ranks 0..N-1 all train (FULL_SHARD over N).

Metric: draft-train tokens/s = N * S / step_time, step_time = max over ranks of the
CUDA-event time of K steps / K.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
REF_PATH = os.path.join(ROOT, "baseline", "_ref")
METRIC = "draft-train tokens/s (box, max over ranks)"
# derived from the reference's published overlapped draft-step medians on
# 8xH100 (72.89 ms at N=2, 58.11 ms at N=4; S=128 tokens per rank).
PUBLISHED = {2: 3512.0, 4: 8810.0}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--config", default="qwen")
    p.add_argument("--seq-len", type=int, default=128)
    p.add_argument("--anchors", type=int, default=8)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-count", action="store_true")
    p.add_argument("--no-graph", action="store_true", help="one rank: run eagerly, not as a CUDA graph")
    p.add_argument("--comm", choices=("peer", "nccl"), default="peer",
                   help="N>1: peer-memory kernels over NVLink (default) or NCCL collectives")
    return p.parse_args()


class Clocks:
    """nvidia-smi sampling (every 200 ms) of this rank's GPU during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        rows = [ln.split(",") for ln in self.file.read().strip().splitlines() if ln.strip()]
        os.unlink(self.file.name)
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for name, v in zip(names, r[5:9]):
                    if v.strip() == "Active":
                        reasons.add(name)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def setup_dist(n):
    world = int(os.environ.get("WORLD_SIZE", 1))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}; launch with torchrun --nproc-per-node {n}")
    rank = int(os.environ.get("RANK", 0))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
    return rank, world, local, dev


def synthetic_batch(c, seq, rank, seed, dev, dtype):
    gen = torch.Generator(device=dev).manual_seed(seed + 1000 + rank)
    ids = torch.randint(c.vocab_size, (1, seq), device=dev, generator=gen)
    states = [torch.randn(1, seq, c.hidden_size, device=dev, dtype=dtype, generator=gen)
              for _ in c.target_layer_ids]
    last = torch.randn(1, seq, c.hidden_size, device=dev, dtype=dtype, generator=gen)
    mask = torch.ones(1, seq, device=dev, dtype=torch.float32)
    if rank % 2:  # unequal supervision exercises global token normalisation
        mask[:, seq // 2: seq // 2 + 2] = 0
    return ids, states, last, mask


def max_over_ranks(x, world, dev):
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def build(impl, c, world, rank, dev, dtype, seed):
    """Returns (model, optimizer, train_fn, TeacherBatch class)."""
    g = torch.Generator().manual_seed(seed + 1)
    emb = torch.randn(c.vocab_size, c.hidden_size, generator=g, dtype=dtype) * 0.1
    head = torch.randn(c.vocab_size, c.hidden_size, generator=g, dtype=dtype) * 0.1
    group = dist.group.WORLD if world > 1 else None
    if impl == "ours":
        import nanospec_b200 as N
        state = N.initialize(c, seed, dtype)
        model = N.DSpark(c, state, emb, head, device=dev, dtype=dtype, group=group, world_size=world, rank=rank)
        opt = N.AdamW(model.sharding, lr=1e-5, weight_decay=0.01, lazy_zero=True)
        return model, opt, N.train, N.TeacherBatch
    sys.path.insert(0, REF_PATH)
    from nanospec.distributed import TeacherBatch
    from nanospec.dspark import DSpark, initialize
    from nanospec.shard import AdamW
    from nanospec.train import train
    torch.set_float32_matmul_precision("highest")
    state = initialize(c, seed, dtype)
    model = DSpark(c, state, emb, head, device=dev, dtype=dtype, group=group, world_size=world, rank=rank)
    opt = AdamW(model.sharding, lr=1e-5, weight_decay=0.01)
    return model, opt, train, TeacherBatch


def profile_step(step_fn):
    """One profiled step (outside the timed region): (kernels of this repository's
    extension launched, communication ms, exposed communication ms). Exposed
    communication is the part of the communication kernels' and peer copies' union
    not covered by compute (utils.trace)."""
    from torch.profiler import ProfilerActivity, profile

    from nanospec_b200.utils.trace import kernel_events, overlap_summary
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step_fn()
        torch.cuda.synchronize()
    n = sum(1 for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA and "ns::" in e.name)
    try:
        with tempfile.TemporaryDirectory() as d:
            path = os.path.join(d, "trace.json")
            prof.export_chrome_trace(path)
            with open(path) as f:
                summary = overlap_summary(kernel_events(json.load(f)["traceEvents"]))
        return n, summary["comm_us"] / 1000.0, summary["exposed_comm_us"] / 1000.0
    except (OSError, ValueError, KeyError) as exc:  # the analysis is optional; the count is not
        print(f"bench: trace analysis skipped ({exc})", file=sys.stderr)
        return n, float("nan"), float("nan")


def main():
    args = parse()
    n = args.gpus
    if args.impl == "reference":
        if n not in (1, 2, 4):
            _print_unavailable(n, "the reference's Shard supports 1, 2 or 4 training ranks "
                                  "(nanospec/shard.py:48-49)", args)
            return
        if not os.path.isdir(os.path.join(REF_PATH, "nanospec")):
            _print_unavailable(n, "reference not installed in baseline/_ref", args)
            return
    rank, world, local, dev = setup_dist(n)
    if args.impl == "ours":
        import nanospec_b200 as N
        c = N.DraftConfig.load(N.config_path(args.config))
        from nanospec_b200.ops._ext import cuda_ops
        cuda_ops()  # fail loudly if the extension is missing
    else:
        sys.path.insert(0, REF_PATH)
        from nanospec.config import DraftConfig, Objective as RObjective
        c = DraftConfig.load(os.path.join(ROOT, "nanospec_b200", "configs", f"{args.config}.json"))
    dtype = torch.bfloat16
    model, opt, train_fn, TB = build(args.impl, c, world, rank, dev, dtype, args.seed)
    if args.impl == "ours":
        o = N.Objective(num_anchors=args.anchors)
    else:
        o = RObjective(num_anchors=args.anchors)
    if args.impl == "ours" and world > 1 and args.comm == "peer":
        model.sharding.enable_peer()
    ids, states, last, mask = synthetic_batch(c, args.seq_len, rank, args.seed, dev, dtype)
    batch = TB(states, last)

    graphed = None
    if args.impl == "ours" and world == 1 and not args.no_graph:
        # Single rank: the whole step (fwd, head, bwd, AdamW) replays as one CUDA graph.
        from nanospec_b200.graphs import GraphedStep
        torch.manual_seed(args.seed + rank)
        graphed = GraphedStep(model, o, opt, ids, batch, loss_mask=mask, warmup=2)

    def step():
        if graphed is not None:
            return graphed.step()
        torch.manual_seed(args.seed + rank)
        return train_fn(ids, model, o, teacher_batch=batch, loss_mask=mask, optimizer=opt)

    with torch.no_grad():
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        clocks = Clocks(local)
        clocks.start()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        start.record()
        for _ in range(args.steps):
            result = step()
        end.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        local_ms = start.elapsed_time(end) / args.steps
        clk = clocks.stop()
        ms = max_over_ranks(local_ms, world, dev)
        loss = float(result.metrics.loss)

        # End-to-end through the public API: pinned host inputs -> device every step,
        # loss read back every step.
        e2e = None
        if not args.no_e2e:
            h_ids = ids.cpu().pin_memory()
            h_states = [s.cpu().pin_memory() for s in states]
            h_last = last.cpu().pin_memory()
            h_mask = mask.cpu().pin_memory()
            bi = sum(t.numel() * t.element_size() for t in (h_ids, h_last, h_mask, *h_states))
            losses = torch.empty(args.steps, dtype=torch.float32).pin_memory()
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            for i in range(args.steps):
                d_ids = h_ids.to(dev, non_blocking=True)
                d_states = [s.to(dev, non_blocking=True) for s in h_states]
                d_last = h_last.to(dev, non_blocking=True)
                d_mask = h_mask.to(dev, non_blocking=True)
                if graphed is not None:
                    r = graphed.step(ids=d_ids, hidden_states=d_states, last_hidden=d_last, loss_mask=d_mask)
                else:
                    torch.manual_seed(args.seed + rank)
                    r = train_fn(d_ids, model, o, teacher_batch=TB(d_states, d_last), loss_mask=d_mask,
                                 optimizer=opt)
                losses[i] = r.metrics.loss.float().cpu()
            e1.record()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world, dev)
            wall_ms = max_over_ranks((time.perf_counter() - t0) * 1000 / args.steps, world, dev)
            e2e = {"value": round(n * args.seq_len / (e2e_ms / 1000), 1), "unit": "tokens/s",
                   "h2d_bytes_per_step": bi, "d2h_bytes_per_step": 4 + 8,
                   "ms_per_step": round(e2e_ms, 3), "wall_ms_per_step": round(wall_ms, 3)}

        launches = comm_ms = exposed_ms = None
        if args.impl == "ours" and not args.no_count:
            per_step, comm, exposed = profile_step(step)
            launches = per_step * args.steps
            comm_ms = max_over_ranks(comm, world, dev)
            exposed_ms = max_over_ranks(exposed, world, dev)
    value = n * args.seq_len / (ms / 1000)
    if rank == 0:
        out = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": "tokens/s",
            "n_gpus": n,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 3),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": round(value / PUBLISHED[n], 3) if n in PUBLISHED else None,
            "dtype": "bf16",
            "data": "synthetic: random token ids and random teacher hidden states; random-init weights",
            "config": {
                "model": f"DSpark {args.config} draft ({c.num_hidden_layers} layers, hidden {c.hidden_size}, "
                         f"vocab {c.vocab_size}) + frozen target embed/LM head",
                "global_batch": n, "seq_len": args.seq_len, "anchors": args.anchors,
                "block_size": 7, "parallelism": f"fsdp{n}" if n > 1 else "single",
                "comm": (args.comm if args.impl == "ours" else "nccl") if n > 1 else None,
                "cuda_graph": graphed is not None,
                "optimizer": "AdamW fp32 masters, lr 1e-5, wd 0.01",
                "l2": "per-step working set (weights, fp32 masters and moments) far exceeds the 126 MB L2",
            },
            "loss": loss,
            "clocks": clk,
            "e2e": e2e,
            "gpu_launches": launches,
            "comm_ms_per_step": None if comm_ms is None or comm_ms != comm_ms else round(comm_ms, 3),
            "exposed_comm_ms_per_step": None if exposed_ms is None or exposed_ms != exposed_ms else round(exposed_ms, 3),
        }
        if args.impl == "reference":
            out["impl"] = "reference"
        print(json.dumps(out), flush=True)
    if world > 1:
        if args.impl == "ours":
            model.sharding.close_peer()
        dist.barrier()
        dist.destroy_process_group()


def _print_unavailable(n, why, args):
    rank = int(os.environ.get("RANK", 0))
    if rank == 0:
        print(json.dumps({"impl": "reference", "unavailable": why, "n_gpus": n, "metric": METRIC}), flush=True)


if __name__ == "__main__":
    main()
