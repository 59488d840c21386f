"""Paired serial / overlapped schedule measurement (2+ GPUs, one process per GPU).

    torchrun --nproc-per-node N -m nanospec_b200.experiments.overlap --config qwen \
        --seq-len 128 --anchors 8 --steps 6 [--comm peer|nccl] --output overlap.json

Mirrors the reference experiment (experiments/overlap.py:28-208): the same fixed
synthetic teacher tensors and anchor RNG on every schedule; a bitwise check over 3
steps of raw reduced gradients, hidden states, param/master/m/v (SHA-256 of the
bytes) between the serial and the overlapped schedule; ABBA timing windows with
3 warm-ups each (device time, max over ranks); one profiled step whose kernel
timeline gives the hidden and the exposed communication time.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import statistics
from datetime import timedelta

import torch
import torch.distributed as dist

import nanospec_b200 as N
from nanospec_b200.utils.trace import kernel_events, overlap_summary


def digest(tensors):
    h = hashlib.sha256()
    for t in tensors:
        h.update(memoryview(t.detach().contiguous().cpu().view(torch.uint8).numpy()))
    return h.hexdigest()


def arguments(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--config", default="qwen")
    p.add_argument("--seq-len", type=int, default=128)
    p.add_argument("--anchors", type=int, default=8)
    p.add_argument("--steps", type=int, default=6)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--comm", choices=("peer", "nccl"), default="peer")
    p.add_argument("--output", default="outputs/overlap.json")
    return p.parse_args(argv)


@torch.no_grad()
def measure(args):
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    c = N.DraftConfig.load(N.config_path(args.config))
    o = N.Objective(num_anchors=args.anchors)
    dtype = torch.bfloat16
    g = torch.Generator().manual_seed(args.seed + 1)
    emb = torch.randn(c.vocab_size, c.hidden_size, generator=g, dtype=dtype) * 0.1
    head = torch.randn(c.vocab_size, c.hidden_size, generator=g, dtype=dtype) * 0.1
    model = N.DSpark(c, N.initialize(c, args.seed, dtype), emb, head, device=dev, dtype=dtype,
                     group=dist.group.WORLD, world_size=world, rank=rank)
    if args.comm == "peer":
        model.sharding.enable_peer()
    opt = N.AdamW(model.sharding, lr=1e-5, weight_decay=0.01)
    initial = [s.param.clone() for s in model.sharding]
    gen = torch.Generator(device=dev).manual_seed(args.seed + 1000 + rank)
    ids = torch.randint(c.vocab_size, (1, args.seq_len), device=dev, generator=gen)
    states = [torch.randn(1, args.seq_len, c.hidden_size, device=dev, dtype=dtype, generator=gen)
              for _ in c.target_layer_ids]
    last = torch.randn(1, args.seq_len, c.hidden_size, device=dev, dtype=dtype, generator=gen)
    batch = N.TeacherBatch(states, last)
    mask = torch.ones_like(ids, dtype=torch.float32)
    if rank % 2:
        mask[:, args.seq_len // 2: args.seq_len // 2 + 2] = 0

    def reset():
        torch.cuda.synchronize()
        for s, p0 in zip(model.sharding, initial):
            s.param.copy_(p0)
            s.master.copy_(s.param)
            s.grad.zero_(), s.m.zero_(), s.v.zero_()
            s.grad_zero = True
        opt.steps = 0
        torch.cuda.synchronize()

    def step(overlap, update=True):
        torch.manual_seed(args.seed + rank)
        return N.train(ids, model, o, teacher_batch=batch, loss_mask=mask,
                       optimizer=opt if update else None, overlap=overlap)

    equality = []
    for overlap in (False, True):
        reset()
        rows = []
        for i in range(3):
            r = step(overlap, update=False)
            grads = digest(s.grad for s in model.sharding)
            upd = N.adamw_step(opt, r.metrics.denominator)
            rows.append({"step": i + 1, "loss": r.metrics.loss.item(), "hidden": digest([r.hidden]),
                         "gradients": grads, "optimizer": upd,
                         "state": digest(getattr(s, f) for s in model.sharding for f in ("param", "master", "m", "v"))})
        equality.append(rows)
    identical = equality[0] == equality[1]

    windows = []
    for overlap in (False, True, True, False):
        reset()
        for _ in range(3):
            step(overlap)
        torch.cuda.synchronize()
        dist.barrier()
        times = []
        for _ in range(args.steps):
            dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            step(overlap)
            e1.record()
            torch.cuda.synchronize()
            t = torch.tensor([e0.elapsed_time(e1)], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            times.append(t.item())
        windows.append({"overlap": overlap, "step_ms": times,
                        "peak_allocated_bytes": torch.cuda.max_memory_allocated(dev)})

    trace_summary = None
    trace_path = os.path.splitext(args.output)[0] + f"-trace-rank{rank}.json"
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
        step(True)
        torch.cuda.synchronize()
    prof.export_chrome_trace(trace_path)
    with open(trace_path) as f:
        events = json.load(f)["traceEvents"]
    trace_summary = overlap_summary(kernel_events(events))
    reports = [None] * world
    dist.all_gather_object(reports, {"rank": rank, "identical": identical, "trace": trace_summary,
                                     "serial": equality[0], "overlap": equality[1]})
    model.sharding.close_peer()
    if rank == 0:
        serial = [t for w in windows if not w["overlap"] for t in w["step_ms"]]
        over = [t for w in windows if w["overlap"] for t in w["step_ms"]]
        s_ms, o_ms = statistics.median(serial), statistics.median(over)
        exposed = max(r["trace"]["exposed_comm_us"] for r in reports) / 1000
        result = {
            "passed": all(r["identical"] for r in reports),
            "bitwise_identical": all(r["identical"] for r in reports),
            "serial_median_ms": s_ms, "overlap_median_ms": o_ms, "speedup": s_ms / o_ms,
            "exposed_comm_ms_per_step": exposed,
            "comm": args.comm, "train_gpus": world, "sequence_length": args.seq_len,
            "config": c.to_dict(), "windows": windows,
            "ranks": [{k: v for k, v in r.items() if k in ("rank", "identical")} |
                      {"comm_us": r["trace"]["comm_us"], "exposed_comm_us": r["trace"]["exposed_comm_us"]}
                      for r in reports],
            "measurement": "draft fwd+bwd+AdamW on fixed synthetic teacher tensors; ABBA windows of "
                           f"{args.steps} steps after 3 warm-ups; CUDA-event device time, max over ranks",
        }
        os.makedirs(os.path.dirname(args.output) or ".", exist_ok=True)
        with open(args.output, "w") as f:
            json.dump(result, f, indent=2)
        print(json.dumps({k: v for k, v in result.items() if k not in ("config", "windows", "ranks")}), flush=True)


def main(argv=None):
    args = arguments(argv)
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    try:
        measure(args)
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
