"""Command-line training run: ``python -m nanospec_b200`` (one process per GPU).

Flags follow the reference CLI (nanospec/train.py:404-573): ``--train-gpus --steps
--dtype --config --output --checkpoint --seq-len --anchors --seed --learning-rate
--tokens``; additions: ``--target PATH`` (an HF-layout Qwen3.5 checkpoint directory),
``--synthetic-target {tiny,27b}`` (write a random-init checkpoint of that shape and
use it; there is no network for the real weights), ``--no-verifier`` (fixed random
teacher tensors instead of a verifier), ``--comm {peer,nccl}``, ``--backend gloo``
(CPU ranks, for tests) and ``--save-every``.

Each step: every rank calls ``train(ids, model, objective, verifier=teacher,
optimizer=opt)``; training ranks pool (numerator, denominator, accept sums) and
rank 0 prints one JSON row ``{step, loss, accept_len, grad_norm, updated,
denominator, seconds, ms_device, phase_ms}`` (``phase_ms``: time per step phase, max
over the training ranks). At the end the trainers save a checkpoint
(same layout as the reference) and rank 0 writes the JSON report.
"""

from __future__ import annotations

import argparse
import json
import os
import time
from dataclasses import asdict
from pathlib import Path

import torch
import torch.distributed as dist

from . import checkpoint
from .config import TARGET_MODEL, TARGET_REVISION, DraftConfig, Objective, Topology, config_path
from .utils.phases import PhaseTimer
from .engine import TrainResult, train
from .models.draft import DSpark, initialize
from .parallel.node import Node, TeacherBatch
from .parallel.optim import AdamW

__all__ = ["train", "TrainResult", "main", "build_draft", "dummy_ids", "arguments"]


def arguments(argv=None):
    p = argparse.ArgumentParser(prog="python -m nanospec_b200")
    p.add_argument("--train-gpus", type=int, default=1, choices=(1, 2, 4, 8))
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--dtype", choices=("float32", "bfloat16"), default="bfloat16")
    p.add_argument("--config", default="qwen")
    p.add_argument("--output", default="outputs/train.json")
    p.add_argument("--checkpoint", default="")
    p.add_argument("--seq-len", type=int, default=32)
    p.add_argument("--anchors", type=int, default=2)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--learning-rate", type=float, default=None)
    p.add_argument("--tokens", default="", help="optional .pt tensor [samples, seq_len] of token ids")
    p.add_argument("--target", default="", help="HF-layout Qwen3.5 checkpoint directory")
    p.add_argument("--synthetic-target", choices=("", "tiny", "27b"), default="")
    p.add_argument("--no-verifier", action="store_true")
    p.add_argument("--comm", choices=("peer", "nccl"), default="peer")
    p.add_argument("--backend", choices=("nccl", "gloo"), default=None)
    p.add_argument("--save-every", type=int, default=0)
    return p.parse_args(argv)


def build_draft(node, c: DraftConfig, dtype, seed, teacher=None):
    """Draft model on a training rank (None elsewhere); frozen tensors from the verifier."""
    if not node.training:
        return None
    if teacher is not None:
        frozen = teacher.checkpoint.frozen()
        emb = frozen["model.language_model.embed_tokens.weight"]
        head = frozen["lm_head.weight"]
    else:
        g = torch.Generator().manual_seed(seed + 1)
        emb = torch.randn(c.vocab_size, c.hidden_size, generator=g, dtype=dtype) * 0.1
        head = torch.randn(c.vocab_size, c.hidden_size, generator=g, dtype=dtype) * 0.1
    group = node.train_group if node.train_gpus > 1 else None
    return DSpark(c, initialize(c, seed, dtype), emb, head, device=node.device, dtype=dtype, group=group,
                  world_size=node.train_gpus, rank=node.rank)


def dummy_ids(node, c, seq_len, seed):
    """[train_gpus, seq_len] random ids, identical on every rank (device generator)."""
    gen = torch.Generator(device=node.device).manual_seed(seed)
    return torch.randint(0, c.vocab_size, (node.train_gpus, seq_len), device=node.device, generator=gen)


def setup_target(node, c: DraftConfig, args):
    from .models.verifier import (Checkpoint, qwen3_5_27b_text_config, tiny_hybrid_text_config,
                                  write_synthetic_checkpoint)
    from .parallel.handoff import Teacher
    path = args.target
    if not path and args.synthetic_target:
        path = str(Path(args.output).with_suffix("")) + f"-synthetic-{args.synthetic_target}"
        if node.rank == 0 and not os.path.exists(os.path.join(path, "config.json")):
            tc = (qwen3_5_27b_text_config() if args.synthetic_target == "27b" else
                  tiny_hybrid_text_config(hidden=c.target_hidden_size, vocab=c.vocab_size))
            tc["num_hidden_layers"] = max(tc["num_hidden_layers"], c.target_num_hidden_layers)
            tc["layer_types"] = ["full_attention" if (i + 1) % 4 == 0 else "linear_attention"
                                 for i in range(tc["num_hidden_layers"])]
            write_synthetic_checkpoint(path, tc, seed=args.seed, fp8=(args.synthetic_target == "27b"))
        if dist.is_initialized():
            dist.barrier()
    if not path:
        return None
    teacher = Teacher(node, path, c.target_layer_ids, checkpoint=Checkpoint(path))
    tc = teacher.config
    if (c.target_hidden_size, c.vocab_size) != (tc["hidden_size"], tc["vocab_size"]) or \
            c.target_num_hidden_layers > tc["num_hidden_layers"]:
        raise ValueError("Draft configuration does not match the target checkpoint")
    return teacher


@torch.no_grad()
def main(argv=None):
    args = arguments(argv)
    if args.steps < 1:
        raise ValueError("steps must be positive")
    world = int(os.environ.get("WORLD_SIZE", 1))
    topo = Topology(world=world, train_gpus=args.train_gpus)
    node = Node(args.train_gpus, topology=topo, backend=args.backend)
    if node.backend == "nccl" and world > 1 and node.rank == 0:
        from .utils.provenance import preflight
        preflight(world)  # GPU count, all-to-all peer access, NVLink (raises otherwise)
    torch.set_float32_matmul_precision("highest")
    c = DraftConfig.load(config_path(args.config))
    o = Objective(num_anchors=args.anchors)
    dtype = getattr(torch, args.dtype)
    teacher = None if args.no_verifier else setup_target(node, c, args)
    model = build_draft(node, c, dtype, args.seed, teacher)
    lr = args.learning_rate if args.learning_rate is not None else 1e-5
    if lr <= 0:
        raise ValueError("learning-rate must be positive")
    opt = AdamW(model.sharding, lr=lr, lazy_zero=True) if model is not None else None
    if model is not None and node.train_gpus > 1 and args.comm == "peer" and node.device.type == "cuda":
        model.sharding.enable_peer(node.train_group)
    start = checkpoint.restore(args.checkpoint, model, opt, o) if (model is not None and args.checkpoint) else 0
    if world > 1:
        t = torch.tensor([start], device=node.device if node.backend == "nccl" else "cpu", dtype=torch.int64)
        dist.broadcast(t, src=0)
        start = int(t.item())
    data = torch.load(args.tokens, weights_only=True) if args.tokens else None
    if data is not None and (data.ndim != 2 or data.shape[1] != args.seq_len or len(data) < node.train_gpus):
        raise ValueError("--tokens needs at least train_gpus rows with --seq-len columns")
    rows = []
    periodic = None
    if args.save_every and model is not None:
        periodic = checkpoint.Periodic(str(Path(args.output).with_suffix("")) + "-checkpoint", model, opt, o,
                                       every=args.save_every, keep=2)
    for offset in range(args.steps):
        step = start + offset
        if data is None:
            ids = dummy_ids(node, c, args.seq_len, args.seed + step)
        else:
            sel = (torch.arange(node.train_gpus) + step * node.train_gpus) % len(data)
            ids = data[sel].long().to(node.device)
        t0 = time.perf_counter()
        ev0 = ev1 = None
        if node.device.type == "cuda":
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
        torch.manual_seed(args.seed + step * node.train_gpus + node.rank)
        timer = PhaseTimer(node.device)
        if teacher is not None:
            result = train(ids, model, o, verifier=teacher, optimizer=opt, phases=timer)
        elif node.training:
            g = torch.Generator(device=node.device).manual_seed(args.seed + 7 * step + node.rank)
            s = args.seq_len
            tb = TeacherBatch([torch.randn(1, s, c.hidden_size, device=node.device, generator=g).to(dtype)
                               for _ in c.target_layer_ids],
                              torch.randn(1, s, c.hidden_size, device=node.device, generator=g).to(dtype))
            result = train(ids[node.rank:node.rank + 1], model, o, teacher_batch=tb, optimizer=opt, phases=timer)
        else:
            result = None
        if node.training:
            m, upd = result.metrics, result.update
            pooled = torch.stack((m.numerator, m.denominator, m.accept_len_sum, m.accept_len_total)).float()
            if node.train_gpus > 1:
                dist.all_reduce(pooled, group=node.train_group)
            row = {"step": step + 1, "loss": float(pooled[0] / pooled[1].clamp_min(1e-6)),
                   "accept_len": float(pooled[2] / pooled[3].clamp_min(1.0)), **upd}
            if ev1 is not None:
                ev1.record()
                torch.cuda.synchronize()
                row["ms_device"] = ev0.elapsed_time(ev1)
            # device ms per phase, max over the training ranks (the slowest rank sets the pace)
            phase = timer.summary()
            names = ("verifier", "draft_forward", "head", "draft_backward", "optimizer")
            pm = torch.tensor([phase.get(n, 0.0) for n in names], dtype=torch.float64,
                              device=node.device if node.train_gpus > 1 else "cpu")
            if node.train_gpus > 1:
                dist.all_reduce(pm, op=dist.ReduceOp.MAX, group=node.train_group)
            row["phase_ms"] = {n: round(float(v), 3) for n, v in zip(names, pm.tolist()) if n in phase}
            row["seconds"] = time.perf_counter() - t0
            rows.append(row)
            if node.rank == 0:
                print(json.dumps(row), flush=True)
            if periodic is not None and offset + 1 < args.steps:
                periodic.step(step + 1)  # asynchronous: host staging overlaps the next steps
        if world > 1:
            dist.barrier()
    ckpt_path = None
    if periodic is not None:
        periodic.close()
    if node.training:
        ckpt_path = checkpoint.save(str(Path(args.output).with_suffix("")) + "-checkpoint", model, opt, o,
                                    start + args.steps)
        if node.rank == 0:
            out = Path(args.output)
            out.parent.mkdir(parents=True, exist_ok=True)
            out.write_text(json.dumps({
                "config": c.to_dict(), "objective": asdict(o), "target": TARGET_MODEL,
                "target_revision": TARGET_REVISION, "train_gpus": args.train_gpus, "world": world,
                "dtype": args.dtype, "learning_rate": opt.lr, "steps": rows, "checkpoint": ckpt_path,
                "verifier": bool(teacher is not None),
                "provenance": _provenance(node, world),
            }, indent=2))
    if model is not None and world > 1:
        model.sharding.close_peer()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return rows


def _provenance(node, world):
    from .utils.provenance import provenance, source_hashes
    if node.backend == "nccl":
        return provenance(world)
    return {"source_files": source_hashes(), "torch": torch.__version__}


if __name__ == "__main__":
    main()
