"""Draft-training throughput on B200: the full verifier + draft step, or the draft phase alone.

Default workload ("full", the target configuration): a Qwen3.5-27B-shaped FP8
verifier (64 layers, 3:1 gated-DeltaNet : full attention, hidden 5120, FFN 17408,
vocab 248,320, e4m3 weights with 128x128 block scales, random init) runs on each
rank's batch row, its captured layers {1, 16, 31, 46, 61} and final normed hidden
state feed the 5-layer 1.75 B-parameter DSPark draft ("qwen" config), and the draft
trains with the 0.1 CE + 0.9 KL objective and AdamW: one
``train(ids, model, objective, verifier=teacher, optimizer=opt)`` per step.
Per rank: one row of S=4096 tokens with 32 anchors (block 7). Layout
``--layout replicated`` (default): every GPU holds a full verifier replica (27 GB
of FP8 weights fit easily in 180 GB) and trains; ``--layout split`` is the
reference's layout (half the GPUs run contiguous verifier partitions, half train).

``--workload draft`` is the reference's draft-phase benchmark
(experiments/overlap.py, VALIDATION.md:22-36): fixed synthetic teacher tensors,
S=128, A=8.

Metric: draft-train tokens/s = (training ranks) * S / step_time, where step_time
is the max over ranks of the CUDA-event time of K steps / K.

``--impl reference`` runs the unmodified reference package (installed under
baseline/_ref) through its own ``train()``: for the full workload it reads a
synthetic 27B-shaped checkpoint in the Hugging Face layout (written once, then
reused) through the reference's ``Teacher``.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...
"""

from __future__ import annotations

import argparse
import json
import os
import shutil
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
# Published reference numbers for the same metric: the draft phase (S=128, A=8, fixed
# teacher tensors) on 8xH100, from the overlapped step medians 72.89 ms (N=2) and
# 58.11 ms (N=4). The full step has no published number at S=4096.
PUBLISHED = {"draft": {2: 3512.0, 4: 8810.0}, "full": {}}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--workload", choices=("full", "draft"), default="full")
    p.add_argument("--layout", choices=("replicated", "split"), default="replicated",
                   help="full workload: verifier replica on every GPU, or the reference's split")
    p.add_argument("--config", default="qwen")
    p.add_argument("--seq-len", type=int, default=None, help="default 4096 (full) / 128 (draft)")
    p.add_argument("--anchors", type=int, default=None, help="default 32 (full) / 8 (draft)")
    p.add_argument("--verifier-layers", type=int, default=64)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-count", action="store_true")
    p.add_argument("--no-graph", action="store_true", help="one rank: run eagerly, not as a CUDA graph")
    p.add_argument("--kernel-table", action="store_true",
                   help="ours: print the device time of every kernel of one step to stderr")
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


def setup_dist(n, timeout_s=600):
    world = int(os.environ.get("WORLD_SIZE", 1))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}; launch with torchrun --nproc-per-node {n}")
    rank = int(os.environ.get("RANK", 0))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1 and not dist.is_initialized():
        dist.init_process_group("nccl", timeout=timedelta(seconds=timeout_s), device_id=dev)
    return rank, world, local, dev


def max_over_ranks(x, world, dev):
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


# ----------------------------------------------------------------------------- workloads
class Workload:
    """What one rank runs per step. ``step(ids)`` -> TrainResult (or None off the trainers)."""

    tokens_per_step = 0          # training ranks * S
    inputs = ()                  # device tensors that are host inputs of a real step
    graphed = False

    def step(self, *inputs):
        raise NotImplementedError

    def loss(self, result):
        if result is None or result.metrics is None:
            return torch.zeros((), device="cuda")
        return result.metrics.loss


def synthetic_teacher(c, seq, rank, seed, dev, dtype):
    gen = torch.Generator(device=dev).manual_seed(seed + 1000 + rank)
    ids = torch.randint(c.vocab_size, (1, seq), device=dev, generator=gen)
    states = [torch.randn(1, seq, c.hidden_size, device=dev, dtype=dtype, generator=gen)
              for _ in c.target_layer_ids]
    last = torch.randn(1, seq, c.hidden_size, device=dev, dtype=dtype, generator=gen)
    mask = torch.ones(1, seq, device=dev, dtype=torch.float32)
    if rank % 2:  # unequal supervision exercises global token normalisation
        mask[:, seq // 2: seq // 2 + 2] = 0
    return ids, states, last, mask


class DraftWorkload(Workload):
    """The reference's draft-phase benchmark: fixed teacher tensors, the draft trains."""

    def __init__(self, args, impl, world, rank, dev):
        dtype = torch.bfloat16
        self.args, self.rank = args, rank
        g = torch.Generator().manual_seed(args.seed + 1)
        if impl == "ours":
            import nanospec_b200 as N
            c = N.DraftConfig.load(N.config_path(args.config))
        else:
            from nanospec.config import DraftConfig
            c = DraftConfig.load(os.path.join(ROOT, "nanospec_b200", "configs", f"{args.config}.json"))
        self.c = c
        emb = torch.randn(c.vocab_size, c.hidden_size, generator=g, dtype=dtype) * 0.1
        head = torch.randn(c.vocab_size, c.hidden_size, generator=g, dtype=dtype) * 0.1
        group = dist.group.WORLD if world > 1 else None
        if impl == "ours":
            import nanospec_b200 as N
            self.model = N.DSpark(c, N.initialize(c, args.seed, dtype), emb, head, device=dev, dtype=dtype,
                                  group=group, world_size=world, rank=rank)
            self.opt = N.AdamW(self.model.sharding, lr=1e-5, weight_decay=0.01, lazy_zero=True)
            self.o = N.Objective(num_anchors=args.anchors)
            self.train, self.TB = N.train, N.TeacherBatch
            if world > 1 and args.comm == "peer":
                self.model.sharding.enable_peer()
        else:
            from nanospec.distributed import TeacherBatch
            from nanospec.dspark import DSpark, initialize
            from nanospec.config import Objective
            from nanospec.shard import AdamW
            from nanospec.train import train
            self.model = DSpark(c, initialize(c, args.seed, dtype), emb, head, device=dev, dtype=dtype,
                                group=group, world_size=world, rank=rank)
            self.opt = AdamW(self.model.sharding, lr=1e-5, weight_decay=0.01)
            self.o = Objective(num_anchors=args.anchors)
            self.train, self.TB = train, TeacherBatch
        ids, states, last, mask = synthetic_teacher(c, args.seq_len, rank, args.seed, dev, dtype)
        self.inputs = (ids, last, mask, *states)
        self.tokens_per_step = world * args.seq_len
        self.gstep = None
        if impl == "ours" and world == 1 and not args.no_graph:
            # Single rank: the whole step (fwd, head, bwd, AdamW) replays as one CUDA graph.
            from nanospec_b200.graphs import GraphedStep
            torch.manual_seed(args.seed + rank)
            self.gstep = GraphedStep(self.model, self.o, self.opt, ids, self.TB(states, last), loss_mask=mask,
                                     warmup=2)
            self.graphed = True

    def step(self, ids, last, mask, *states):
        if self.gstep is not None:
            return self.gstep.step(ids=ids, hidden_states=list(states), last_hidden=last, loss_mask=mask)
        torch.manual_seed(self.args.seed + self.rank)
        return self.train(ids, self.model, self.o, teacher_batch=self.TB(list(states), last), loss_mask=mask,
                          optimizer=self.opt)

    def close(self, world):
        if world > 1 and hasattr(self.model.sharding, "close_peer"):
            self.model.sharding.close_peer()


def synthetic_checkpoint_dir(args, layers):
    base = os.environ.get("NANOSPEC_SYNTH_CKPT_DIR", tempfile.gettempdir())
    return os.path.join(base, f"nanospec_synth_qwen35_27b_L{layers}_seed{args.seed}")


def ensure_synthetic_checkpoint(path, text_config, seed, rank, world, dev):
    """Rank 0 writes the random-init HF-layout checkpoint once (generated on its GPU)."""
    done = os.path.join(path, "complete")
    if rank == 0 and not os.path.exists(done):
        need = 1.15 * sum(_tensor_bytes(text_config))
        parent = os.path.dirname(path) or "."
        free = shutil.disk_usage(parent).free
        if free < need:
            raise RuntimeError(f"need {need / 1e9:.0f} GB free under {parent} for the synthetic checkpoint, "
                               f"have {free / 1e9:.0f} GB")
        from nanospec_b200.models.verifier import write_synthetic_checkpoint
        write_synthetic_checkpoint(path, text_config, seed=seed, fp8=True, device=dev)
        open(done, "w").write("ok\n")
    if world > 1:
        dist.barrier()


def _tensor_bytes(tc):
    from nanospec_b200.models.verifier import layer_tensor_shapes
    h, v = tc["hidden_size"], tc["vocab_size"]
    yield 2 * 2 * h * v
    for i in range(tc["num_hidden_layers"]):
        for shape, quant in layer_tensor_shapes(tc, i).values():
            n = 1
            for d in shape:
                n *= d
            yield n * (1 if quant else 2)


def reference_node(world, rank, dev):
    """The reference's ``Node`` for a box of ``world`` GPUs.

    With 8 GPUs this is the reference's own constructor (4 training ranks, 4
    verifier partitions). Its constructor refuses any other world size
    (nanospec/distributed.py:20-21); for 1, 2 and 4 GPUs the same object is built
    with every GPU training and the verifier partitioned over all of them (the
    reference's pipeline and broadcast code is unchanged and runs as written).
    """
    from nanospec.distributed import Node
    if world == 8:
        return Node(4)
    node = Node.__new__(Node)
    node.rank, node.world, node.device = rank, world, dev
    if not dist.is_initialized():
        # A one-process group: the reference's verifier path calls barriers and broadcasts.
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(29500 + (os.getpid() % 2000)))
        os.environ.setdefault("RANK", str(rank))
        os.environ.setdefault("WORLD_SIZE", str(world))
        dist.init_process_group("nccl", timeout=timedelta(minutes=30), device_id=dev)
    node.train_gpus = world
    node.train_group = dist.new_group(list(range(world)), backend="nccl")
    node.training = True
    node.inference_ranks = list(range(world))
    return node


class FullWorkload(Workload):
    """Verifier + draft: one ``train(ids, model, o, verifier=teacher, optimizer=opt)`` per step."""

    def __init__(self, args, impl, world, rank, dev):
        dtype = torch.bfloat16
        self.args, self.rank, self.world = args, rank, world
        from nanospec_b200.models.verifier import qwen3_5_27b_text_config
        tc = qwen3_5_27b_text_config()
        if args.verifier_layers != tc["num_hidden_layers"]:
            tc["num_hidden_layers"] = args.verifier_layers
            tc["layer_types"] = tc["layer_types"][:args.verifier_layers]
        self.tc = tc
        if impl == "ours":
            import nanospec_b200 as N
            from nanospec_b200.parallel.handoff import Teacher
            c = N.DraftConfig.load(N.config_path(args.config))
            if args.verifier_layers != 64:
                c = _shrink_targets(N.DraftConfig, c, args.verifier_layers)
            if args.layout == "replicated":
                topo = N.Topology.replicated(world)
            else:
                topo = N.Topology.for_world(world)
            node = N.Node(topo.train_gpus, topology=topo)
            self.node = node
            g = torch.Generator(device=dev).manual_seed(args.seed + 1)
            # The frozen target embedding and LM head are shared by the verifier and the draft.
            emb = (torch.randn(c.vocab_size, c.hidden_size, device=dev, generator=g) * 0.02).to(dtype)
            head = (torch.randn(c.vocab_size, c.hidden_size, device=dev, generator=g) * 0.02).to(dtype)
            self.teacher = Teacher.random(node, tc, c.target_layer_ids, seed=args.seed, embed=emb, lm_head=head)
            self.model = None
            if node.training:
                group = node.train_group if node.train_gpus > 1 else None
                self.model = N.DSpark(c, N.initialize(c, args.seed, dtype), emb, head, device=dev, dtype=dtype,
                                      group=group, world_size=node.train_gpus, rank=rank)
                self.opt = N.AdamW(self.model.sharding, lr=1e-5, weight_decay=0.01, lazy_zero=True)
                if node.train_gpus > 1 and args.comm == "peer":
                    self.model.sharding.enable_peer(node.train_group)
            else:
                self.opt = None
            self.o = N.Objective(num_anchors=args.anchors)
            self.train = N.train
            ntrain = node.train_gpus
        else:
            from nanospec.config import DraftConfig, Objective
            from nanospec.distributed import Teacher
            from nanospec.shard import AdamW
            from nanospec.train import build_draft, train
            torch.set_float32_matmul_precision("highest")
            c = DraftConfig.load(os.path.join(ROOT, "nanospec_b200", "configs", f"{args.config}.json"))
            if args.verifier_layers != 64:
                c = _shrink_targets(DraftConfig, c, args.verifier_layers)
            node = reference_node(world, rank, dev)
            self.node = node
            path = synthetic_checkpoint_dir(args, tc["num_hidden_layers"])
            ensure_synthetic_checkpoint(path, tc, args.seed, rank, world, dev)
            self.teacher = Teacher(node, path, c.target_layer_ids)
            self.model = build_draft(node, c, dtype, args.seed, self.teacher)
            self.opt = AdamW(self.model.sharding, lr=1e-5, weight_decay=0.01) if self.model is not None else None
            self.o = Objective(num_anchors=args.anchors)
            self.train = train
            ntrain = node.train_gpus
        self.c = c
        self.ntrain = ntrain
        gen = torch.Generator(device=dev).manual_seed(args.seed + 7)
        ids = torch.randint(c.vocab_size, (ntrain, args.seq_len), device=dev, generator=gen)
        self.inputs = (ids,)
        self.tokens_per_step = ntrain * args.seq_len

    def step(self, ids, phases=None):
        torch.manual_seed(self.args.seed + self.rank)
        kw = {"phases": phases} if phases is not None else {}
        return self.train(ids, self.model, self.o, verifier=self.teacher, optimizer=self.opt, **kw)

    def phase_ms(self, dev):
        """Device ms per phase of one more step (ours only): verifier, draft fwd, head, bwd, AdamW."""
        from nanospec_b200.utils.phases import PhaseTimer
        timer = PhaseTimer(dev)
        self.step(*self.inputs, phases=timer)
        return {k: round(v, 2) for k, v in timer.summary().items()}

    def close(self, world):
        if self.model is not None and world > 1 and hasattr(self.model.sharding, "close_peer"):
            self.model.sharding.close_peer()


def _shrink_targets(cls, c, layers):
    """A draft config whose capture layers fit a verifier of ``layers`` layers (quick runs)."""
    d = c.to_dict()
    d["target_num_hidden_layers"] = layers
    d["target_layer_ids"] = [min(i, layers - 1) for i in d["target_layer_ids"]]
    return cls(**d)


# ----------------------------------------------------------------------------- measurement
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


def _kernel_table(step_fn, top=40):
    """Device microseconds per kernel name over one step (torch.profiler), to stderr."""
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step_fn()
        torch.cuda.synchronize()
    agg = {}
    for e in prof.events():
        if e.device_type == torch.autograd.DeviceType.CUDA:
            name = e.name.split("(")[0].replace("void ", "").strip()[:90]
            t, n = agg.get(name, (0.0, 0))
            agg[name] = (t + e.device_time_total, n + 1)
    rows = sorted(agg.items(), key=lambda kv: -kv[1][0])[:top]
    total = sum(t for t, _ in agg.values())
    print(f"kernel table: {total / 1000:.2f} ms device time in one step", file=sys.stderr)
    for name, (t, n) in rows:
        print(f"  {t / 1000:9.3f} ms  {n:5d}x  {name}", file=sys.stderr)


def main():
    # stdout carries exactly one JSON line (rank 0); anything a library prints on the
    # process's stdout (NCCL's version banner, for one) is sent to stderr instead.
    global _OUT_FD
    _OUT_FD = os.dup(1)
    os.dup2(2, 1)
    args = parse()
    full = args.workload == "full"
    if args.seq_len is None:
        args.seq_len = 4096 if full else 128
    if args.anchors is None:
        args.anchors = 32 if full else 8
    n = args.gpus
    if args.impl == "reference":
        if not os.path.isdir(os.path.join(REF_PATH, "nanospec")):
            _print_unavailable(n, "reference not installed in baseline/_ref", args)
            return
        if not full and n not in (1, 2, 4):
            _print_unavailable(n, "the reference's Shard supports 1, 2 or 4 training ranks "
                                  "(nanospec/shard.py:48-49)", args)
            return
        sys.path.insert(0, REF_PATH)
    rank, world, local, dev = setup_dist(n, timeout_s=1800 if args.impl == "reference" else 600)
    if args.impl == "ours":
        from nanospec_b200.ops._ext import cuda_ops
        cuda_ops()  # fail loudly if the extension is missing
    if world > 1 and rank == 0:
        from nanospec_b200.utils.provenance import preflight
        preflight(world)  # GPU count, all-to-all peer access, NVLink (raises otherwise)
    wl = (FullWorkload if full else DraftWorkload)(args, args.impl, world, rank, dev)
    inputs = wl.inputs

    with torch.no_grad():
        for _ in range(args.warmup):
            result = wl.step(*inputs)
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
            result = wl.step(*inputs)
        end.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        local_ms = start.elapsed_time(end) / args.steps
        clk = clocks.stop()
        ms = max_over_ranks(local_ms, world, dev)
        loss = float(wl.loss(result))

        # End-to-end through the public API: every step copies its inputs from pinned
        # host memory to the device and reads the loss back.
        e2e = None
        if not args.no_e2e:
            host = [t.cpu().pin_memory() for t in inputs]
            bi = sum(t.numel() * t.element_size() for t in host)
            losses = torch.empty(args.steps, dtype=torch.float32).pin_memory()
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            for i in range(args.steps):
                d_in = [t.to(dev, non_blocking=True) for t in host]
                r = wl.step(*d_in)
                losses[i] = wl.loss(r).float().cpu()
            e1.record()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world, dev)
            wall_ms = max_over_ranks((time.perf_counter() - t0) * 1000 / args.steps, world, dev)
            e2e = {"value": round(wl.tokens_per_step / (e2e_ms / 1000), 1), "unit": "tokens/s",
                   "h2d_bytes_per_step": bi, "d2h_bytes_per_step": 4,
                   "ms_per_step": round(e2e_ms, 3), "wall_ms_per_step": round(wall_ms, 3)}

        phase = None
        if args.impl == "ours" and full:
            phase = wl.phase_ms(dev)
        if args.impl == "ours" and args.kernel_table and rank == 0:
            _kernel_table(lambda: wl.step(*inputs))
        launches = comm_ms = exposed_ms = None
        if args.impl == "ours" and not args.no_count:
            per_step, comm, exposed = profile_step(lambda: wl.step(*inputs))
            launches = per_step * args.steps
            comm_ms = max_over_ranks(comm, world, dev)
            exposed_ms = max_over_ranks(exposed, world, dev)
    value = wl.tokens_per_step / (ms / 1000)
    if rank == 0:
        c = wl.c
        pub = PUBLISHED[args.workload].get(n)
        if full:
            tc = wl.tc
            model = (f"Qwen3.5-27B-shaped FP8 verifier ({tc['num_hidden_layers']} layers, hidden "
                     f"{tc['hidden_size']}, FFN {tc['intermediate_size']}, vocab {tc['vocab_size']}) + DSpark "
                     f"{args.config} draft ({c.num_hidden_layers} layers, hidden {c.hidden_size})")
            if args.impl == "reference":
                layout = ("4 verifier partitions + 4 trainers" if world == 8 else
                          f"verifier partitioned over all {world} GPUs, {world} trainers")
            elif args.layout == "replicated":
                layout = f"verifier replica + trainer on each of {world} GPUs"
            else:
                layout = f"{world - wl.ntrain} verifier partitions + {wl.ntrain} trainers" if world > 1 else \
                    "colocated"
        else:
            model = (f"DSpark {args.config} draft ({c.num_hidden_layers} layers, hidden {c.hidden_size}, "
                     f"vocab {c.vocab_size}) + frozen target embed/LM head; fixed teacher tensors")
            layout = f"{world} trainers"
        ntrain = wl.tokens_per_step // args.seq_len
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
            "vs_baseline": round(value / pub, 3) if pub else None,
            "dtype": "bf16",
            "data": "synthetic: random token ids; random-init weights" +
                    ("" if full else "; random teacher hidden states"),
            "config": {
                "model": model, "workload": args.workload,
                "global_batch": ntrain, "seq_len": args.seq_len, "anchors": args.anchors,
                "block_size": 7, "parallelism": f"fsdp{ntrain}" if ntrain > 1 else "single",
                "layout": layout,
                "comm": (args.comm if args.impl == "ours" else "nccl") if ntrain > 1 else None,
                "cuda_graph": wl.graphed,
                "optimizer": "AdamW fp32 masters, lr 1e-5, wd 0.01",
                "l2": "inputs larger than L2: every step streams the weights (GBs) from HBM",
            },
            "loss": loss,
            "clocks": clk,
            "e2e": e2e,
            "gpu_launches": launches,
            "phase_ms_rank0": phase,
            "comm_ms_per_step": None if comm_ms is None or comm_ms != comm_ms else round(comm_ms, 3),
            "exposed_comm_ms_per_step": None if exposed_ms is None or exposed_ms != exposed_ms else round(exposed_ms, 3),
        }
        if args.impl == "reference":
            out["impl"] = "reference"
        out["provenance"] = _provenance(world)
        _emit(out)
    wl.close(world)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _provenance(world):
    """Compact provenance for the JSON line: devices, versions, git head, one sha256
    over every product source file, and the link types between the GPUs."""
    import re

    from nanospec_b200.utils.provenance import provenance
    p = provenance(world)
    links = sorted(set(re.findall(r"\bNV\d+\b", p.pop("topology", ""))))
    p.pop("source_files", None)
    p.pop("peer_access", None)
    p["links"] = links
    return p


_OUT_FD = None


def _emit(obj):
    """Write the result line to the original stdout."""
    sys.stdout.flush()
    line = (json.dumps(obj) + "\n").encode()
    os.write(_OUT_FD if _OUT_FD is not None else 1, line)


def _print_unavailable(n, why, args):
    rank = int(os.environ.get("RANK", 0))
    if rank == 0:
        _emit({"impl": "reference", "unavailable": why, "n_gpus": n, "metric": METRIC})


if __name__ == "__main__":
    main()
