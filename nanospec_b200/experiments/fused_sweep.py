"""Fused compute + collective sweep (2+ GPUs, one process per GPU).

    torchrun --nproc-per-node N -m nanospec_b200.experiments.fused_sweep \
        [--M 4096 --K 5120 --N 5120 17408 --reps 10 --warmup 3] [--output sweep.json]

For every weight shape W [N, K] (bf16, sharded over the ranks as an FSDP unit) and
M tokens, times on the device (CUDA events on the launching stream, max over
ranks, L2 flushed by a 256 MB write between repetitions):

* all-gather -> GEMM. NCCL path: ``all_gather_into_tensor`` of the shards, then
  ``torch.matmul(x, W.T)``; the reference does this in ``nanospec/shard.py:104-116``
  and its linear op. Fused path: ``ag_gemm``, which gathers the unit into the
  resident buffer and multiplies as W's chunks arrive.
* weight-gradient GEMM -> reduce-scatter. NCCL path: ``torch.matmul(dy.T, x)``,
  then ``reduce_scatter_tensor(AVG)`` (``nanospec/shard.py:140-150``). Fused path:
  ``gemm_rs`` (the epilogue stores into the owners' window slots), the flag
  exchange, then ``peer_reduce_local``.

Each fused path is reported against its roofline: the slower of FLOPs at the
measured bf16 GEMM peak and the bytes that must cross NVLink at the measured
770 GB/s per direction per GPU. The peaks come from ``MEASURED_PEAKS.json`` at
the repository root when present.
"""

from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

from nanospec_b200.ops._ext import cuda_ops

NVLINK_GBS = 770.0


def _peaks():
    p = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d.get("bf16_tflops", 1590.0)), "measured"
    return 1590.0, "fallback"


def _time(fn, reps, warmup, flush):
    for _ in range(warmup):
        fn()
    times = []
    for _ in range(reps):
        flush.zero_()
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b) * 1e3)
    t = torch.tensor(sorted(times)[len(times) // 2], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def _open_window(C, rank, world, nbytes):
    wid, _ = C.window_create(nbytes, rank, world)
    handles = [None] * world
    dist.all_gather_object(handles, C.window_ipc_handle(wid).tolist())
    C.window_open(wid, torch.tensor(handles, dtype=torch.uint8))
    return wid


def sweep(M, K, Ns, reps, warmup):
    C = cuda_ops()
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", torch.cuda.current_device())
    peak_tflops, peak_src = _peaks()
    flush = torch.empty(256 << 20, device=dev, dtype=torch.uint8)
    rows = []
    for N in Ns:
        numel = N * K
        ss = -(-numel // (8 * world)) * 8
        full = ss * world
        g = torch.Generator(device=dev).manual_seed(1 + rank)
        shard = (torch.randn(ss, device=dev, generator=g) * 0.02).bfloat16()
        x = torch.randn(M, K, device=dev, generator=g).bfloat16()
        dy = torch.randn(M, N, device=dev, generator=g).bfloat16()
        flops = 2.0 * M * N * K
        remote = (world - 1) * ss * 2  # bytes each rank receives (AG) or sends (RS)
        roof_us = max(flops / (peak_tflops * 1e12), remote / (NVLINK_GBS * 1e9)) * 1e6

        # ---------------------------------------------------------------- all-gather -> GEMM
        gathered = torch.empty(full, device=dev, dtype=torch.bfloat16)

        def nccl_ag():
            dist.all_gather_into_tensor(gathered, shard)
            return torch.matmul(x, gathered[:numel].view(N, K).t())

        slot_off = 4096 + ((ss * 2 + 4095) // 4096) * 4096
        wid = _open_window(C, rank, world, slot_off + full * 2)
        C.window_view(wid, 4096, ss, torch.bfloat16).copy_(shard)
        resident = torch.empty(full, device=dev, dtype=torch.bfloat16)
        out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        flags = torch.zeros(-(-full // min(16384, ss)), device=dev, dtype=torch.int32)
        claim = torch.zeros(1, device=dev, dtype=torch.int32)
        epoch = [0]
        torch.cuda.synchronize()
        dist.barrier()

        def fused_ag():
            epoch[0] += 1
            C.ag_gemm(wid, 4096, ss, resident, 0, N, K, x, out, flags, claim, epoch[0], 200_000_000)

        t_nccl_ag = _time(nccl_ag, reps, warmup, flush)
        t_fused_ag = _time(fused_ag, reps, warmup, flush)
        ref = nccl_ag()
        fused_ag()
        torch.cuda.synchronize()
        ag_err = ((out.float() - ref.float()).norm() / ref.float().norm()).item()
        w_local = gathered[:numel].view(N, K)
        t_gemm = _time(lambda: torch.matmul(x, w_local.t()), reps, warmup, flush)

        # ---------------------------------------------------------------- GEMM -> reduce-scatter
        red = torch.empty(ss, device=dev, dtype=torch.bfloat16)
        dw_full = torch.zeros(full, device=dev, dtype=torch.bfloat16)

        def nccl_rs():
            dw_full[:numel].view(N, K).copy_(torch.matmul(dy.t(), x))
            dist.reduce_scatter_tensor(red, dw_full, op=dist.ReduceOp.AVG)

        grad = torch.zeros(ss, device=dev, dtype=torch.bfloat16)
        seq = [0]

        def fused_rs():
            seq[0] += 1
            C.gemm_rs(wid, slot_off, ss, 0, dy, x)
            if full > numel:
                C.peer_push(wid, slot_off, ss, dw_full, numel, full)
            C.peer_signal(wid, 0, 4, seq[0])
            C.peer_wait(wid, 0, 4, seq[0], 200_000_000)
            grad.zero_()
            C.peer_reduce_local(wid, slot_off, ss, grad)
            C.peer_signal(wid, 0, 5, seq[0])  # slot consumed: peers may push again
            C.peer_wait(wid, 0, 5, seq[0], 200_000_000)

        t_nccl_rs = _time(nccl_rs, reps, warmup, flush)
        t_fused_rs = _time(fused_rs, reps, warmup, flush)
        nccl_rs()
        fused_rs()
        torch.cuda.synchronize()
        rs_err = ((grad.float() - red.float()).norm() / red.float().norm().clamp_min(1e-30)).item()
        assert C.device_error() == 0, "a bounded wait timed out"
        dist.barrier()
        C.window_close(wid)
        rows.append({
            "M": M, "K": K, "N": N, "world": world,
            "roofline_us": round(roof_us, 1),
            "gemm_alone_us": round(t_gemm, 1),
            "allgather_gemm": {"nccl_torch_us": round(t_nccl_ag, 1), "fused_us": round(t_fused_ag, 1),
                               "fused_frac_of_roofline": round(roof_us / t_fused_ag, 3),
                               "speedup": round(t_nccl_ag / t_fused_ag, 3), "rel_err": ag_err},
            "gemm_reduce_scatter": {"nccl_torch_us": round(t_nccl_rs, 1), "fused_us": round(t_fused_rs, 1),
                                    "fused_frac_of_roofline": round(roof_us / t_fused_rs, 3),
                                    "speedup": round(t_nccl_rs / t_fused_rs, 3), "rel_err": rs_err},
        })
    return {"peak_bf16_tflops": peak_tflops, "peak_source": peak_src, "nvlink_gbs": NVLINK_GBS, "rows": rows}


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--M", type=int, default=4096)
    p.add_argument("--K", type=int, default=5120)
    p.add_argument("--N", type=int, nargs="+", default=[5120, 17408])
    p.add_argument("--reps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--output")
    a = p.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    try:
        res = sweep(a.M, a.K, a.N, a.reps, a.warmup)
        if dist.get_rank() == 0:
            line = json.dumps(res)
            print(line, flush=True)
            if a.output:
                Path(a.output).write_text(line + "\n")
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
