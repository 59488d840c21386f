"""Microbenchmarks of single hot ops on one GPU (CUDA-event timing, JSON lines).

    python -m nanospec_b200.utils.kernel_bench gemm --kind fwd --T 56 --nout 5120 --k 5120
    python -m nanospec_b200.utils.kernel_bench adamw --n 300000000
    python -m nanospec_b200.utils.kernel_bench head --T 56 --hidden 5120 --vocab 248320
    python -m nanospec_b200.utils.kernel_bench attention --S 128 --blocks 8
    python -m nanospec_b200.utils.kernel_bench fp8 --T 4096 --k 5120 --nout 17408
    python -m nanospec_b200.utils.kernel_bench gdn --S 4096 --heads 48
    python -m nanospec_b200.utils.kernel_bench gemm-suite
    python -m nanospec_b200.utils.kernel_bench verifier --S 4096

``verifier`` runs four random-init decoder layers of the Qwen3.5-27B shape (three
gated-DeltaNet layers and one full-attention layer) on one row of S tokens and
reports the device time of every verifier op, summed per op kind, plus the whole
4-layer stage.

``gemm-suite`` times every linear product of one draft layer at the benchmark
shape (forward, input and weight gradients; qwen draft: hidden 5120, FFN 15360,
8 KV heads x 128, 56 draft and 128 context tokens) against ``torch.matmul``
(cuBLAS) on the same operands. Each call sequence is captured once in a CUDA
graph and replayed, so host launch cost is excluded, and weights rotate through
three copies (> L2).

Each run does ``--warmup`` untimed calls, then times ``--reps`` calls between two
events on the launching stream. Operands rotate through enough copies to exceed
the 126 MB L2 when ``--rotate`` is set, so every call streams from HBM.
"""

from __future__ import annotations

import argparse
import json

import torch


def _time(fn, reps, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) * 1000.0 / reps  # microseconds


def _copies(make, bytes_each, rotate):
    n = max(1, (160 << 20) // max(1, bytes_each)) if rotate else 1
    return [make() for _ in range(min(n, 16))]


def bench_gemm(a):
    from nanospec_b200 import ops
    dev = "cuda"
    ws = _copies(lambda: (torch.randn(a.nout, a.k, device=dev) * 0.02).bfloat16(), a.nout * a.k * 2, a.rotate)
    x = torch.randn(a.T, a.k, device=dev).bfloat16()
    dy = torch.randn(a.T, a.nout, device=dev).bfloat16()
    y = torch.empty(a.T, a.nout, device=dev).bfloat16()
    dx = torch.empty(a.T, a.k, device=dev).bfloat16()
    dw = torch.empty(a.nout, a.k, device=dev).bfloat16()
    it = [0]

    def w():
        it[0] = (it[0] + 1) % len(ws)
        return ws[it[0]]
    fn = {"fwd": lambda: ops.linear(x, w(), out=y),
          "dgrad": lambda: ops.linear_dgrad(dy, w(), out=dx),
          "wgrad": lambda: ops.linear_wgrad(dy, x, dw)}[a.kind]
    us = _time(fn, a.reps, a.warmup)
    flops = 2.0 * a.T * a.nout * a.k
    wbytes = a.nout * a.k * 2
    return {"op": f"gemm_{a.kind}", "T": a.T, "nout": a.nout, "k": a.k, "us": round(us, 2),
            "tflops": round(flops / us / 1e6, 1), "weight_TBps": round(wbytes / us / 1e6, 3)}


def bench_adamw(a):
    from nanospec_b200.ops._ext import cuda_ops
    C = cuda_ops()
    n = a.n
    p = torch.zeros(n, device="cuda").bfloat16()
    g = torch.zeros(n, device="cuda").bfloat16()
    m32, mm, vv = (torch.zeros(n, device="cuda") for _ in range(3))
    f = torch.ones(1, device="cuda")
    n2 = torch.ones(1, device="cuda")
    zero = not a.lazy
    us = _time(lambda: C.adamw_update(p, m32, mm, vv, g, f, n2, 1e-5, 0.01, 0.9, 0.999, 1e-8, 0.1, 0.03, 1.0,
                                      None, zero), a.reps, a.warmup)
    # reads grad 2 + master/m/v 12; writes master/m/v 12 + param 2 (+ zeroed grad 2)
    per = 30.0 if zero else 28.0
    tbps = per * n / us / 1e6
    return {"op": "adamw", "n": n, "zero_grad": zero, "bytes_per_param": per, "us": round(us, 1),
            "TBps": round(tbps, 3), "of_measured_hbm": _of_peak(tbps * 1000)}


def _of_peak(gbps):
    """Fraction of the measured HBM copy bandwidth (MEASURED_PEAKS.json at the repo root)."""
    import os
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return round(gbps / float(json.load(f)["hbm_gbs"]), 3)
    except (OSError, KeyError, ValueError):
        return None


def bench_head(a):
    import nanospec_b200 as N
    from nanospec_b200.objective import head_loss
    dev = "cuda"
    o = N.Objective(num_anchors=a.T // 7)
    ids = torch.randint(0, a.vocab, (1, 4 * a.T), device=dev)
    prep = N.prepare(ids, torch.ones(1, 4 * a.T, device=dev), o)
    t = prep.weights.numel()
    h = (torch.randn(t, a.hidden, device=dev) * 0.3).bfloat16()
    th = (torch.randn(t, a.hidden, device=dev) * 0.3).bfloat16()
    W = (torch.randn(a.vocab, a.hidden, device=dev) * 0.02).bfloat16()
    e = (torch.randn(t, a.rank, device=dev) * 0.3).bfloat16()
    w2 = (torch.randn(a.vocab, a.rank, device=dev) * 0.02).bfloat16()
    dw2 = torch.empty_like(w2)
    us = _time(lambda: head_loss(h, W, e, w2, prep, o, target_hidden=th, dw2_out=dw2), a.reps, a.warmup)
    # forward: draft logits (H) + Markov logits (r) + teacher logits (H); backward:
    # dh (H), de (r), dW2 (r). Large T (chunked) also recomputes both logits blocks.
    flops = 2.0 * t * a.vocab * (3 * a.hidden + 3 * a.rank)
    reads = 2 * W.numel() * 2  # the LM head streams once per pass
    return {"op": "ce_kl_head", "tokens": t, "vocab": a.vocab, "us": round(us, 1),
            "tflops": round(flops / us / 1e6, 1), "lm_head_reads_TBps": round(reads / us / 1e6, 3),
            "of_measured_hbm": _of_peak(reads / us / 1e3)}


def bench_attention(a):
    from nanospec_b200 import ops
    dev = "cuda"
    b, S, nb, bs, hq, hk, d = 1, a.S, a.blocks, 7, 40, 8, 128
    td = nb * bs
    q = torch.randn(b, td, hq, d, device=dev).bfloat16()
    kv = torch.randn(b * (S + td), 2 * hk * d, device=dev).bfloat16()
    k, v = kv[:, :hk * d].view(-1, hk, d), kv[:, hk * d:].view(-1, hk, d)
    anchors = torch.sort(torch.randint(0, S - bs, (b, nb), device=dev)).values
    keep = torch.ones(b, nb, dtype=torch.bool, device=dev)
    out, lse = ops.attention(q, k, v, anchors, keep, S, bs)
    dout = torch.randn_like(q)
    f_us = _time(lambda: ops.attention(q, k, v, anchors, keep, S, bs), a.reps, a.warmup)
    b_us = _time(lambda: ops.attention_backward(dout, q, k, v, out, lse, anchors, keep, S, bs), a.reps, a.warmup)
    return {"op": "draft_attention", "S": S, "blocks": nb, "fwd_us": round(f_us, 1), "bwd_us": round(b_us, 1)}


def bench_fp8(a):
    from nanospec_b200.models.verifier import quantize_weight_blocks
    from nanospec_b200.ops import verifier_ops as vops
    w, s = quantize_weight_blocks(torch.randn(a.nout, a.k) * 0.02)
    w, s = w.cuda(), s.cuda()
    x = torch.randn(a.T, a.k, device="cuda").bfloat16()
    us = _time(lambda: vops.fp8_linear(x, w, s), a.reps, a.warmup)
    return {"op": "fp8_linear", "T": a.T, "nout": a.nout, "k": a.k, "us": round(us, 1),
            "tflops": round(2.0 * a.T * a.nout * a.k / us / 1e6, 1)}


def bench_gdn(a):
    from nanospec_b200.ops import verifier_ops as vops
    b, s, nk, nv, d = 1, a.S, a.heads // 3, a.heads, 128
    q = torch.randn(b, s, nk, d, device="cuda").bfloat16()
    k = torch.randn(b, s, nk, d, device="cuda").bfloat16()
    v = torch.randn(b, s, nv, d, device="cuda").bfloat16()
    g = -torch.rand(b, s, nv, device="cuda") * 0.1
    beta = torch.rand(b, s, nv, device="cuda").bfloat16()
    us = _time(lambda: vops.gated_delta_rule(q, k, v, g, beta, nv // nk), a.reps, a.warmup)
    dout = torch.randn(b, s, nv, d, device="cuda").bfloat16()
    bus = _time(lambda: vops.gated_delta_rule_backward(q, k, v, g, beta, dout, nv // nk), a.reps, a.warmup)
    # chunked form, chunk 64: per head about 4*S*64*d (intra-chunk) + 4*S*d*d (state) MACs forward
    flops = 2.0 * nv * (4 * s * 64 * d + 4 * s * d * d)
    kern = _kernel_times(lambda: vops.gated_delta_rule(q, k, v, g, beta, nv // nk))
    bkern = _kernel_times(lambda: vops.gated_delta_rule_backward(q, k, v, g, beta, dout, nv // nk))
    return {"op": "gdn_chunk", "S": s, "heads": nv, "fwd_us": round(us, 1), "bwd_us": round(bus, 1),
            "fwd_tflops": round(flops / us / 1e6, 2), "fwd_kernels_us": kern, "bwd_kernels_us": bkern}


def bench_conv(a):
    """Causal depthwise conv + SiLU over the q/k/v channels of the fused GDN
    projection output (strided token rows), the verifier's shape by default."""
    from nanospec_b200.ops import verifier_ops as vops
    ld, ch = a.k, a.nout  # row stride of the projection output, conv channels
    x = torch.randn(1, a.S, ld, device="cuda").bfloat16()
    w = (torch.randn(ch, 4, device="cuda") * 0.3).bfloat16()
    us = _time(lambda: vops.causal_conv_silu_rows(x, ld, w, ch), a.reps, a.warmup)
    moved = a.S * ch * 2 * 2  # read and write the conv channels once
    return {"op": "conv_silu", "S": a.S, "channels": ch, "us": round(us, 1),
            "GBps": round(moved / us / 1e3, 1), "of_measured_hbm": _of_peak(moved / us / 1e3)}


def bench_verifier(a):
    from nanospec_b200.models.verifier import (QwenStage, qwen3_5_27b_text_config, random_verifier_weights,
                                               stage_forward, synthetic_hf_config)
    from nanospec_b200.ops import verifier_ops as vops
    tc = qwen3_5_27b_text_config()
    tc["num_hidden_layers"] = 4
    tc["layer_types"] = tc["layer_types"][:4]
    w = random_verifier_weights(tc, 0, 4, device="cuda", first=True, last=True, seed=0)
    st = QwenStage(None, 0, 4, device="cuda", first=True, last=True, weights=w,
                   config=synthetic_hf_config(tc))
    ids = torch.randint(0, tc["vocab_size"], (1, a.S), device="cuda")
    names = ("embedding", "add", "silu_mul", "qwen_norm", "qwen_gated_norm", "fp8_linear", "causal_conv_silu",
             "gdn_gates", "gated_delta_rule", "causal_attention_gated", "gated_attention", "fp8_gemm", "quantize",
             "add_norm", "silu_mul_quantize", "gated_norm_quantize", "causal_conv_silu_rows")
    times, orig = {}, {n: getattr(vops, n) for n in names}

    def wrap(name, fn):
        def run(*args, **kw):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            out = fn(*args, **kw)
            e1.record()
            times.setdefault(name, []).append((e0, e1))
            return out
        return run
    for _ in range(a.warmup):
        stage_forward(st, ids)
    torch.cuda.synchronize()
    whole = _time(lambda: stage_forward(st, ids), a.reps, 0) / 1000.0
    for n in names:
        setattr(vops, n, wrap(n, orig[n]))
    try:
        for _ in range(a.reps):
            stage_forward(st, ids)
        torch.cuda.synchronize()
    finally:
        for n in names:
            setattr(vops, n, orig[n])
    per = {n: round(sum(e0.elapsed_time(e1) for e0, e1 in v) / a.reps, 3) for n, v in times.items()}
    gemm_ms = per.get("fp8_gemm", 0.0) + per.get("fp8_linear", 0.0)
    kern = _kernel_times(lambda: stage_forward(st, ids), reps=2)
    return {"op": "verifier_4_layers", "S": a.S, "stage_ms": round(whole, 3), "op_ms": per, "kernel_us": kern,
            "fp8_tflops": round(_verifier_fp8_flops(tc, a.S) / (gemm_ms * 1e9), 1) if gemm_ms else None}


def _verifier_fp8_flops(tc, s):
    from nanospec_b200.models.verifier import layer_tensor_shapes
    total = 0.0
    for i in range(tc["num_hidden_layers"]):
        for (shape, quant) in layer_tensor_shapes(tc, i).values():
            if quant and len(shape) == 2:
                total += 2.0 * s * shape[0] * shape[1]
    return total


def _kernel_times(fn, reps=3):
    """Mean device microseconds per call of every kernel ``fn`` launches (torch.profiler)."""
    from torch.profiler import ProfilerActivity, profile
    fn()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(reps):
            fn()
        torch.cuda.synchronize()
    out = {}
    for e in prof.events():
        if e.device_type == torch.autograd.DeviceType.CUDA:
            name = e.name.split("(")[0].split("<")[0].replace("void ", "").strip()
            out[name] = out.get(name, 0.0) + e.device_time_total / reps
    return {k: round(v, 1) for k, v in sorted(out.items(), key=lambda kv: -kv[1])}


def _graph_time(fns, reps):
    """Per-call time of `fns` (one call each) captured in one CUDA graph and replayed."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for f in fns:
            f()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for f in fns:
            f()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1000.0 / (reps * len(fns))


def bench_gemm_suite(a):
    from nanospec_b200 import ops
    dev, R = "cuda", 3
    rows = []

    def case(kind, T, nout, k, residual=False):
        if kind == "wgrad":
            dy = torch.randn(T, nout, device=dev).bfloat16()
            x = torch.randn(T, k, device=dev).bfloat16()
            outs = [torch.empty(nout, k, device=dev, dtype=torch.bfloat16) for _ in range(R)]
            ours = [lambda o=o: ops.linear_wgrad(dy, x, o) for o in outs]
            ref = [lambda o=o: torch.matmul(dy.t(), x, out=o) for o in outs]
        else:
            ws = [torch.randn(nout, k, device=dev).bfloat16() for _ in range(R)]
            if kind == "fwd":
                x = torch.randn(T, k, device=dev).bfloat16()
                r = torch.randn(T, nout, device=dev).bfloat16() if residual else None
                outs = [torch.empty(T, nout, device=dev, dtype=torch.bfloat16) for _ in range(R)]
                ours = [lambda w=w, o=o: ops.linear(x, w, out=o, residual=r) for w, o in zip(ws, outs)]
                ref = [lambda w=w, o=o: torch.matmul(x, w.t(), out=o) for w, o in zip(ws, outs)]
            else:
                dy = torch.randn(T, nout, device=dev).bfloat16()
                outs = [torch.empty(T, k, device=dev, dtype=torch.bfloat16) for _ in range(R)]
                ours = [lambda w=w, o=o: ops.linear_dgrad(dy, w, out=o) for w, o in zip(ws, outs)]
                ref = [lambda w=w, o=o: torch.matmul(dy, w, out=o) for w, o in zip(ws, outs)]
        o_us, c_us = _graph_time(ours, a.reps), _graph_time(ref, a.reps)
        wb = 2.0 * nout * k
        rows.append({"kind": kind, "T": T, "nout": nout, "k": k, "residual": residual, "ours_us": round(o_us, 1),
                     "cublas_us": round(c_us, 1), "ours_TBps": round(wb / o_us / 1e6, 2),
                     "cublas_TBps": round(wb / c_us / 1e6, 2)})

    for kind, T, nout, k, res in [("fwd", 56, 5120, 5120, False), ("fwd", 184, 2048, 5120, False),
                                  ("fwd", 56, 5120, 5120, True), ("fwd", 56, 30720, 5120, False),
                                  ("fwd", 56, 5120, 15360, True), ("dgrad", 56, 5120, 5120, False),
                                  ("dgrad", 184, 2048, 5120, False), ("dgrad", 56, 30720, 5120, False),
                                  ("dgrad", 56, 5120, 15360, False), ("wgrad", 56, 30720, 5120, False),
                                  ("wgrad", 56, 5120, 15360, False), ("wgrad", 56, 5120, 5120, False),
                                  ("wgrad", 184, 2048, 5120, False), ("wgrad", 128, 5120, 25600, False)]:
        case(kind, T, nout, k, res)
    return {"op": "gemm_suite", "cases": rows, "total_ours_us": round(sum(r["ours_us"] for r in rows), 1),
            "total_cublas_us": round(sum(r["cublas_us"] for r in rows), 1)}


def bench_fused(a):
    """The fused collective GEMMs on ONE GPU: a window of world 1, so every "peer"
    access is local. Measures the kernels' own efficiency (no NVLink) against the
    plain GEMMs of the same shape: x [T, k] · W [nout, k]^T and dy^T · x."""
    from nanospec_b200 import ops
    from nanospec_b200.ops._ext import cuda_ops
    C = cuda_ops()
    dev = torch.device("cuda")
    T, N, K = a.T, a.nout, a.k
    ss = -(-N * K // 8) * 8
    wid, _ = C.window_create(4096 + 2 * ss * 2 + 4096, 0, 1)
    C.window_open(wid, C.window_ipc_handle(wid).view(1, -1))
    param_off, slot_off = 4096, 4096 + ((ss * 2 + 4095) // 4096) * 4096
    g = torch.Generator(device=dev).manual_seed(0)
    C.window_view(wid, param_off, ss, torch.bfloat16).copy_((torch.randn(ss, device=dev, generator=g) * 0.02).bfloat16())
    x = torch.randn(T, K, device=dev, generator=g).bfloat16()
    dy = torch.randn(T, N, device=dev, generator=g).bfloat16()
    resident = torch.empty(ss, device=dev, dtype=torch.bfloat16)
    out = torch.empty(T, N, device=dev, dtype=torch.bfloat16)
    flags = torch.zeros(-(-ss // min(16384, ss)), device=dev, dtype=torch.int32)
    claim = torch.zeros(1, device=dev, dtype=torch.int32)
    ep = [0]

    def ag():
        ep[0] += 1
        C.ag_gemm(wid, param_off, ss, resident, 0, N, K, x, out, flags, claim, ep[0], 200_000_000)

    w = resident[:N * K].view(N, K)
    dw = torch.empty(N, K, device=dev, dtype=torch.bfloat16)
    flops = 2.0 * T * N * K
    res = {"op": "fused", "T": T, "nout": N, "k": K}
    for name, fn in (("ag_gemm", ag), ("linear", lambda: ops.linear(x, w)),
                     ("gemm_rs", lambda: C.gemm_rs(wid, slot_off, ss, 0, dy, x)),
                     ("linear_wgrad", lambda: ops.linear_wgrad(dy, x, dw)),
                     ("torch_wgrad", lambda: torch.matmul(dy.t(), x))):
        us = _time(fn, a.reps, a.warmup)
        res[name + "_us"] = round(us, 1)
        res[name + "_tflops"] = round(flops / us / 1e6, 1)
    torch.cuda.synchronize()
    assert C.device_error() == 0
    C.window_close(wid)
    return res


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("op", choices=("gemm", "adamw", "head", "attention", "fp8", "gdn", "gemm-suite",
                                     "verifier", "fused", "conv"))
    p.add_argument("--kind", choices=("fwd", "dgrad", "wgrad"), default="fwd")
    p.add_argument("--T", type=int, default=56)
    p.add_argument("--nout", type=int, default=5120)
    p.add_argument("--k", type=int, default=5120)
    p.add_argument("--n", type=int, default=300_000_000)
    p.add_argument("--hidden", type=int, default=5120)
    p.add_argument("--vocab", type=int, default=248320)
    p.add_argument("--rank", type=int, default=256)
    p.add_argument("--S", type=int, default=128)
    p.add_argument("--blocks", type=int, default=8)
    p.add_argument("--heads", type=int, default=48)
    p.add_argument("--reps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--rotate", action="store_true", help="rotate operands through > L2 bytes")
    p.add_argument("--lazy", action="store_true", help="adamw: leave the gradient in place (lazy_zero)")
    a = p.parse_args(argv)
    fn = {"gemm": bench_gemm, "adamw": bench_adamw, "head": bench_head, "attention": bench_attention,
          "fp8": bench_fp8, "gdn": bench_gdn, "gemm-suite": bench_gemm_suite,
          "verifier": bench_verifier, "fused": bench_fused, "conv": bench_conv}[a.op]
    print(json.dumps(fn(a)), flush=True)


if __name__ == "__main__":
    main()
