"""Numerical comparison against the reference implementation (single process).

    python -m nanospec_b200.experiments.compare --config qwen-parity --dtype bfloat16 \
        --steps 3 --device cuda --output compare.json

The oracle is the unmodified reference package (installed under baseline/_ref): its
own ``train()`` with the same initial weights (same seed and init stream), the same
fixed synthetic teacher tensors, the same anchors (identical RNG state) and an
unequal supervision mask. Per step it compares the loss, the raw gradients (cosine,
relative L2), the updated parameters and the grad norm, with the reference's own
tolerance table (experiments/compare.py:325-337 of the reference project).
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

import nanospec_b200 as N

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF = os.path.join(ROOT, "baseline", "_ref")


def tolerances(fp32: bool):
    return {
        "loss_relative": 2e-5 if fp32 else 0.02,
        "gradient_cosine": 0.99999 if fp32 else 0.995,
        "gradient_relative_l2": 2e-4 if fp32 else 0.06,
        "draft_hidden_cosine": 0.99999 if fp32 else 0.99,
        "parameter_relative_l2": 1e-5 if fp32 else 0.003,
    }


def similarity(a, b):
    a, b = a.float().flatten(), b.float().flatten()
    return {"cosine": torch.nn.functional.cosine_similarity(a, b, dim=0).item(),
            "relative_l2": ((a - b).norm() / b.norm().clamp_min(1e-12)).item(),
            "max_abs": (a - b).abs().max().item()}


def arguments(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--config", default="tiny")
    p.add_argument("--dtype", choices=("float32", "bfloat16"), default="bfloat16")
    p.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--seq-len", type=int, default=32)
    p.add_argument("--anchors", type=int, default=2)
    p.add_argument("--learning-rate", type=float, default=3e-4)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--output", default="outputs/compare.json")
    return p.parse_args(argv)


@torch.no_grad()
def compare(args):
    if REF not in sys.path:
        sys.path.append(REF)
    import nanospec.config as RC
    import nanospec.distributed as RDist
    import nanospec.dspark as RD
    import nanospec.shard as RS
    import nanospec.train as RT
    torch.set_float32_matmul_precision("highest")
    dtype = getattr(torch, args.dtype)
    dev = torch.device(args.device)
    c = N.DraftConfig.load(N.config_path(args.config))
    rc = RC.DraftConfig(**c.to_dict())
    o = N.Objective(num_anchors=args.anchors)
    ro = RC.Objective(num_anchors=args.anchors)
    g = torch.Generator().manual_seed(args.seed + 1)
    emb = torch.randn(c.vocab_size, c.hidden_size, generator=g, dtype=dtype) * 0.1
    head = torch.randn(c.vocab_size, c.hidden_size, generator=g, dtype=dtype) * 0.1
    ours = N.DSpark(c, N.initialize(c, args.seed, dtype), emb, head, device=dev, dtype=dtype)
    theirs = RD.DSpark(rc, RD.initialize(rc, args.seed, dtype), emb, head, device=dev, dtype=dtype)
    del emb, head
    opt = N.AdamW(ours.sharding, lr=args.learning_rate, weight_decay=0.01)
    ropt = RS.AdamW(theirs.sharding, lr=args.learning_rate, weight_decay=0.01)
    gen = torch.Generator(device=dev).manual_seed(args.seed + 100)
    s = args.seq_len
    ids = torch.randint(0, c.vocab_size, (1, s), device=dev, generator=gen)
    hs = [torch.randn(1, s, c.hidden_size, device=dev, generator=gen).to(dtype) for _ in c.target_layer_ids]
    last = torch.randn(1, s, c.hidden_size, device=dev, generator=gen).to(dtype)
    mask = torch.ones(1, s, device=dev)
    mask[:, s // 2: s // 2 + 2] = 0
    tol = tolerances(dtype == torch.float32)
    rows = []
    for step in range(args.steps):
        torch.manual_seed(args.seed + step)
        r = N.train(ids, ours, o, teacher_batch=N.TeacherBatch(hs, last), loss_mask=mask)
        grads = [u.grad.clone() for u in ours.sharding]
        torch.manual_seed(args.seed + step)
        rr = RT.train(ids, theirs, ro, teacher_batch=RDist.TeacherBatch(hs, last), loss_mask=mask)
        rgrads = [u.grad.clone() for u in theirs.sharding]
        u = N.adamw_step(opt, r.metrics.denominator)
        ru = RS.adamw_step(ropt, rr.metrics.denominator)
        gsim = similarity(torch.cat([x.flatten() for x in grads]), torch.cat([x.flatten() for x in rgrads]))
        psim = similarity(torch.cat([x.master.flatten() for x in ours.sharding]),
                          torch.cat([x.master.flatten() for x in theirs.sharding]))
        hsim = similarity(r.hidden, rr.hidden)
        rows.append({"step": step + 1, "loss": r.metrics.loss.item(), "reference_loss": rr.metrics.loss.item(),
                     "accept_len": r.metrics.accept_len.item(), "reference_accept_len": rr.metrics.accept_len.item(),
                     "grad_norm": u["grad_norm"], "reference_grad_norm": ru["grad_norm"],
                     "gradients": gsim, "parameters": psim, "draft_hidden": hsim})
        print(json.dumps({k: v for k, v in rows[-1].items() if k in ("step", "loss", "reference_loss")} |
                         {"grad_cos": gsim["cosine"], "param_rel_l2": psim["relative_l2"]}), flush=True)
    passed = all(
        abs(r["loss"] - r["reference_loss"]) / max(abs(r["reference_loss"]), 1e-8) < tol["loss_relative"]
        and r["gradients"]["cosine"] > tol["gradient_cosine"]
        and r["gradients"]["relative_l2"] < tol["gradient_relative_l2"]
        and r["draft_hidden"]["cosine"] > tol["draft_hidden_cosine"]
        and r["parameters"]["relative_l2"] < tol["parameter_relative_l2"]
        for r in rows)
    report = {"passed": passed, "tolerances": tol, "config": c.to_dict(), "dtype": args.dtype,
              "device": str(dev), "seq_len": s, "anchors": args.anchors, "rows": rows,
              "oracle": "reference train() from baseline/_ref on the same device"}
    os.makedirs(os.path.dirname(args.output) or ".", exist_ok=True)
    with open(args.output, "w") as f:
        json.dump(report, f, indent=2)
    print(json.dumps({"passed": passed}), flush=True)
    return report


def main(argv=None):
    return compare(arguments(argv))


if __name__ == "__main__":
    main()
