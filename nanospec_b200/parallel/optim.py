"""Sharded FP32-master AdamW with global clipping and pooled token normalisation.

Semantics (reference: nanospec/shard.py:306-356):

1. all-reduce the local weighted-token count ``den`` over the training ranks;
2. ``factor = N * accumulation_steps / den`` (0 when den == 0) - gradients were
   reduce-scattered with AVG, so this gives sum-of-gradients / global count;
3. the optimizer's gradient is ``bf16(grad * factor)`` (rounded to the grad dtype);
   its squared norm is all-reduced; a non-finite norm skips the update and zeroes
   the gradients (``updated: False``);
4. ``clip = min(1, max_norm / (norm + 1e-6))``; decoupled weight decay; Adam moments;
   bias-corrected update of the fp32 master; ``param = master`` in the compute dtype.

On CUDA, steps 3-4 are two kernels per shard (a squared-norm reduction and one
fused update that also zeroes the gradient), and the finite check happens on the
device: the update kernel reads the norm and skips itself when it is not finite.
The host reads the three scalars once, at the end.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from ..ops import reference as ref
from ..ops._ext import cuda_ops


class AdamW:
    """Hyper-parameters and step count of the sharded optimizer (state lives in the shards).

    On CUDA the step count is kept on the device (it only advances on finite updates,
    which the device decides); ``steps`` reads it back on demand. ``sync=False`` makes
    ``adamw_step`` return 0-dim device tensors instead of Python floats, so a training
    loop never waits for the GPU between steps. ``lazy_zero`` skips writing zeros into
    single-rank gradients that the next backward overwrites anyway.
    """

    def __init__(self, shards, lr=6e-4, weight_decay=0.0, betas=(0.9, 0.999), eps=1e-8,
                 max_grad_norm=1.0, sync=True, lazy_zero=False):
        self.shards = list(shards)
        self.lr, self.weight_decay, self.betas = lr, weight_decay, tuple(betas)
        self.eps, self.max_grad_norm = eps, max_grad_norm
        self.sync = sync
        # lazy_zero: on one rank, leave the consumed gradient in place instead of
        # writing zeros; the shard stays marked ``grad_zero`` and the next backward
        # binds it directly and overwrites every element (copy semantics), so the
        # stale values are never read. Saves 2 bytes/parameter of HBM writes.
        self.lazy_zero = lazy_zero
        self._steps = 0
        self._dev_step = None

    @property
    def steps(self):
        if self._dev_step is not None:
            return int(self._dev_step.item())
        return self._steps

    @steps.setter
    def steps(self, value):
        self._steps = int(value)
        if self._dev_step is not None:
            self._dev_step.fill_(int(value))


def step_factor(den, world, accumulation_steps):
    """``N * accumulation_steps / den`` (0 when den == 0): the optimizer's gradient scale."""
    return torch.where(den > 0, world * accumulation_steps / den.clamp_min(1e-6), torch.zeros_like(den))


class FusedGradNorm:
    """Squared gradient norm collected by the weight-gradient GEMMs while they write.

    One training rank only (the norm is over the final gradient, which with N > 1
    exists only after the reduce-scatter). The GEMM epilogues write per-CTA partials
    of sum bf16(grad * factor)^2 into ``part`` in launch order; ``norm2`` adds them
    in that order and runs the ordinary norm kernel over every gradient range no
    GEMM covered (norm weights, embeddings, the Markov head), so the result is
    deterministic and no second pass reads the GEMM-written gradients.
    """

    CAPACITY = 1 << 16

    def __init__(self, factor):
        self.factor = factor.reshape(1).contiguous()
        self.part = torch.empty(self.CAPACITY, device=factor.device, dtype=torch.float32)
        self.offset = 0
        self.covered = {}
        self.ok = True

    def bind(self, shard):
        return _BoundNorm(self, shard)

    def norm2(self, shards, factor):
        """Global squared norm (1-element fp32 tensor) for ``shards``; ``factor`` must
        equal the one the GEMMs used (same ``step_factor`` inputs)."""
        C = cuda_ops()
        n2 = self.part[:self.offset].sum().reshape(1) if self.offset else torch.zeros(
            1, device=factor.device, dtype=torch.float32)
        ranges = []
        for s in shards:
            start = 0
            for a, b in sorted(self.covered.get(id(s), ())):
                if a > start:
                    ranges.append(s.grad[start:a])
                start = max(start, b)
            if start < s.grad.numel():
                ranges.append(s.grad[start:])
        if ranges:
            C.grad_norm_sq_ranges(ranges, factor, n2)
        return n2


class _BoundNorm:
    def __init__(self, acc, shard):
        self.acc, self.shard = acc, shard

    def launch(self, gemm, out):
        acc, grad = self.acc, self.shard.grad
        start = (out.data_ptr() - grad.data_ptr()) // grad.element_size()
        inside = 0 <= start and start + out.numel() <= grad.numel() and out.is_contiguous()
        if not acc.ok or not inside or acc.offset + 1024 > acc.CAPACITY:
            acc.ok = False
            gemm(None, None, 0)
            return
        used = gemm(acc.factor, acc.part, acc.offset)
        acc.offset += int(used)
        acc.covered.setdefault(id(self.shard), []).append((start, start + out.numel()))


def zero_grad(optimizer):
    for s in optimizer.shards:
        s.grad.zero_()
        s.grad_zero = True


@torch.no_grad()
def adamw_step(optimizer, local_denominator, accumulation_steps=1, fused_norm=None):
    """``fused_norm``: a ``FusedGradNorm`` filled during this step's backward (one rank,
    CUDA); it replaces the separate squared-norm pass over the gradients."""
    first = optimizer.shards[0]
    den = local_denominator.detach().clone().float().reshape(())
    if first.world_size > 1:
        dist.all_reduce(den, group=first.group)
    factor = step_factor(den, first.world_size, accumulation_steps)
    b1, b2 = optimizer.betas
    if first.param.is_cuda:
        if fused_norm is not None and (first.world_size != 1 or not fused_norm.ok):
            fused_norm = None
        return _adamw_cuda(optimizer, den, factor, b1, b2, fused_norm)
    norm2 = torch.zeros_like(den)
    for s in optimizer.shards:
        norm2 += ref.scaled_grad(s.grad, factor).square().sum()
    if first.world_size > 1:
        dist.all_reduce(norm2, group=first.group)
    norm = norm2.sqrt()
    if not torch.isfinite(norm).item():
        zero_grad(optimizer)
        return {"grad_norm": float(norm), "updated": False, "denominator": float(den)}
    clip = (optimizer.max_grad_norm / (norm + 1e-6)).clamp(max=1.0)
    optimizer.steps += 1
    for s in optimizer.shards:
        ref.adamw_update(s.master, s.m, s.v, s.grad, factor, clip, optimizer.lr,
                         optimizer.weight_decay, b1, b2, optimizer.eps, optimizer.steps)
        s.param.copy_(s.master)
    zero_grad(optimizer)
    return {"grad_norm": float(norm), "updated": True, "denominator": float(den)}


def _adamw_cuda(optimizer, den, factor, b1, b2, fused_norm=None):
    C = cuda_ops()
    first = optimizer.shards[0]
    # norm2 and the update both consume factor from device memory: no host sync.
    f = factor.reshape(1).contiguous()
    if fused_norm is not None:
        norm2 = fused_norm.norm2(optimizer.shards, f)
    else:
        norm2 = torch.zeros(1, device=den.device, dtype=torch.float32)
        for s in optimizer.shards:
            C.grad_norm_sq(s.grad, f, norm2)
    if first.world_size > 1:
        dist.all_reduce(norm2, group=first.group)
    if optimizer._dev_step is None:
        optimizer._dev_step = torch.tensor([optimizer._steps], dtype=torch.int64, device=den.device)
        optimizer._bc = torch.empty(2, dtype=torch.float32, device=den.device)
    # On the device: advance the step if the norm is finite, form the bias corrections.
    C.adam_prepare(norm2, optimizer._dev_step, float(b1), float(b2), optimizer._bc)
    for s in optimizer.shards:
        lazy = optimizer.lazy_zero and s.world_size == 1
        C.adamw_update(s.param, s.master, s.m, s.v, s.grad, f, norm2, float(optimizer.lr),
                       float(optimizer.weight_decay), float(b1), float(b2), float(optimizer.eps),
                       1.0, 1.0, float(optimizer.max_grad_norm), optimizer._bc, not lazy)
        s.grad_zero = True
        hook = getattr(s, "on_updated", None)
        if hook is not None:
            hook(s)  # e.g. the peer schedule starts the next step's gather of this shard
    norm = norm2.sqrt().reshape(())
    if not optimizer.sync:
        return {"grad_norm": norm, "updated": torch.isfinite(norm), "denominator": den.reshape(())}
    vals = torch.stack((norm, den.reshape(()))).tolist()
    return {"grad_norm": vals[0], "updated": math.isfinite(vals[0]), "denominator": vals[1]}
