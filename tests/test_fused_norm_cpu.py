"""Bookkeeping of the fused gradient norm (parallel.optim.FusedGradNorm) on CPU.

The GEMM side is emulated: each "launch" writes the squared norm of the gradient
range it produced into one partial slot. Whatever ranges are covered, the total
(partials + the norm pass over every uncovered range) must equal the norm of the
whole gradient, and each element must be counted exactly once.
"""

from types import SimpleNamespace

import torch
from hypothesis import given, settings
from hypothesis import strategies as st

import nanospec_b200.parallel.optim as optim


def _sq(g, f):
    return (g.float() * f).to(g.dtype).float().square().sum()


class _FakeOps:
    def grad_norm_sq_ranges(self, ranges, factor, n2):
        for r in ranges:
            n2 += _sq(r, factor.item())


@settings(max_examples=60, deadline=None)
@given(sizes=st.lists(st.integers(1, 300), min_size=1, max_size=4), data=st.data())
def test_partials_plus_uncovered_ranges_equal_full_norm(sizes, data):
    f = torch.tensor([0.7])
    shards = [SimpleNamespace(grad=torch.randn(n).bfloat16()) for n in sizes]
    acc = optim.FusedGradNorm.__new__(optim.FusedGradNorm)  # CPU: skip the device buffer
    acc.factor, acc.part, acc.offset, acc.covered, acc.ok = f, torch.zeros(1 << 12), 0, {}, True
    for s in shards:
        n = s.grad.numel()
        # random disjoint covered ranges inside this shard
        cuts = sorted(set(data.draw(st.lists(st.integers(0, n), max_size=6))))
        for a, b in zip(cuts[0::2], cuts[1::2]):
            if b <= a:
                continue
            view = s.grad[a:b]

            def gemm(fac, part, off, view=view):
                part[off] = _sq(view, fac.item())
                return 1

            optim._BoundNorm(acc, s).launch(gemm, view)
    old = optim.cuda_ops
    optim.cuda_ops = lambda: _FakeOps()
    try:
        got = acc.norm2(shards, f).item()
    finally:
        optim.cuda_ops = old
    want = sum(_sq(s.grad, 0.7).item() for s in shards)
    assert abs(got - want) <= 1e-5 * max(1.0, want)
