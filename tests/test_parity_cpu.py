"""Step-level parity with the reference's own ``train()`` on CPU (same seeds, anchors, masks)."""

import pytest
import torch

import nanospec_b200 as N


def _build(ref, name, dtype, seq=128, anchors=8):
    c = N.DraftConfig.load(N.config_path(name))
    rc = ref.config.DraftConfig(**c.to_dict())
    g = torch.Generator().manual_seed(43)
    emb = (torch.randn(c.vocab_size, c.hidden_size, generator=g) * 0.1).to(dtype)
    head = (torch.randn(c.vocab_size, c.hidden_size, generator=g) * 0.1).to(dtype)
    ids = torch.randint(0, c.vocab_size, (1, seq), generator=g)
    hs = [torch.randn(1, seq, c.hidden_size, generator=g).to(dtype) for _ in range(c.num_target_layers)]
    last = torch.randn(1, seq, c.hidden_size, generator=g).to(dtype)
    mask = torch.ones(1, seq)
    mask[:, seq // 2: seq // 2 + 2] = 0
    ours = N.DSpark(c, N.initialize(c, 42, dtype), emb, head, device="cpu", dtype=dtype)
    theirs = ref.dspark.DSpark(rc, ref.dspark.initialize(rc, 42, dtype), emb, head, device="cpu", dtype=dtype)
    return c, ours, theirs, ids, hs, last, mask


def test_initialize_matches_reference(reference):
    c = N.DraftConfig.load(N.config_path("tiny"))
    a = N.initialize(c, 7, torch.float32)
    b = reference.dspark.initialize(reference.config.DraftConfig(**c.to_dict()), 7, torch.float32)
    assert list(a) == list(b)
    assert all(torch.equal(a[k], b[k]) for k in a)


def test_prepare_matches_reference(reference):
    o = N.Objective(num_anchors=8, block_size=4)
    ro = reference.config.Objective(num_anchors=8, block_size=4)
    ids = torch.randint(0, 100, (2, 40))
    mask = torch.ones(2, 40)
    mask[1, 10:14] = 0
    torch.manual_seed(3)
    p = N.prepare(ids, mask, o)
    torch.manual_seed(3)
    q = reference.dspark.prepare(ids, mask, ro)
    for f in ("anchors", "keep", "positions", "target_ids", "previous", "weights", "valid",
              "teacher_indices", "mask"):
        assert torch.equal(getattr(p, f), getattr(q, f)), f


@pytest.mark.parametrize("name,dtype,tol", [("tiny", torch.float32, 2e-5),
                                            ("tiny-hybrid", torch.float32, 2e-5),
                                            ("tiny", torch.bfloat16, 0.02)])
def test_train_step_parity(reference, name, dtype, tol):
    c, ours, theirs, ids, hs, last, mask = _build(reference, name, dtype)
    o, ro = N.Objective(num_anchors=8), reference.config.Objective(num_anchors=8)
    opt = N.AdamW(ours.sharding, lr=1e-3, weight_decay=0.01)
    ropt = reference.shard.AdamW(theirs.sharding, lr=1e-3, weight_decay=0.01)
    for step in range(3):
        torch.manual_seed(step)
        r = N.train(ids, ours, o, teacher_batch=N.TeacherBatch(hs, last), loss_mask=mask)
        torch.manual_seed(step)
        rr = reference.train.train(ids, theirs, ro, teacher_batch=reference.distributed.TeacherBatch(hs, last),
                                   loss_mask=mask)
        rel = abs(r.metrics.loss.item() - rr.metrics.loss.item()) / abs(rr.metrics.loss.item())
        assert rel < tol
        assert abs(r.metrics.accept_len.item() - rr.metrics.accept_len.item()) < 50 * tol
        for a, b in zip(ours.sharding, theirs.sharding):
            cos = torch.nn.functional.cosine_similarity(a.grad.float(), b.grad.float(), dim=0).item()
            assert cos > (0.99999 if dtype == torch.float32 else 0.995)
        u = N.adamw_step(opt, r.metrics.denominator)
        ru = reference.shard.adamw_step(ropt, rr.metrics.denominator)
        assert u["updated"] and ru["updated"]
        assert abs(u["grad_norm"] - ru["grad_norm"]) / ru["grad_norm"] < tol
        for a, b in zip(ours.sharding, theirs.sharding):
            prel = ((a.master - b.master).norm() / b.master.norm()).item()
            assert prel < (1e-5 if dtype == torch.float32 else 3e-3)


def test_teacher_logits_path_matches(reference):
    c, ours, theirs, ids, hs, last, mask = _build(reference, "tiny", torch.float32)
    logits = torch.randn(1, ids.shape[1], c.vocab_size)
    o, ro = N.Objective(num_anchors=8), reference.config.Objective(num_anchors=8)
    torch.manual_seed(0)
    r = N.train(ids, ours, o, teacher_batch=N.TeacherBatch(hs, last, logits), loss_mask=mask)
    torch.manual_seed(0)
    rr = reference.train.train(ids, theirs, ro, teacher_batch=reference.distributed.TeacherBatch(hs, last, logits),
                               loss_mask=mask)
    assert abs(r.metrics.loss.item() - rr.metrics.loss.item()) < 1e-5
    assert torch.allclose(r.hidden, rr.hidden, atol=1e-5)


def test_gdn_backward_oracle_matches_finite_differences():
    from nanospec_b200.ops import reference as R
    torch.manual_seed(0)
    b, s, h, d = 1, 9, 1, 4
    args = [torch.randn(b, s, h, d, dtype=torch.float64) for _ in range(3)]
    args += [-torch.rand(b, s, h, dtype=torch.float64), torch.rand(b, s, h, dtype=torch.float64)]
    w = torch.randn(b, s, h, d, dtype=torch.float64)
    grads = R.gated_delta_rule_backward(*args, w)
    eps = 1e-3
    for which in range(5):
        x = args[which]
        idx = (0, 3) + ((0, 1) if x.dim() == 4 else (0,))
        plus = [a.clone() for a in args]
        minus = [a.clone() for a in args]
        plus[which][idx] += eps
        minus[which][idx] -= eps
        f = lambda a: (R.gated_delta_rule_recurrent(*[t.float() for t in a]).double() * w).sum()  # noqa: E731
        fd = (f(plus) - f(minus)) / (2 * eps)
        assert abs(fd.item() - grads[which][idx].item()) < 2e-2 * max(1.0, abs(fd.item()))


def test_chunked_gdn_backward_statements_match_autograd():
    """The explicit chunked backward (the statements the CUDA kernels implement)
    equals autograd through the token recurrence, with and without a partial chunk."""
    from nanospec_b200.ops import reference as R
    torch.manual_seed(0)
    for b, s, h, d, chunk in [(1, 70, 2, 16, 16), (2, 130, 3, 32, 64), (1, 64, 1, 16, 64)]:
        q, k, v = (torch.randn(b, s, h, d) for _ in range(3))
        g, beta = -torch.rand(b, s, h) * 0.5, torch.rand(b, s, h)
        dout = torch.randn(b, s, h, d)
        want = R.gated_delta_rule_backward(q, k, v, g, beta, dout)
        got = R.gated_delta_rule_backward_chunked(q, k, v, g, beta, dout, chunk=chunk)
        for x, y in zip(got, want):
            assert ((x - y).norm() / y.norm()).item() < 1e-5
