"""End-to-end train() on the GPU (CUDA kernels) vs the CPU path of the same model."""

import pytest
import torch

import nanospec_b200 as N

pytestmark = pytest.mark.gpu
cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")


def _model(c, dev, dtype):
    g = torch.Generator().manual_seed(43)
    emb = (torch.randn(c.vocab_size, c.hidden_size, generator=g) * 0.1).to(dtype)
    head = (torch.randn(c.vocab_size, c.hidden_size, generator=g) * 0.1).to(dtype)
    return N.DSpark(c, N.initialize(c, 42, dtype), emb, head, device=dev, dtype=dtype)


@cuda
@pytest.mark.parametrize("name,seq,batch", [("tiny", 128, 1), ("tiny-hybrid", 128, 1), ("tiny", 96, 2)])
def test_train_step_gpu_matches_cpu(name, seq, batch):
    c = N.DraftConfig.load(N.config_path(name))
    o = N.Objective(num_anchors=8)
    dtype = torch.bfloat16
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(0, c.vocab_size, (batch, seq), generator=g)
    hs = [torch.randn(batch, seq, c.hidden_size, generator=g).to(dtype) for _ in range(c.num_target_layers)]
    last = torch.randn(batch, seq, c.hidden_size, generator=g).to(dtype)
    mask = torch.ones(batch, seq)
    mask[:, 40:42] = 0
    res = {}
    for dev in ("cpu", "cuda"):
        m = _model(c, dev, dtype)
        opt = N.AdamW(m.sharding, lr=1e-3, weight_decay=0.01)
        torch.manual_seed(0)
        anchors = N.sample_anchors(ids, mask, o)
        to = lambda t: t.to(dev)  # noqa: E731
        losses = []
        for _ in range(2):
            r = N.train(to(ids), m, o, teacher_batch=N.TeacherBatch([to(h) for h in hs], to(last)),
                        loss_mask=to(mask), anchors=(to(anchors[0]), to(anchors[1])), optimizer=None)
            grads = [s.grad.float().cpu().clone() for s in m.sharding]
            u = N.adamw_step(opt, r.metrics.denominator)
            losses.append((r.metrics.loss.item(), r.metrics.accept_len.item(), u["grad_norm"]))
        res[dev] = (losses, grads, [s.master.cpu().clone() for s in m.sharding])
    (lc, gc, mc), (lg, gg, mg) = res["cpu"], res["cuda"]
    for a, b in zip(lc, lg):
        assert abs(a[0] - b[0]) / abs(a[0]) < 0.02
        assert abs(a[1] - b[1]) < 0.05
        assert abs(a[2] - b[2]) / a[2] < 0.05
    for a, b in zip(gc, gg):
        cos = torch.nn.functional.cosine_similarity(a, b, dim=0).item()
        assert cos > 0.99, cos
    for a, b in zip(mc, mg):
        assert ((a - b).norm() / a.norm()).item() < 3e-3


@cuda
def test_train_step_deterministic():
    c = N.DraftConfig.load(N.config_path("tiny-hybrid"))
    o = N.Objective(num_anchors=8)
    ids = torch.randint(0, c.vocab_size, (1, 128), device="cuda")
    hs = [torch.randn(1, 128, c.hidden_size, device="cuda").bfloat16() for _ in range(2)]
    last = torch.randn(1, 128, c.hidden_size, device="cuda").bfloat16()
    out = []
    for _ in range(2):
        m = _model(c, "cuda", torch.bfloat16)
        torch.manual_seed(3)
        r = N.train(ids, m, o, teacher_batch=N.TeacherBatch(hs, last))
        out.append(([s.grad.clone() for s in m.sharding], r.hidden.clone()))
    for a, b in zip(out[0][0], out[1][0]):
        assert torch.equal(a, b)
    assert torch.equal(out[0][1], out[1][1])


@cuda
def test_graphed_step_matches_eager():
    from nanospec_b200.graphs import GraphedStep
    c = N.DraftConfig.load(N.config_path("tiny-hybrid"))
    o = N.Objective(num_anchors=8)
    g = torch.Generator(device="cuda").manual_seed(3)
    ids = torch.randint(0, c.vocab_size, (1, 128), device="cuda", generator=g)
    hs = [torch.randn(1, 128, c.hidden_size, device="cuda", generator=g).bfloat16() for _ in range(2)]
    last = torch.randn(1, 128, c.hidden_size, device="cuda", generator=g).bfloat16()
    mask = torch.ones(1, 128, device="cuda")
    torch.manual_seed(0)
    anchors = N.sample_anchors(ids, mask, o)
    runs = []
    for graphed in (False, True):
        m = _model(c, "cuda", torch.bfloat16)
        opt = N.AdamW(m.sharding, lr=1e-3)
        losses = []
        if graphed:
            gs = GraphedStep(m, o, opt, ids, N.TeacherBatch(hs, last), loss_mask=mask, anchors=anchors, warmup=1)
            for _ in range(3):
                losses.append(float(gs.step().metrics.loss))
        else:
            for _ in range(4):  # the graphed run also performs one eager warm-up step
                r = N.train(ids, m, o, teacher_batch=N.TeacherBatch(hs, last), loss_mask=mask, anchors=anchors,
                            optimizer=opt)
                losses.append(float(r.metrics.loss))
            losses = losses[1:]
        runs.append((losses, [s.master.clone() for s in m.sharding], opt.steps))
    assert runs[0][0] == runs[1][0]
    assert runs[0][2] == runs[1][2] == 4
    for a, b in zip(runs[0][1], runs[1][1]):
        assert torch.equal(a, b)


@cuda
def test_lazy_zero_matches_eager_zero():
    # Skipping the gradient zeroing on one rank must not change any step's result.
    c = N.DraftConfig.load(N.config_path("tiny-hybrid"))
    o = N.Objective(num_anchors=8)
    g = torch.Generator(device="cuda").manual_seed(5)
    ids = torch.randint(0, c.vocab_size, (1, 128), device="cuda", generator=g)
    hs = [torch.randn(1, 128, c.hidden_size, device="cuda", generator=g).bfloat16() for _ in range(2)]
    last = torch.randn(1, 128, c.hidden_size, device="cuda", generator=g).bfloat16()
    runs = []
    for lazy in (False, True):
        m = _model(c, "cuda", torch.bfloat16)
        opt = N.AdamW(m.sharding, lr=1e-3, lazy_zero=lazy)
        torch.manual_seed(11)
        losses = [float(N.train(ids, m, o, teacher_batch=N.TeacherBatch(hs, last), optimizer=opt).metrics.loss)
                  for _ in range(3)]
        runs.append((losses, [s.master.clone() for s in m.sharding]))
    assert runs[0][0] == runs[1][0]
    for a, b in zip(runs[0][1], runs[1][1]):
        assert torch.equal(a, b)


@cuda
def test_fused_grad_norm_matches_separate_pass():
    # The norm written by the weight-gradient GEMM epilogues (+ the uncovered ranges)
    # equals the separate squared-norm pass over the same gradients.
    from nanospec_b200.ops._ext import cuda_ops
    from nanospec_b200.parallel.optim import step_factor
    c = N.DraftConfig.load(N.config_path("tiny-hybrid"))
    o = N.Objective(num_anchors=8)
    g = torch.Generator(device="cuda").manual_seed(9)
    ids = torch.randint(0, c.vocab_size, (1, 128), device="cuda", generator=g)
    hs = [torch.randn(1, 128, c.hidden_size, device="cuda", generator=g).bfloat16() for _ in range(2)]
    last = torch.randn(1, 128, c.hidden_size, device="cuda", generator=g).bfloat16()
    m = _model(c, "cuda", torch.bfloat16)
    torch.manual_seed(4)
    r = N.train(ids, m, o, teacher_batch=N.TeacherBatch(hs, last))
    fused = m._draft_step.norm
    assert fused is not None and fused.ok and fused.offset > 0
    den = r.metrics.denominator.detach().clone().float().reshape(())
    f = step_factor(den, 1, 1).reshape(1).contiguous()
    a = fused.norm2(list(m.sharding), f)
    b = torch.zeros(1, device="cuda")
    for s in m.sharding:
        cuda_ops().grad_norm_sq(s.grad, f, b)
    assert abs(a.item() - b.item()) <= 1e-5 * b.item(), (a.item(), b.item())


@cuda
def test_phase_timer_on_device():
    from nanospec_b200.utils.phases import PhaseTimer
    c = N.DraftConfig.load(N.config_path("tiny-hybrid"))
    m = _model(c, "cuda", torch.bfloat16)
    ids = torch.randint(0, c.vocab_size, (1, 128), device="cuda")
    hs = [torch.randn(1, 128, c.hidden_size, device="cuda").bfloat16() for _ in range(2)]
    last = torch.randn(1, 128, c.hidden_size, device="cuda").bfloat16()
    timer = PhaseTimer("cuda")
    N.train(ids, m, N.Objective(num_anchors=8), teacher_batch=N.TeacherBatch(hs, last),
            optimizer=N.AdamW(m.sharding, lr=1e-3), phases=timer)
    ph = timer.summary()
    assert set(ph) == {"draft_forward", "head", "draft_backward", "optimizer"}
    assert all(v > 0 for v in ph.values())


@cuda
def test_train_raises_when_a_device_wait_times_out():
    """A bounded device wait that runs out inside a real train() step (here: a peer
    flag wait on a flag that nothing sets, injected at the head phase) makes train()
    raise DeviceWaitTimeout on the host instead of returning a silent step; the
    device state is reset and the next step runs normally."""
    from nanospec_b200.ops._ext import cuda_ops
    from nanospec_b200.utils.health import DeviceWaitTimeout
    from nanospec_b200.utils.phases import PhaseTimer
    C = cuda_ops()
    C.clear_device_error()
    wid, _ = C.window_create(1 << 20, 0, 1)
    C.window_open(wid, C.window_ipc_handle(wid).view(1, -1))

    class Stuck(PhaseTimer):
        def mark(self, name):
            super().mark(name)
            if name == "head":
                C.peer_wait(wid, 0, 5, 1, 2000)  # gives up after ~0.4 ms of polling

    c = N.DraftConfig.load(N.config_path("tiny"))
    dev = torch.device("cuda")
    m = _model(c, dev, torch.bfloat16)
    opt = N.AdamW(m.sharding, lr=1e-3)
    o = N.Objective(num_anchors=4)
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(0, c.vocab_size, (1, 64), generator=g).cuda()
    tb = N.TeacherBatch([torch.randn(1, 64, c.hidden_size, generator=g).bfloat16().cuda()
                         for _ in range(c.num_target_layers)],
                        torch.randn(1, 64, c.hidden_size, generator=g).bfloat16().cuda())
    try:
        with pytest.raises(DeviceWaitTimeout, match="peer-memory flag wait.*draft forward/backward"):
            N.train(ids, m, o, teacher_batch=tb, optimizer=opt, phases=Stuck(dev))
        assert C.device_error() == 0  # reset before raising
        r = N.train(ids, m, o, teacher_batch=tb, optimizer=opt)
        assert r.update["updated"]
    finally:
        torch.cuda.synchronize()
        C.window_close(wid)
