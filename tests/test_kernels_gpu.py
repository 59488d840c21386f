"""sm_100a kernels vs the plain PyTorch fp32 statement of the same op (ops.reference)."""

import pytest
import torch

from nanospec_b200 import ops
from nanospec_b200.ops import reference as ref

pytestmark = pytest.mark.gpu

cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")


def C():
    from nanospec_b200.ops._ext import cuda_ops
    return cuda_ops()


def close(a, b, rtol=2e-2, atol=2e-2):
    a, b = a.float().cpu(), b.float().cpu()
    err = (a - b).abs().max().item()
    scale = b.abs().max().item() + 1e-6
    cos = torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0).item()
    assert err <= atol + rtol * scale, f"max err {err} vs scale {scale}"
    assert cos > 0.999 or b.abs().max() < 1e-6, f"cos {cos}"


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(0)
    yield
    if torch.cuda.is_available():
        torch.cuda.synchronize()
        assert C().device_error() == 0


@cuda
@pytest.mark.parametrize("M,N,K", [(128, 64, 64), (256, 128, 512), (304, 200, 1000), (1024, 256, 4096),
                                   (128, 192, 128), (5120, 56, 5120), (96, 40, 64),
                                   # more tiles than SMs: persistent kernel (ragged M/N/K edges)
                                   (2056, 2600, 200), (30720, 56, 384), (4096, 5120, 56)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (True, False), (False, True), (True, True)])
def test_gemm_majors(M, N, K, a_mn, b_mn):
    # TMA needs 16-byte row strides: the contiguous dimension of each operand is a multiple of 8.
    dev = "cuda"
    a = torch.randn(M, K, device=dev).bfloat16()
    b = torch.randn(N, K, device=dev).bfloat16()
    A = a.t().contiguous() if a_mn else a
    B = b.t().contiguous() if b_mn else b
    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    C().gemm_test(A, a_mn, B, b_mn, out, 0)
    close(out, a.float() @ b.float().t(), rtol=1e-2)


@cuda
def test_linear_family_persistent():
    # every product has more output tiles than SMs (persistent kernel, residual / accumulate epilogues)
    T = 4100
    x = torch.randn(T, 3072, device="cuda").bfloat16()
    w = (torch.randn(2560, 3072, device="cuda") * 0.05).bfloat16()
    res = torch.randn(T, 2560, device="cuda").bfloat16()
    close(ops.linear(x, w, residual=res), res.float() + x.float() @ w.float().t())
    dy = torch.randn(T, 2560, device="cuda").bfloat16()
    acc = torch.randn(T, 3072, device="cuda").bfloat16()
    base = acc.clone()
    ops.linear_dgrad(dy, w, out=acc, accumulate=True)
    close(acc, base.float() + dy.float() @ w.float())
    dw = torch.empty(2560, 3072, device="cuda", dtype=torch.bfloat16)
    ops.linear_wgrad(dy, x, dw)
    close(dw, dy.float().t() @ x.float())


@cuda
@pytest.mark.parametrize("splits", [1, 3, 7, 16])  # 3, 7: cluster (DSMEM) reduction; 16: global fix-up
def test_gemm_splitk_deterministic(splits):
    a = torch.randn(512, 2048, device="cuda").bfloat16()
    b = torch.randn(128, 2048, device="cuda").bfloat16()
    o1 = torch.empty(512, 128, device="cuda", dtype=torch.bfloat16)
    o2 = torch.empty_like(o1)
    C().gemm_test(a, False, b, False, o1, splits)
    C().gemm_test(a, False, b, False, o2, splits)
    assert torch.equal(o1, o2)
    close(o1, a.float() @ b.float().t(), rtol=1e-2)


@cuda
@pytest.mark.parametrize("T", [56, 184, 600])
def test_linear_family(T):
    x = torch.randn(T, 1024, device="cuda").bfloat16()
    w = (torch.randn(768, 1024, device="cuda") * 0.05).bfloat16()
    res = torch.randn(T, 768, device="cuda").bfloat16()
    y = ops.linear(x, w, residual=res)
    close(y, res.float() + x.float() @ w.float().t())
    dy = torch.randn(T, 768, device="cuda").bfloat16()
    dx = ops.linear_dgrad(dy, w)
    close(dx, dy.float() @ w.float())
    acc = torch.randn(T, 1024, device="cuda").bfloat16()
    base = acc.clone()
    ops.linear_dgrad(dy, w, out=acc, accumulate=True)
    close(acc, base.float() + dy.float() @ w.float())
    dw = torch.empty(768, 1024, device="cuda", dtype=torch.bfloat16)
    ops.linear_wgrad(dy, x, dw)
    close(dw, dy.float().t() @ x.float())


@cuda
def test_linear_strided_views():
    # K/V projection output views and split-layout inputs are strided row-major.
    big = torch.randn(100, 2048, device="cuda").bfloat16()
    x = big[:, 1024:]
    w = (torch.randn(512, 1024, device="cuda") * 0.05).bfloat16()
    close(ops.linear(x, w), x.float() @ w.float().t())


@cuda
@pytest.mark.parametrize("rows,n", [(56, 5120), (7, 64), (300, 1000), (5, 1001)])  # 1001: scalar path
def test_rms_norm(rows, n):
    x = torch.randn(rows, n, device="cuda").bfloat16()
    w = (1 + 0.1 * torch.randn(n, device="cuda")).bfloat16()
    y, inv = ops.rms_norm(x, w, 1e-6)
    ry, rinv = ref.rms_norm(x, w, 1e-6)
    close(y, ry, rtol=1e-2)
    close(inv, rinv, rtol=1e-5)
    dy = torch.randn(rows, n, device="cuda").bfloat16()
    res = torch.randn(rows, n, device="cuda").bfloat16()
    dw = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    dx = ops.rms_norm_backward(dy, x, inv, w, dw, residual=res)
    rdx, rdw = ref.rms_norm_backward(dy, x, rinv, w)
    close(dx, res.float() + rdx.float(), rtol=2e-2)
    close(dw, rdw, rtol=2e-2)


@cuda
@pytest.mark.parametrize("D", [16, 128])
def test_head_norm_rope(D):
    T, H = 60, 5
    big = torch.randn(T, 2 * H * D, device="cuda").bfloat16()
    x = big[:, :H * D].view(T, H, D)  # strided rows, like the K half of a K/V projection
    w = (1 + 0.1 * torch.randn(D, device="cuda")).bfloat16()
    pos = torch.randint(0, 500, (T,), device="cuda")
    cos, sin = ref.rotary_factors(pos, D, 1e6, torch.bfloat16)
    y, inv = ops.head_norm_rope(x, w, 1e-6, cos, sin)
    ry, rinv = ref.head_norm_rope(x, w, 1e-6, cos, sin)
    close(y, ry, rtol=1e-2)
    dy = torch.randn(T, H, D, device="cuda").bfloat16()
    dw = torch.empty(D, device="cuda", dtype=torch.bfloat16)
    dxbig = torch.zeros(T, 2 * H * D, device="cuda", dtype=torch.bfloat16)
    ops.head_norm_rope_backward(dy, x, inv, w, cos, sin, dw, out=dxbig[:, :H * D].view(T, H, D))
    rdx, rdw = ref.head_norm_rope_backward(dy, x, rinv, w, cos, sin)
    close(dxbig[:, :H * D].view(T, H, D), rdx, rtol=2e-2)
    close(dw, rdw, rtol=2e-2)
    assert dxbig[:, H * D:].abs().max() == 0


@cuda
def test_swiglu():
    gu = torch.randn(56, 2 * 640, device="cuda").bfloat16()
    p = ops.swiglu(gu)
    close(p, torch.nn.functional.silu(gu[:, :640].float()) * gu[:, 640:].float())
    dp = torch.randn(56, 640, device="cuda").bfloat16()
    dgu = ops.swiglu_backward(dp, gu)
    dg, du = ref.swiglu_backward(dp.float(), gu[:, :640].float(), gu[:, 640:].float())
    close(dgu[:, :640], dg)
    close(dgu[:, 640:], du)


@cuda
def test_embedding():
    w = torch.randn(300, 64, device="cuda").bfloat16()
    ids = torch.randint(0, 300, (90,), device="cuda")
    ids[5] = ids[9] = 17  # repeated rows accumulate
    assert torch.equal(ops.embedding(ids, w), w[ids])
    dy = torch.randn(90, 64, device="cuda").bfloat16()
    g = torch.full((300, 64), 7.0, device="cuda", dtype=torch.bfloat16)  # must be overwritten
    ops.embedding_backward(dy, ids, g)
    close(g, ref.embedding_backward(dy, ids, 300))


def _attn_case(b=2, S=40, nb=4, bs=7, hq=10, hk=2, d=128):
    td = nb * bs
    q = torch.randn(b, td, hq, d, device="cuda").bfloat16()
    kv = torch.randn(b * (S + td), 2 * hk * d, device="cuda").bfloat16()
    k = kv[:, :hk * d].view(-1, hk, d)
    v = kv[:, hk * d:].view(-1, hk, d)
    anchors = torch.randint(0, S - bs, (b, nb), device="cuda")
    anchors[0, 0] = 0
    keep = torch.ones(b, nb, dtype=torch.bool, device="cuda")
    keep[1, -1] = False
    return q, k, v, anchors, keep, S, bs


@cuda
@pytest.mark.parametrize("d,hq,hk,S,bs", [(128, 10, 2, 40, 7), (128, 40, 8, 130, 7), (32, 4, 2, 70, 7),
                                         (64, 4, 2, 70, 12), (32, 2, 2, 50, 20)])  # row capacities 8 / 16 / 32
def test_attention(d, hq, hk, S, bs):
    q, k, v, anchors, keep, S, bs = _attn_case(hq=hq, hk=hk, d=d, S=S, bs=bs)
    out, lse = ops.attention(q, k, v, anchors, keep, S, bs)
    qc, kc, vc = q.cpu().float(), k.cpu().float(), v.cpu().float()
    rout, rlse = ops.attention(qc, kc, vc, anchors.cpu(), keep.cpu(), S, bs)
    close(out, rout, rtol=1e-2)
    assert torch.allclose(lse.cpu()[rlse.isfinite()], rlse[rlse.isfinite()], atol=1e-3)
    assert torch.equal(lse.cpu().isfinite(), rlse.isfinite())
    dout = torch.randn_like(q)
    dq, dk, dv = ops.attention_backward(dout, q, k, v, out, lse, anchors, keep, S, bs)
    rq, rk, rv = ops.attention_backward(dout.cpu().float(), qc, kc, vc, out.cpu().float(), rlse,
                                        anchors.cpu(), keep.cpu(), S, bs)
    close(dq, rq, rtol=2e-2)
    close(dk, rk, rtol=2e-2)
    close(dv, rv, rtol=2e-2)


@cuda
@pytest.mark.parametrize("path", ["streamed", "materialize"])
@pytest.mark.parametrize("markov,teacher_logits,chunk", [(True, False, 0), (False, False, 0), (True, True, 0),
                                                          (True, False, 4096), (True, True, 4096)])
def test_head_loss(markov, teacher_logits, chunk, path, monkeypatch):
    """Both CUDA head paths against the fp32 statements: the streamed one (logits
    only in TMEM, gradient per vocabulary chunk) and the materialised one."""
    import nanospec_b200 as N
    import nanospec_b200.ops.head as head_mod
    from nanospec_b200.objective import head_loss
    monkeypatch.setattr(head_mod, "VOCAB_CHUNK", chunk)  # 0: whole vocabulary; 4096: five chunks
    monkeypatch.setenv("NANOSPEC_HEAD", path)
    torch.manual_seed(1)
    V, H, r = 20003, 256, 32  # V % 8 != 0: scalar tails and padded row strides
    b, nb, bs, S = 1, 8, 7, 64
    o = N.Objective(num_anchors=nb, block_size=bs)
    ids = torch.randint(0, V, (b, S))
    mask = torch.ones(b, S)
    mask[0, 30:32] = 0
    torch.manual_seed(3)
    prep = N.prepare(ids, mask, o)
    t = b * nb * bs
    hid = (torch.randn(t, H) * 0.5).bfloat16()
    W = (torch.randn(V, H) * 0.1).bfloat16()
    th = (torch.randn(t, H) * 0.5).bfloat16()
    e = (torch.randn(t, r) * 0.5).bfloat16() if markov else None
    w2 = (torch.randn(V, r) * 0.1).bfloat16() if markov else None
    tl = (torch.randn(t, V) * 2).bfloat16() if teacher_logits else None
    kw = dict(target_logits=tl) if teacher_logits else dict(target_hidden=th)
    dw2 = torch.empty(V, r).bfloat16() if markov else None
    m_ref, dh_ref, de_ref = head_loss(hid, W, e, w2, prep, o, dw2_out=dw2, **kw)

    def g(x):
        return None if x is None else x.cuda()
    prep_g = N.prepare(ids.cuda(), mask.cuda(), o, anchors=(prep.anchors.cuda(), prep.keep.cuda()))
    kwg = {k: g(v) for k, v in kw.items()}
    dw2g = torch.empty(V, r, device="cuda").bfloat16() if markov else None
    m, dh, de = head_loss(g(hid), g(W), g(e), g(w2), prep_g, o, dw2_out=dw2g, **kwg)
    for f in ("ce", "kl", "numerator", "denominator", "accept_len_sum", "accept_len_total"):
        a, bb = getattr(m, f).item(), getattr(m_ref, f).item()
        assert abs(a - bb) <= 2e-3 * max(1.0, abs(bb)), (f, a, bb)
    close(dh, dh_ref, rtol=3e-2)
    if markov:
        close(de, de_ref, rtol=3e-2)
        close(dw2g, dw2, rtol=3e-2)


@cuda
def test_adamw_matches_reference():
    import nanospec_b200 as N
    from nanospec_b200.parallel.optim import adamw_step

    class U:  # a minimal one-rank shard
        pass
    torch.manual_seed(0)
    shards = []
    for dev in ("cpu", "cuda"):
        u = U()
        gen = torch.Generator().manual_seed(5)
        u.param = torch.randn(10000, generator=gen).bfloat16().to(dev)
        u.master = u.param.float()
        u.m = torch.zeros_like(u.master)
        u.v = torch.zeros_like(u.master)
        u.grad = (torch.randn(10000, generator=gen) * 0.01).bfloat16().to(dev)
        u.world_size, u.group = 1, None
        shards.append(u)
    res = []
    for u in shards:
        opt = N.AdamW([u], lr=1e-3, weight_decay=0.01)
        res.append(adamw_step(opt, torch.tensor(37.0, device=u.param.device)))
    assert abs(res[0]["grad_norm"] - res[1]["grad_norm"]) < 1e-4 * res[0]["grad_norm"]
    close(shards[1].master.cpu(), shards[0].master, rtol=1e-5, atol=1e-6)
    assert shards[1].grad.abs().max().item() == 0


@cuda
def test_adamw_nonfinite_skips():
    import nanospec_b200 as N
    from nanospec_b200.parallel.optim import adamw_step

    class U:
        pass
    u = U()
    u.param = torch.ones(1000, device="cuda").bfloat16()
    u.master = u.param.float()
    u.m = torch.zeros_like(u.master)
    u.v = torch.zeros_like(u.master)
    u.grad = torch.ones(1000, device="cuda").bfloat16()
    u.grad[3] = float("nan")
    u.world_size, u.group = 1, None
    opt = N.AdamW([u], lr=1e-3)
    r = adamw_step(opt, torch.tensor(10.0, device="cuda"))
    assert r["updated"] is False and opt.steps == 0
    assert torch.equal(u.master, torch.ones(1000, device="cuda"))
    assert u.grad.abs().max().item() == 0


@cuda
@pytest.mark.parametrize("nout,k", [(2560, 3072), (96, 200)])  # persistent / single-wave kernels
def test_wgrad_norm_side_output(nout, k):
    # Per-CTA partials of sum bf16(dW * f)^2 written by the GEMM equal the norm pass over dW.
    T = 56
    dy = torch.randn(T, nout, device="cuda").bfloat16()
    x = torch.randn(T, k, device="cuda").bfloat16()
    out = torch.empty(nout, k, device="cuda", dtype=torch.bfloat16)
    f = torch.tensor([0.37], device="cuda")
    part = torch.full((4096,), float("nan"), device="cuda")
    used = C().linear_wgrad(dy, x, out, False, f, part, 5)
    assert 0 < used <= 148 * 4
    close(out, dy.float().t() @ x.float())
    ref = torch.zeros(1, device="cuda")
    C().grad_norm_sq(out.reshape(-1), f, ref)
    got = part[5:5 + used].sum().item()
    assert abs(got - ref.item()) <= 1e-5 * ref.item(), (got, ref.item())


@cuda
def test_grad_norm_ranges_matches_per_range():
    g = torch.randn(300001, device="cuda").bfloat16()
    f = torch.tensor([1.7], device="cuda")
    ranges = [g[3:1000], g[1000:1001], g[5000:250007], g[250007:]]  # unaligned starts, a 1-element range
    a = torch.zeros(1, device="cuda")
    C().grad_norm_sq_ranges(ranges, f, a)
    b = torch.zeros(1, device="cuda")
    for r in ranges:
        C().grad_norm_sq(r, f, b)
    ref = (g[3:].float() * 1.7).bfloat16().float().square().sum().item() - \
        (g[1001:5000].float() * 1.7).bfloat16().float().square().sum().item()
    assert abs(a.item() - b.item()) <= 1e-5 * b.item()
    assert abs(a.item() - ref) <= 1e-4 * ref
