"""Verifier kernels (FP8 GEMM, GDN, conv, norms, attention) vs the CPU statements."""

import pytest
import torch

from nanospec_b200.ops import reference as ref
from nanospec_b200.ops import verifier_ops as vops

pytestmark = pytest.mark.gpu
cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")


def close(a, b, rtol=2e-2, cos_min=0.999):
    a, b = a.float().cpu(), b.float().cpu()
    err = (a - b).abs().max().item()
    scale = b.abs().max().item() + 1e-6
    cos = torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0).item()
    assert err <= rtol * scale + 1e-3, f"max err {err} vs scale {scale}"
    assert cos > cos_min, f"cos {cos}"


@pytest.fixture(autouse=True)
def _check():
    torch.manual_seed(0)
    yield
    if torch.cuda.is_available():
        torch.cuda.synchronize()
        from nanospec_b200.ops._ext import cuda_ops
        assert cuda_ops().device_error() == 0


@cuda
@pytest.mark.parametrize("T,K,N", [(200, 512, 384), (16, 256, 128), (1000, 1024, 640), (300, 512, 768),
                                   (128, 256, 512), (1100, 1024, 2560)])
def test_fp8_linear(T, K, N):
    from nanospec_b200.models.verifier import quantize_weight_blocks
    x = torch.randn(T, K).bfloat16()
    w, s = quantize_weight_blocks(torch.randn(N, K) * 0.05)
    expect = ref.fp8_linear(x, w, s)
    got = vops.fp8_linear(x.cuda(), w.cuda(), s.cuda())
    close(got, expect, rtol=1e-2, cos_min=0.9999)


@cuda
def test_small_verifier_ops():
    x = torch.randn(3, 50, 96).bfloat16()
    w = (torch.randn(96) * 0.1).bfloat16()
    close(vops.qwen_norm(x.cuda(), w.cuda(), 1e-6), ref.qwen_norm(x, w, 1e-6), rtol=1e-2)
    gt = torch.randn(150, 96).bfloat16()
    close(vops.qwen_gated_norm(x.view(-1, 96).cuda(), gt.cuda(), w.cuda(), 1e-6),
          ref.qwen_gated_norm(x.view(-1, 96), gt, w, 1e-6), rtol=2e-2)
    cw = (torch.randn(96, 1, 4) * 0.3).bfloat16()
    close(vops.causal_conv_silu(x.cuda(), cw.cuda()), ref.causal_conv_silu(x, cw), rtol=2e-2)
    # the row-strided, token-windowed conv of the fused path: the first 96 channels of
    # 160-wide rows, three sequences of 50 tokens (windows straddle sequence starts)
    xr = torch.randn(3, 50, 160).bfloat16()
    close(vops.causal_conv_silu_rows(xr.cuda(), 160, cw.cuda(), 96), ref.causal_conv_silu(xr[..., :96], cw),
          rtol=2e-2)
    a, b = torch.randn(3, 50, 6).bfloat16(), torch.randn(3, 50, 6).bfloat16()
    alog, dtb = torch.randn(6), torch.rand(6)
    g1, b1 = vops.gdn_gates(a.cuda(), b.cuda(), alog.cuda(), dtb.cuda())
    g2, b2 = ref.gdn_gates(a, b, alog, dtb)
    close(g1, g2, rtol=1e-3)
    close(b1, b2, rtol=1e-2)


@cuda
@pytest.mark.parametrize("D,s,groups", [(16, 100, 2), (128, 130, 3)])
def test_gated_delta_rule(D, s, groups):
    b, nk = 2, 2
    nv = nk * groups
    q = torch.randn(b, s, nk, D).bfloat16()
    k = torch.randn(b, s, nk, D).bfloat16()
    v = torch.randn(b, s, nv, D).bfloat16()
    g = -torch.rand(b, s, nv) * 0.5
    beta = torch.rand(b, s, nv).bfloat16()
    got = vops.gated_delta_rule(q.cuda(), k.cuda(), v.cuda(), g.cuda(), beta.cuda(), groups)
    expect = ref.gated_delta_rule_recurrent(q.repeat_interleave(groups, 2).double(),
                                            k.repeat_interleave(groups, 2).double(), v.double(), g.double(),
                                            beta.double())
    close(got, expect, rtol=3e-2, cos_min=0.999)


@cuda
@pytest.mark.parametrize("D,rd,hq,hk,s", [(32, 16, 4, 2, 70), (256, 64, 6, 2, 150)])
def test_causal_attention_gated(D, rd, hq, hk, s):
    b = 2
    q = torch.randn(b, s, hq, D).bfloat16()
    k = torch.randn(b, s, hk, D).bfloat16()
    v = torch.randn(b, s, hk, D).bfloat16()
    gate = torch.randn(b, s, hq, D).bfloat16()
    pos = torch.arange(s).expand(b, s)
    cos, sin = ref.rotary_factors(pos, rd, 1e6, torch.bfloat16)
    expect = vops.causal_attention_gated(q, k, v, gate, cos, sin, rd)
    got = vops.causal_attention_gated(q.cuda(), k.cuda(), v.cuda(), gate.cuda(), cos.cuda(), sin.cuda(), rd)
    close(got, expect, rtol=3e-2, cos_min=0.999)


@cuda
def test_stage_forward_matches_cpu(tmp_path):
    from nanospec_b200.models.verifier import (Checkpoint, QwenStage, stage_forward, tiny_hybrid_text_config,
                                               write_synthetic_checkpoint)
    tc = tiny_hybrid_text_config(hidden=128, vocab=512, heads=4, head_dim=32, ffn=256)
    path = write_synthetic_checkpoint(tmp_path / "ckpt", tc, seed=1, fp8=True)
    ck = Checkpoint(path)
    ids = torch.randint(0, 512, (2, 96))
    outs = {}
    for dev in ("cpu", "cuda"):
        st = QwenStage(ck, 0, 4, device=dev, first=True, last=True)
        x, cap = stage_forward(st, ids.to(dev), capture=(1, 3))
        outs[dev] = (x, cap)
    close(outs["cuda"][0], outs["cpu"][0], rtol=5e-2, cos_min=0.995)
    for i in (1, 3):
        close(outs["cuda"][1][i], outs["cpu"][1][i], rtol=5e-2, cos_min=0.995)


@cuda
@pytest.mark.parametrize("D,s,groups", [(16, 70, 2), (64, 200, 1), (128, 130, 3), (128, 64, 1)])
def test_gated_delta_rule_backward(D, s, groups):
    """Head dims 64 / 128 run the chunked kernels, 16 the token-serial ones; both
    against autograd through the fp32 token recurrence."""
    b, nk = 1, 2
    nv = nk * groups
    q = torch.randn(b, s, nk, D).bfloat16()
    k = torch.randn(b, s, nk, D).bfloat16()
    v = torch.randn(b, s, nv, D).bfloat16()
    g = -torch.rand(b, s, nv) * 0.5
    beta = torch.rand(b, s, nv).bfloat16()
    dout = torch.randn(b, s, nv, D).bfloat16()
    expect = vops.gated_delta_rule_backward(q, k, v, g, beta, dout, groups)
    got = vops.gated_delta_rule_backward(q.cuda(), k.cuda(), v.cuda(), g.cuda(), beta.cuda(), dout.cuda(), groups)
    for name, x, y in zip(("dq", "dk", "dv", "dg", "dbeta"), got, expect):
        close(x, y, rtol=3e-2, cos_min=0.999)


@cuda
def test_chunked_and_serial_gdn_backward_agree(monkeypatch):
    """The chunked kernels and the token-serial kernels give the same gradients."""
    torch.manual_seed(5)
    b, s, nk, groups, D = 2, 300, 2, 2, 128
    nv = nk * groups
    q = torch.randn(b, s, nk, D).bfloat16().cuda()
    k = torch.randn(b, s, nk, D).bfloat16().cuda()
    v = torch.randn(b, s, nv, D).bfloat16().cuda()
    g = (-torch.rand(b, s, nv) * 0.5).cuda()
    beta = torch.rand(b, s, nv).bfloat16().cuda()
    dout = torch.randn(b, s, nv, D).bfloat16().cuda()
    chunked = vops.gated_delta_rule_backward(q, k, v, g, beta, dout, groups)
    monkeypatch.setenv("NANOSPEC_GDN_BWD", "serial")
    serial = vops.gated_delta_rule_backward(q, k, v, g, beta, dout, groups)
    for x, y in zip(chunked, serial):
        close(x.cpu(), y.cpu(), rtol=2e-2, cos_min=0.9999)


@cuda
@pytest.mark.parametrize("D,rd,hq,hk,s,b", [(64, 32, 4, 2, 200, 2), (128, 64, 4, 4, 130, 1),
                                          (256, 64, 6, 2, 150, 2), (256, 64, 24, 4, 640, 1)])
def test_gated_attention_tensor_core_path(D, rd, hq, hk, s, b):
    """Fused norm + partial RoPE + tcgen05 flash attention + sigmoid gate vs the CPU
    statements (qwen_norm, partial_rope, bf16 scores, fp32 softmax, bf16 P @ V)."""
    qg = torch.randn(b, s, hq, 2 * D).bfloat16()
    k = torch.randn(b, s, hk, D).bfloat16()
    v = torch.randn(b, s, hk, D).bfloat16()
    wq = (torch.randn(D) * 0.1).bfloat16()
    wk = (torch.randn(D) * 0.1).bfloat16()
    pos = torch.arange(s).expand(b, s)
    cos, sin = ref.rotary_factors(pos, rd, 1e7, torch.bfloat16)
    expect = vops.gated_attention(qg, k, v, wq, wk, 1e-6, cos, sin, rd)
    got = vops.gated_attention(qg.cuda(), k.cuda(), v.cuda(), wq.cuda(), wk.cuda(), 1e-6, cos.cuda(), sin.cuda(), rd)
    close(got, expect, rtol=3e-2, cos_min=0.999)


@cuda
def test_gated_attention_large_logits_rescale():
    """Large, growing scores (norm weight 3 gives logits of std ~20) force the kernel's
    running-maximum rescale of O in TMEM. Oracle: the same normalised, RoPE'd q / k
    with fp32 scores and softmax (the bf16-score statement is too coarse at this scale)."""
    b, s, hq, hk, D, rd = 1, 384, 2, 1, 128, 32
    qg = torch.randn(b, s, hq, 2 * D).bfloat16()
    k = torch.randn(b, s, hk, D).bfloat16()
    v = torch.randn(b, s, hk, D).bfloat16()
    w = torch.full((D,), 3.0).bfloat16()
    pos = torch.arange(s).expand(b, s)
    cos, sin = ref.rotary_factors(pos, rd, 1e7, torch.bfloat16)
    q = ref.partial_rope(vops.qwen_norm(qg[..., :D], w, 1e-6), cos, sin, rd)
    kr = ref.partial_rope(vops.qwen_norm(k, w, 1e-6), cos, sin, rd)
    g = hq // hk
    qt = q.float().transpose(1, 2)
    kt = kr.float().repeat_interleave(g, 2).transpose(1, 2)
    vt = v.float().repeat_interleave(g, 2).transpose(1, 2)
    sc = (qt @ kt.transpose(-1, -2)) * D ** -0.5
    assert sc.std() > 10  # the rescale path is exercised
    sc = sc.masked_fill(torch.ones(s, s, dtype=torch.bool).triu(1), float("-inf"))
    o = (sc.softmax(-1) @ vt).transpose(1, 2).bfloat16()
    expect = o * qg[..., D:].sigmoid()
    got = vops.gated_attention(qg.cuda(), k.cuda(), v.cuda(), w.cuda(), w.cuda(), 1e-6, cos.cuda(), sin.cuda(), rd)
    close(got, expect, rtol=3e-2, cos_min=0.999)


@cuda
def test_fused_stage_matches_cpu(tmp_path):
    """The CUDA fused path (concatenated projections, residual add fused with the next
    norm, producers that emit e4m3 + scales, tcgen05 attention, chunked GDN) against
    the CPU statement path on a small config with the 27B head geometry (d_v = 128,
    attention head_dim 128, FP8 projections)."""
    from nanospec_b200.models.verifier import (Checkpoint, QwenStage, stage_forward, tiny_hybrid_text_config,
                                               write_synthetic_checkpoint)
    tc = tiny_hybrid_text_config(hidden=256, vocab=512, heads=2, head_dim=128, ffn=512)
    tc.update(linear_num_key_heads=1, linear_num_value_heads=2, linear_key_head_dim=128, linear_value_head_dim=128,
              num_key_value_heads=1)
    path = write_synthetic_checkpoint(tmp_path / "ckpt", tc, seed=3, fp8=True)
    ck = Checkpoint(path)
    ids = torch.randint(0, 512, (2, 200))
    outs = {}
    for dev in ("cpu", "cuda"):
        st = QwenStage(ck, 0, 4, device=dev, first=True, last=True)
        assert st.fused == (dev == "cuda")
        outs[dev] = stage_forward(st, ids.to(dev), capture=(0, 1, 2, 3))
    # The fused CUDA path against the CUDA statement path: the same mixer kernels, so
    # only the fusion (concatenated GEMMs, add+norm, quantising producers) differs and
    # only through roundings inside fp32 reductions (a 1-ulp bf16 flip of a norm output
    # can move an e4m3 code). With random weights such differences grow by a few times
    # per layer, so the criterion is relative L2 and cosine, not the largest element.
    st = QwenStage(ck, 0, 4, device="cuda", first=True, last=True)
    st.fused = False
    plain = stage_forward(st, ids.cuda(), capture=(0, 1, 2, 3))
    for got, ref_ in [(outs["cuda"][1][i], plain[1][i]) for i in range(4)] + [(outs["cuda"][0], plain[0])]:
        rel_close(got, ref_, rel=3e-2, cos_min=0.9995)
    # against the CPU statements (bf16 attention scores, fp32 dequantised GEMMs, fp32 GDN)
    for got, ref_ in [(outs["cuda"][1][i], outs["cpu"][1][i]) for i in range(4)] + [(outs["cuda"][0], outs["cpu"][0])]:
        rel_close(got, ref_, rel=1e-1, cos_min=0.995)


def rel_close(a, b, rel, cos_min):
    a, b = a.float().cpu(), b.float().cpu()
    r = ((a - b).norm() / b.norm().clamp_min(1e-12)).item()
    cos = torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0).item()
    assert r <= rel and cos >= cos_min, f"relative L2 {r:.3e}, cos {cos:.6f}"
