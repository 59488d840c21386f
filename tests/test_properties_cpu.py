"""Property tests (hypothesis) of the CPU statements against the reference package.

Random shapes, masks and seeds. The batch preparation, the RMSNorm forward/backward
and the anchor-layout draft attention (split K/V layout, no dense mask tensor in the
API) must reproduce the reference's own functions (nanospec/dspark.py:95-144,
nanospec/ops.py:48-66 and 129-162). These CPU statements are also the oracles the
GPU kernel tests compare against.
"""

import torch
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

import nanospec_b200 as N
from nanospec_b200 import ops

SETTINGS = settings(max_examples=60, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])


@SETTINGS
@given(b=st.integers(1, 3), s=st.integers(24, 80), anchors=st.integers(1, 6), bs=st.integers(2, 7),
       hole=st.integers(0, 20), seed=st.integers(0, 10_000))
def test_prepare_matches_reference(reference, b, s, anchors, bs, hole, seed):
    o = N.Objective(num_anchors=anchors, block_size=bs)
    ro = reference.config.Objective(num_anchors=anchors, block_size=bs)
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, 97, (b, s), generator=g)
    mask = torch.ones(b, s)
    mask[b - 1, hole:hole + 3] = 0
    torch.manual_seed(seed)
    p = N.prepare(ids, mask, o)
    torch.manual_seed(seed)
    q = reference.dspark.prepare(ids, mask, ro)
    for f in ("anchors", "keep", "positions", "target_ids", "previous", "weights", "valid",
              "teacher_indices", "mask"):
        assert torch.equal(getattr(p, f), getattr(q, f)), f


@SETTINGS
@given(rows=st.integers(1, 9), n=st.integers(1, 130), bf16=st.booleans(), seed=st.integers(0, 10_000))
def test_rms_norm_matches_reference(reference, rows, n, bf16, seed):
    dtype = torch.bfloat16 if bf16 else torch.float32
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, n, generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(n, generator=g)).to(dtype)
    dy = torch.randn(rows, n, generator=g).to(dtype)
    y, inv = ops.rms_norm(x, w, 1e-6)
    ry, saved = reference.ops.rms_norm(x, w, 1e-6)
    assert torch.equal(y, ry)
    dw = torch.empty(n, dtype=dtype)
    rdw = torch.empty(n, dtype=dtype)
    dx = ops.rms_norm_backward(dy, x, inv, w, dw)
    rdx = reference.ops.rms_norm_backward(dy, saved, w, rdw)
    torch.testing.assert_close(dx.float(), rdx.float(), rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(dw.float(), rdw.float(), rtol=1e-5, atol=1e-5)


@SETTINGS
@given(b=st.integers(1, 2), s=st.integers(20, 48), nb=st.integers(1, 4), bs=st.integers(2, 6),
       groups=st.sampled_from([1, 2, 4]), hk=st.integers(1, 2), d=st.sampled_from([8, 16]),
       seed=st.integers(0, 10_000))
def test_draft_attention_matches_reference(reference, b, s, nb, bs, groups, hk, d, seed):
    o = N.Objective(num_anchors=nb, block_size=bs)
    ro = reference.config.Objective(num_anchors=nb, block_size=bs)
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, 50, (b, s), generator=g)
    mask = torch.ones(b, s)
    torch.manual_seed(seed)
    p = N.prepare(ids, mask, o)
    torch.manual_seed(seed)
    rp = reference.dspark.prepare(ids, mask, ro)
    nbk = p.anchors.shape[1]  # anchors actually placed
    td = nbk * bs
    hq = hk * groups
    q = torch.randn(b, td, hq, d, generator=g)
    ctx_k, ctx_v = torch.randn(b, s, hk, d, generator=g), torch.randn(b, s, hk, d, generator=g)
    dr_k, dr_v = torch.randn(b, td, hk, d, generator=g), torch.randn(b, td, hk, d, generator=g)
    # split layout: context rows of every batch row, then draft rows of every batch row
    k = torch.cat((ctx_k.reshape(b * s, hk, d), dr_k.reshape(b * td, hk, d)))
    v = torch.cat((ctx_v.reshape(b * s, hk, d), dr_v.reshape(b * td, hk, d)))
    out, lse = ops.attention(q, k, v, p.anchors, p.keep, s, bs)
    # reference: batched [b, heads, keys, d] with its dense [b, 1, td, s + td] mask
    kb = torch.cat((ctx_k, dr_k), 1).transpose(1, 2)
    vb = torch.cat((ctx_v, dr_v), 1).transpose(1, 2)
    rout, saved = reference.ops.attention(q.transpose(1, 2), kb, vb, rp.mask)
    torch.testing.assert_close(out, rout.transpose(1, 2), rtol=1e-5, atol=1e-5)
    dout = torch.randn(b, td, hq, d, generator=g)
    dq, dk, dv = ops.attention_backward(dout, q, k, v, out, lse, p.anchors, p.keep, s, bs)
    rq, rk, rv = reference.ops.attention_backward(dout.transpose(1, 2), saved)
    torch.testing.assert_close(dq, rq.transpose(1, 2), rtol=1e-4, atol=1e-5)
    rk, rv = rk.transpose(1, 2), rv.transpose(1, 2)  # [b, s + td, hk, d]
    torch.testing.assert_close(dk[:b * s].reshape(b, s, hk, d), rk[:, :s], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(dk[b * s:].reshape(b, td, hk, d), rk[:, s:], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(dv[:b * s].reshape(b, s, hk, d), rv[:, :s], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(dv[b * s:].reshape(b, td, hk, d), rv[:, s:], rtol=1e-4, atol=1e-5)


@SETTINGS
@given(b=st.integers(1, 2), s=st.integers(1, 70), h=st.integers(1, 3), dk=st.sampled_from([4, 8]),
       dv=st.sampled_from([4, 8]), chunk=st.sampled_from([4, 16, 64]), seed=st.integers(0, 10_000))
def test_gated_delta_rule_forms_agree(reference, b, s, h, dk, dv, chunk, seed):
    # Our chunked (WY) form, our token-by-token oracle and the reference's chunked
    # implementation (nanospec/ops.py:203-239) give the same outputs.
    from nanospec_b200.ops import reference as ref
    g_ = torch.Generator().manual_seed(seed)
    q = torch.randn(b, s, h, dk, generator=g_)
    k = torch.randn(b, s, h, dk, generator=g_)
    v = torch.randn(b, s, h, dv, generator=g_)
    g = -torch.rand(b, s, h, generator=g_) * 0.5
    beta = torch.rand(b, s, h, generator=g_)
    rec = ref.gated_delta_rule_recurrent(q, k, v, g, beta)
    ours = ref.gated_delta_rule_chunked(q, k, v, g, beta, chunk)
    theirs = reference.ops.chunk_delta_rule(q, k, v, g, beta, chunk_size=chunk)
    torch.testing.assert_close(ours, rec, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(theirs.float(), rec, rtol=1e-4, atol=1e-5)
