"""Verifier (frozen Qwen3.5 hybrid) ops: forward only.

CUDA tensors run the sm_100a kernels of ``nanospec_b200._C``; CPU tensors run the
plain PyTorch statements in ``ops.reference`` (reference math:
nanospec/ops.py:85-239 and the verifier loop of nanospec/train.py:53-157).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import reference as ref
from ._ext import cuda_ops


def _c():
    return cuda_ops()


def embedding(ids, w):
    if w.is_cuda:
        out = torch.empty(*ids.shape, w.shape[1], device=w.device, dtype=w.dtype)
        _c().embedding_fwd(ids.reshape(-1).contiguous(), w, out.view(-1, w.shape[1]))
        return out
    return F.embedding(ids, w)


def add(x, y):
    """x + y in the compute dtype (one rounding)."""
    if x.is_cuda:
        out = torch.empty_like(x)
        _c().add_bf16(x.contiguous(), y.contiguous(), out)
        return out
    return x + y


def silu_mul(gate, up):
    """bf16(bf16(silu(gate)) * up)."""
    if gate.is_cuda:
        m = gate.shape[-1]
        out = torch.empty_like(gate)
        _c().silu_mul(gate.contiguous().view(-1, m), up.contiguous().view(-1, m), out.view(-1, m))
        return out
    return F.silu(gate) * up


def qwen_norm(x, w, eps):
    """(1 + w)-RMSNorm over the last dim, fp32 inside, one cast."""
    if x.is_cuda:
        n = x.shape[-1]
        out = torch.empty(x.shape, device=x.device, dtype=x.dtype)
        _c().qwen_norm(x.reshape(-1, n) if x.is_contiguous() else x.contiguous().view(-1, n), w, float(eps),
                       out.view(-1, n))
        return out
    return ref.qwen_norm(x, w, eps)


def qwen_gated_norm(x, gate, w, eps):
    if x.is_cuda:
        n = x.shape[-1]
        out = torch.empty(x.shape, device=x.device, dtype=x.dtype)
        _c().gated_norm(x.contiguous().view(-1, n), gate.contiguous().view(-1, n), w, float(eps), out.view(-1, n))
        return out
    return ref.qwen_gated_norm(x, gate, w, eps)


def fp8_linear(x, w, scale_inv):
    """Block-scaled FP8 projection (1 x 128 dynamic activations, 128 x 128 weight blocks)."""
    if x.is_cuda:
        n_out = w.shape[0]
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        out = torch.empty(x2.shape[0], n_out, device=x.device, dtype=x.dtype)
        if w.dtype == torch.float8_e4m3fn:
            _c().fp8_linear(x2.contiguous(), w, scale_inv, out)
        else:
            _c().linear(x2.contiguous(), w, out, None)
        return out.view(*lead, n_out)
    return ref.fp8_linear(x, w, scale_inv)


def causal_conv_silu(x, w):
    """Depthwise causal conv (kernel K) + SiLU over tokens; x [b, s, C] token-major."""
    if x.is_cuda:
        out = torch.empty_like(x)
        _c().conv_silu(x.contiguous(), w.reshape(w.shape[0], -1).contiguous(), out)
        return out
    return ref.causal_conv_silu(x, w)


def gdn_gates(a, b, a_log, dt_bias):
    if a.is_cuda:
        g = torch.empty(a.shape, device=a.device, dtype=torch.float32)
        beta = torch.empty(b.shape, device=b.device, dtype=b.dtype)
        _c().gdn_gates(a.contiguous(), b.contiguous(), a_log.float().contiguous(), dt_bias.float().contiguous(), g, beta)
        return g, beta
    return ref.gdn_gates(a, b, a_log, dt_bias)


def gated_delta_rule(q, k, v, g, beta, groups=1, chunk=64):
    """Gated delta rule with GQA: value head h uses key head h // groups.

    q, k [b, s, nk, dk]; v [b, s, nv, dv]; g [b, s, nv] fp32; beta [b, s, nv].
    """
    if q.is_cuda:
        out = torch.empty(v.shape, device=v.device, dtype=v.dtype)
        _c().gdn_chunk_fwd(_rows(q), _rows(k), _rows(v), g.contiguous(), beta.contiguous(), int(groups), out)
        return out
    if groups > 1:
        q = q.repeat_interleave(groups, 2)
        k = k.repeat_interleave(groups, 2)
    return ref.gated_delta_rule_chunked(q, k, v, g, beta, chunk)


def _rows(t):
    """``t`` [b, s, heads, D] as the kernels read it: contiguous heads and one token
    stride (a view into a fused projection qualifies); otherwise a contiguous copy."""
    b, s, h, d = t.shape
    ok = (t.stride(3) == 1 and t.stride(2) == d and t.stride(0) == s * t.stride(1) and t.stride(1) % 4 == 0
          and t.data_ptr() % 8 == 0)
    return t if ok else t.contiguous()


def rotary_factors(positions, dim, theta, dtype):
    return ref.rotary_factors(positions, dim, theta, dtype)


def causal_attention_gated(q, k, v, gate, cos, sin, rotary_dim):
    """Partial RoPE on q/k, causal GQA attention, then ``out * sigmoid(gate)``.

    q [b, s, Hq, D] and k, v [b, s, Hk, D] (q, k already (1+w)-normalised); gate
    [b, s, Hq, D]; cos/sin [b, s, rotary_dim]. Returns [b, s, Hq, D].
    """
    if q.is_cuda:
        out = torch.empty(q.shape, device=q.device, dtype=q.dtype)
        _c().causal_attn_fwd(q.contiguous(), k.contiguous(), v.contiguous(), gate.contiguous(),
                             cos[0].contiguous(), sin[0].contiguous(), int(rotary_dim), out)
        return out
    q = ref.partial_rope(q, cos, sin, rotary_dim)
    k = ref.partial_rope(k, cos, sin, rotary_dim)
    o = ref.causal_attention(q, k, v)
    return o * gate.sigmoid()


def gated_attention(qg, k, v, q_norm_w, k_norm_w, eps, cos, sin, rotary_dim):
    """The verifier's full-attention mixer after its projections.

    qg [b, s, Hq, 2D] is the interleaved q_proj output (query | output gate per head),
    k and v [b, s, Hk, D]. Per head: (1+w)-RMSNorm of q and k, partial RoPE on their
    first ``rotary_dim`` channels, causal GQA softmax attention, then
    ``out * sigmoid(gate)``; returns [b, s, Hq, D]. Reference statement order:
    nanospec/train.py:109-136 with nanospec/ops.py:115-126.

    CUDA: one fused norm + RoPE kernel per operand, then the tcgen05 flash-attention
    kernel (head_dim 64, 128 or 256; the scores never reach HBM). Narrower test
    heads use the CUDA-core kernel.
    """
    b, s, hq, d2 = qg.shape
    d = d2 // 2
    hk = k.shape[2]
    if qg.is_cuda and d in (64, 128, 256) and qg.stride(-1) == 1 and k.stride(-1) == 1 and v.stride(-1) == 1:
        # q / gate / k / v may be strided views of one fused projection output
        c = _c()
        cs, sn = cos[0].contiguous(), sin[0].contiguous()
        q_rot = torch.empty(b, s, hq, d, device=qg.device, dtype=qg.dtype)
        k_rot = torch.empty(b, s, hk, d, device=qg.device, dtype=qg.dtype)
        c.head_norm_rope(qg, hq, qg.stride(1), qg.stride(2), s, q_norm_w, float(eps), cs, sn, int(rotary_dim), q_rot)
        c.head_norm_rope(k, hk, k.stride(1), k.stride(2), s, k_norm_w, float(eps), cs, sn, int(rotary_dim), k_rot)
        out = torch.empty(b, s, hq, d, device=qg.device, dtype=qg.dtype)
        c.vattn_fwd(q_rot, k_rot, v, qg[..., d:], qg.stride(1), qg.stride(2), out)
        return out
    q, gate = qg[..., :d], qg[..., d:]
    q = qwen_norm(q, q_norm_w, eps)
    k = qwen_norm(k, k_norm_w, eps)
    return causal_attention_gated(q, k, v, gate, cos, sin, rotary_dim)


# ---------------------------------------------------------------------------- fused producers (CUDA)
def quantize(x):
    """1 x 128 dynamic e4m3 quantisation of bf16 rows: (codes uint8 [T, K], scales fp32 [T, K/128])."""
    t, k = x.shape
    q = torch.empty(t, k, device=x.device, dtype=torch.uint8)
    s = torch.empty(t, k // 128, device=x.device, dtype=torch.float32)
    _c().quant_e4m3(x.contiguous(), q, s)
    return q, s


def fp8_gemm(q, s, w, scale_inv):
    """bf16 [T, N] = block-scaled GEMM of pre-quantised activations (``quantize``) and e4m3 weights."""
    out = torch.empty(q.shape[0], w.shape[0], device=q.device, dtype=torch.bfloat16)
    _c().fp8_gemm(q, s, w, scale_inv, out)
    return out


def add_norm(x, y, w, eps, *, want_bf16=True, want_q=False, peer=None):
    """x' = x + y (y may be None), n = (1+w)-RMSNorm(x'); returns (x', n bf16 or None,
    (codes, scales) or None). One kernel; the quantised form feeds ``fp8_gemm``.

    ``peer``: ``(window id, (x_dst, x_off) or None, (n_dst, n_off) or None)``; the
    kernel's epilogue then also stores x' / n into rank x_dst's / n_dst's peer window
    at those byte offsets (the verifier -> trainer hand-off)."""
    h = x.shape[-1]
    rows = x.numel() // h
    x2 = x.reshape(rows, h)
    xo = torch.empty_like(x2) if y is not None else None
    n = torch.empty_like(x2) if (want_bf16 or (peer is not None and peer[2] is not None)) else None
    q = torch.empty(rows, h, device=x.device, dtype=torch.uint8) if want_q else None
    sc = torch.empty(rows, h // 128, device=x.device, dtype=torch.float32) if want_q else None
    y2 = None if y is None else y.reshape(rows, h)
    if peer is None:
        _c().add_norm(x2, y2, w, float(eps), xo, n, q, sc)
    else:
        win, xt, nt = peer
        xd, xof = xt if xt is not None else (-1, 0)
        nd, nof = nt if nt is not None else (-1, 0)
        _c().add_norm_peer(x2, y2, w, float(eps), xo, n, q, sc, int(win), int(xd), int(xof), int(nd), int(nof))
    xo = x if xo is None else xo.view(x.shape)
    return xo, (None if n is None else n.view(x.shape)), ((q, sc) if want_q else None)


def silu_mul_quantize(gu):
    """[T, 2m] fused gate|up projection -> e4m3 codes and scales of bf16(silu(gate) * up)."""
    t, m2 = gu.shape
    m = m2 // 2
    q = torch.empty(t, m, device=gu.device, dtype=torch.uint8)
    s = torch.empty(t, m // 128, device=gu.device, dtype=torch.float32)
    _c().silu_mul_quant(gu, q, s)
    return q, s


def gated_norm_quantize(o, z, nv, z_row_stride, w, eps):
    """o [T * nv, 128] with gates z (token rows of ``z_row_stride``) -> e4m3 codes and scales."""
    rows = o.shape[0]
    q = torch.empty(rows, 128, device=o.device, dtype=torch.uint8)
    s = torch.empty(rows, 1, device=o.device, dtype=torch.float32)
    _c().gated_norm_quant(o, z, int(nv), int(z_row_stride), w, float(eps), q, s)
    return q, s


def causal_conv_silu_rows(x, ld, w, channels):
    """Causal depthwise conv + SiLU over the first ``channels`` of token rows of stride ``ld``."""
    b, s = x.shape[0], x.shape[1]
    y = torch.empty(b, s, channels, device=x.device, dtype=x.dtype)
    _c().conv_silu_vec(x, int(ld), w.reshape(w.shape[0], -1).contiguous(), y)
    return y


def gated_delta_rule_backward(q, k, v, g, beta, dout, groups=1):
    """Gradients (dq, dk, dv, dg, dbeta) of the gated delta rule w.r.t. its raw inputs.

    Not needed to train the draft (the verifier is frozen); provided as an op with a
    hand-written backward for completeness and benchmarking.
    """
    if q.is_cuda:
        return tuple(_c().gdn_chunk_bwd(q.contiguous(), k.contiguous(), v.contiguous(), g.float().contiguous(),
                                        beta.contiguous(), dout.contiguous(), int(groups)))
    if groups > 1:
        qr, kr = q.repeat_interleave(groups, 2), k.repeat_interleave(groups, 2)
    else:
        qr, kr = q, k
    dq, dk, dv, dg, db = ref.gated_delta_rule_backward(qr, kr, v, g, beta, dout)
    if groups > 1:
        b, s, nv, d = dq.shape
        dq = dq.view(b, s, nv // groups, groups, d).sum(3)
        dk = dk.view(b, s, nv // groups, groups, d).sum(3)
    return dq, dk, dv, dg, db
