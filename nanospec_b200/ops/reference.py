"""Plain PyTorch statements of every op: the CPU path and the numerical oracle.

Casting boundaries follow the reference's ops (nanospec/ops.py:34-239 and
nanospec/objective.py:39-80): RMSNorm normalises in fp32, rounds to the compute
dtype, then multiplies by the weight in that dtype; draft attention runs in fp32;
CE runs on compute-dtype logits while KL and the softmaxes run in fp32. The CUDA
kernels are tested against these functions.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


# --------------------------------------------------------------------- linear
def linear(x, w):
    return F.linear(x, w)


def linear_dgrad(dy, w):
    return dy @ w


def linear_wgrad(dy, x):
    return dy.reshape(-1, dy.shape[-1]).t() @ x.reshape(-1, x.shape[-1])


# --------------------------------------------------------------------- RMSNorm
def rms_norm(x, w, eps):
    """Returns (y, inv) with inv = rsqrt(mean(x^2) + eps) in fp32 over the last dim."""
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    normalized = (xf * inv).to(x.dtype)
    return w * normalized, inv


def rms_norm_backward(dy, x, inv, w):
    """Returns (dx, dw). dw sums over all leading dims in fp32 then casts."""
    normalized = (x.float() * inv).to(x.dtype)
    dw = (dy * normalized).reshape(-1, dy.shape[-1]).float().sum(0).to(w.dtype)
    dz = (dy * w).float()
    xf = x.float()
    dinv = (dz * xf).sum(-1, keepdim=True)
    dvar = dinv * (-0.5 * inv.pow(3))
    dx = dz * inv + (dvar / x.shape[-1]) * (2.0 * xf)
    return dx.to(x.dtype), dw


# --------------------------------------------------------------------- RoPE
def rotary_factors(positions, dim, theta, dtype):
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, device=positions.device).float() / dim))
    ang = positions.float().unsqueeze(-1) * inv
    ang = torch.cat((ang, ang), -1)
    return ang.cos().to(dtype), ang.sin().to(dtype)


def rotate_half(x):
    a, b = x.chunk(2, dim=-1)
    return torch.cat((-b, a), dim=-1)


def rope(x, cos, sin):
    return x * cos + rotate_half(x) * sin


def rope_backward(dy, cos, sin):
    return dy * cos - rotate_half(dy * sin)


def head_norm_rope(x, w, eps, cos, sin):
    """Per-head RMSNorm then RoPE. x [T, H, D]; cos/sin [T, D]. Returns (y, inv[T,H,1])."""
    y, inv = rms_norm(x, w, eps)
    return rope(y, cos.unsqueeze(1), sin.unsqueeze(1)), inv


def head_norm_rope_backward(dy, x, inv, w, cos, sin):
    d = rope_backward(dy, cos.unsqueeze(1), sin.unsqueeze(1))
    return rms_norm_backward(d, x, inv, w)


# --------------------------------------------------------------------- activations
def silu_backward(dy, x):
    s = x.sigmoid()
    return dy * (s * (1 + x * (1 - s)))


def swiglu(gate, up):
    return F.silu(gate) * up


def swiglu_backward(dp, gate, up):
    dgate = silu_backward(dp * up, gate)
    dup = dp * F.silu(gate)
    return dgate, dup


# --------------------------------------------------------------------- draft attention
def draft_attention(q, k, v, mask):
    """q [b,Hq,Tq,D], k/v [b,Hk,Tk,D], mask [b,1,Tq,Tk] bool. fp32 math.

    Returns (out [b,Hq,Tq,D] in q.dtype, lse [b,Hq,Tq] fp32). Rows with no visible
    key produce zeros (and lse = -inf).
    """
    g = q.shape[1] // k.shape[1]
    kr = k.repeat_interleave(g, 1).float()
    vr = v.repeat_interleave(g, 1).float()
    s = (q.float() @ kr.transpose(-1, -2)) * q.shape[-1] ** -0.5
    s = s.masked_fill(~mask, float("-inf"))
    lse = torch.logsumexp(s, -1)
    valid = mask.any(-1, keepdim=True)
    p = torch.where(valid, torch.exp(s - torch.where(valid, lse.unsqueeze(-1), 0.0)), 0.0)
    out = (p @ vr).to(q.dtype)
    return out, lse


def draft_attention_backward(dout, q, k, v, out, lse, mask):
    g = q.shape[1] // k.shape[1]
    kr = k.repeat_interleave(g, 1).float()
    vr = v.repeat_interleave(g, 1).float()
    scale = q.shape[-1] ** -0.5
    s = (q.float() @ kr.transpose(-1, -2)) * scale
    valid = mask.any(-1, keepdim=True)
    p = torch.where(mask & valid, torch.exp(s - torch.where(valid, lse.unsqueeze(-1), 0.0)), 0.0)
    do = dout.float()
    dp = do @ vr.transpose(-1, -2)
    delta = (do * out.float()).sum(-1, keepdim=True)
    ds = p * (dp - delta) * scale
    dq = ds @ kr
    dk = ds.transpose(-1, -2) @ q.float()
    dv = p.transpose(-1, -2) @ do
    b, hk, t, d = k.shape
    dk = dk.view(b, hk, g, t, d).sum(2)
    dv = dv.view(b, hk, g, t, d).sum(2)
    return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype)


# --------------------------------------------------------------------- embedding
def embedding(ids, w):
    return F.embedding(ids, w)


def embedding_backward(dy, ids, num_rows):
    out = torch.zeros(num_rows, dy.shape[-1], dtype=torch.float32, device=dy.device)
    out.index_add_(0, ids.reshape(-1), dy.reshape(-1, dy.shape[-1]).float())
    return out


# --------------------------------------------------------------------- CE + KL
def ce_kl_terms(logits, target_logits, labels, weights, valid, ce_w, kl_w, accumulation_steps=1):
    """Loss terms and the logits gradient for the draft objective.

    logits/target_logits [..., V] in compute dtype; labels/weights/valid [...].
    Returns dict(ce, kl, accept_sum, accept_total) (weighted sums, un-normalised)
    and dl [..., V] in logits dtype.
    """
    lf = logits.float()
    tf = target_logits.float()
    ce_tok = F.cross_entropy(logits.reshape(-1, logits.shape[-1]), labels.reshape(-1),
                             reduction="none").view_as(weights)
    logp = lf.log_softmax(-1)
    logq = tf.log_softmax(-1)
    p = logp.exp()
    q = logq.exp()
    kl_tok = (q * (logq - logp)).sum(-1)
    ce = (ce_tok * weights).sum()
    kl = (kl_tok * weights).sum()
    rate = torch.minimum(p, q).sum(-1)
    prefix = (rate * valid).cumprod(-1)
    block_valid = valid.any(-1)
    lengths = prefix.sum(-1) + 1.0
    accept_sum = (lengths * block_valid).sum()
    accept_total = block_valid.float().sum()
    scale = weights / accumulation_steps
    ce_scale = (scale * ce_w).to(logits.dtype).unsqueeze(-1)
    dl = logits.log_softmax(-1).exp() * ce_scale
    dl.scatter_add_(-1, labels.unsqueeze(-1), -ce_scale)
    kl_grad = (p - q) * (scale * kl_w).unsqueeze(-1)
    dl = dl + kl_grad.to(logits.dtype)
    return dict(ce=ce, kl=kl, accept_sum=accept_sum, accept_total=accept_total), dl


# --------------------------------------------------------------------- AdamW
def scaled_grad(grad, factor):
    """The optimizer's view of a gradient shard: ``grad * factor`` rounded to grad's dtype, in fp32."""
    return (grad.float() * factor).to(grad.dtype).float()


def adamw_update(master, m, v, grad, factor, clip, lr, wd, b1, b2, eps, step):
    """In-place fp32 AdamW on one flat shard (reference math: nanospec/shard.py:317-351)."""
    g = scaled_grad(grad, factor) * clip
    master.mul_(1 - lr * wd)
    m.lerp_(g, 1 - b1)
    v.mul_(b2).addcmul_(g, g, value=1 - b2)
    denom = v.sqrt().div_((1 - b2 ** step) ** 0.5).add_(eps)
    master.addcdiv_(m, denom, value=-lr / (1 - b1 ** step))
