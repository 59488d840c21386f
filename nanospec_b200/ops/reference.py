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


# --------------------------------------------------------------------- verifier ops
def qwen_norm(x, w, eps):
    """Qwen3.5 RMSNorm: weight applied as (1 + w), everything in fp32, one final cast."""
    y = x.float()
    y = y * torch.rsqrt(y.pow(2).mean(-1, keepdim=True) + eps)
    return (y * (1.0 + w.float())).to(x.dtype)


def qwen_gated_norm(x, gate, w, eps):
    """w * bf16(rmsnorm(x)) * silu(gate) (fp32 gate), cast to x.dtype."""
    xf = x.float()
    n = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)
    return (w * n * F.silu(gate.float())).to(x.dtype)


def quantize_fp8_rows(x, block=128):
    """Dynamic 1 x 128 e4m3 quantisation: returns (q [.., K] e4m3, scale [.., K/128] fp32)."""
    xb = x.float().reshape(*x.shape[:-1], -1, block)
    s = xb.abs().amax(-1, keepdim=True) / 448.0
    q = (xb / s.clamp_min(torch.finfo(torch.float32).tiny)).clamp(-448, 448).to(torch.float8_e4m3fn)
    return q.reshape(x.shape), s.squeeze(-1)


def fp8_linear(x, w, scale_inv, block=128):
    """Block-scaled FP8 projection: dequantised activations and weights, fp32 GEMM, cast.

    Non-FP8 weights run a plain linear. The dequantise-then-fp32-GEMM form is the
    numerical oracle for the tensor-core kernel.
    """
    if w.dtype != torch.float8_e4m3fn:
        return F.linear(x, w)
    n, k = w.shape
    if n % block or k % block:
        raise ValueError("FP8 weights need 128 x 128 blocks")
    q, s = quantize_fp8_rows(x, block)
    xd = (q.float().reshape(*x.shape[:-1], -1, block) * s.unsqueeze(-1)).reshape(x.shape)
    wd = (w.float().view(n // block, block, k // block, block) * scale_inv[:, None, :, None]).reshape(n, k)
    return F.linear(xd, wd).to(x.dtype)


def causal_conv_silu(x, w):
    """Depthwise causal conv1d (kernel K, left padding K-1) followed by SiLU.

    x [b, s, C] (token-major), w [C, 1, K]. Returns [b, s, C] in x.dtype.
    """
    b, s, c = x.shape
    kk = w.shape[-1]
    y = F.conv1d(x.transpose(1, 2), w, padding=kk - 1, groups=c)[..., :s]
    return F.silu(y).transpose(1, 2)


def gdn_gates(a, b, a_log, dt_bias):
    """g = -exp(A_log) * softplus(a + dt_bias) (fp32) and beta = sigmoid(b)."""
    g = -a_log.float().exp() * F.softplus(a.float() + dt_bias.float())
    return g, b.sigmoid()


def l2norm(x, eps=1e-6):
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def gated_delta_rule_recurrent(q, k, v, g, beta):
    """Token-by-token gated delta rule in fp32 (oracle).

    q, k [b, s, h, dk]; v [b, s, h, dv]; g, beta [b, s, h]. q and k are L2-normalised
    here and q is scaled by dk^-1/2. State S [dk, dv]:
    S <- exp(g) S;  S <- S + k (beta (v - S^T k))^T;  o = S^T q.
    """
    dtype = q.dtype
    q = l2norm(q.float()) * q.shape[-1] ** -0.5
    k = l2norm(k.float())
    v, g, beta = v.float(), g.float(), beta.float()
    b, s, h, dk = k.shape
    state = torch.zeros(b, h, dk, v.shape[-1], dtype=torch.float32, device=q.device)
    out = torch.empty(b, s, h, v.shape[-1], dtype=torch.float32, device=q.device)
    for t in range(s):
        state = state * g[:, t].exp()[..., None, None]
        kv = torch.einsum("bhkv,bhk->bhv", state, k[:, t])
        delta = (v[:, t] - kv) * beta[:, t, :, None]
        state = state + k[:, t, :, :, None] * delta[:, :, None, :]
        out[:, t] = torch.einsum("bhkv,bhk->bhv", state, q[:, t])
    return out.to(dtype)


def gated_delta_rule_chunked(q, k, v, g, beta, chunk=64):
    """Chunked (WY-form) gated delta rule; same math as the recurrence, fp32 inside.

    Per chunk with in-chunk cumulative decay G: T = (I + tril(beta k k^T e^{G_i-G_j}, -1))^-1,
    U = T (beta v), W = T (beta k e^G); then with the carried state S:
    v' = U - W S;  o = (q e^G) S + tril(q k^T e^{G_i-G_j}) v';  S = e^{G_last} S + (k e^{G_last-G})^T v'.
    """
    dtype = q.dtype
    q = l2norm(q.float()) * q.shape[-1] ** -0.5
    k = l2norm(k.float())
    v, g, beta = v.float(), g.float(), beta.float()
    b, s, h, dk = k.shape
    dv = v.shape[-1]
    pad = (-s) % chunk
    if pad:
        z = lambda t: F.pad(t, (0, 0, 0, 0, 0, pad)) if t.dim() == 4 else F.pad(t, (0, 0, 0, pad))  # noqa: E731
        q, k, v, g, beta = z(q), z(k), z(v), z(g), z(beta)
    n = (s + pad) // chunk
    # [b, h, n, C, d]
    r = lambda t: t.view(b, n, chunk, h, -1).permute(0, 3, 1, 2, 4)  # noqa: E731
    q, k, v = r(q), r(k), r(v)
    g = g.view(b, n, chunk, h).permute(0, 3, 1, 2).cumsum(-1)
    beta = beta.view(b, n, chunk, h).permute(0, 3, 1, 2)
    eye = torch.eye(chunk, device=q.device)
    strict = torch.ones(chunk, chunk, device=q.device, dtype=torch.bool).tril(-1)
    incl = torch.ones(chunk, chunk, device=q.device, dtype=torch.bool).tril()
    decay = torch.where(incl, (g.unsqueeze(-1) - g.unsqueeze(-2)).clamp(max=0).exp(), torch.zeros((), device=q.device))
    kb = k * beta.unsqueeze(-1)
    m = torch.where(strict, (kb @ k.transpose(-1, -2)) * decay, torch.zeros((), device=q.device))
    tinv = torch.linalg.solve_triangular(eye + m, eye.expand_as(m), upper=False, unitriangular=True)
    u = tinv @ (v * beta.unsqueeze(-1))
    w = tinv @ (kb * g.exp().unsqueeze(-1))
    state = torch.zeros(b, h, dk, dv, device=q.device)
    out = torch.empty(b, h, n, chunk, dv, device=q.device)
    for i in range(n):
        gi = g[:, :, i]
        vn = u[:, :, i] - w[:, :, i] @ state
        att = torch.where(incl, (q[:, :, i] @ k[:, :, i].transpose(-1, -2)) * decay[:, :, i],
                          torch.zeros((), device=q.device))
        out[:, :, i] = (q[:, :, i] * gi.exp().unsqueeze(-1)) @ state + att @ vn
        last = gi[..., -1:]
        state = state * last.exp().unsqueeze(-1) + (k[:, :, i] * (last - gi).exp().unsqueeze(-1)).transpose(-1, -2) @ vn
    out = out.permute(0, 2, 3, 1, 4).reshape(b, n * chunk, h, dv)[:, :s]
    return out.to(dtype)


def gated_delta_rule_backward_chunked(q, k, v, g, beta, dout, chunk=64):
    """Gradients (dq, dk, dv, dg, dbeta) of the gated delta rule, chunked, explicit.

    The statements that the chunked backward kernels (csrc/gdn_bwd.cu) implement;
    fp32, no autograd. q, k [b, s, h, dk] raw (per value head), v/dout [b, s, h, dv],
    g, beta [b, s, h]. Per chunk (in-chunk cumulative decay G, gam = e^G, Gam the
    causal decay matrix, T = I + M with M = strict(beta k k^T * Gam)):
      U = T^-1 (beta v), W = T^-1 (beta gam k), A = incl(q k^T * Gam),
      Kh = e^{G_C - G} k, VN = U - W S0, O = gam q S0 + A VN, S1 = e^{G_C} S0 + Kh^T VN.
    Both carried quantities obey one linear recurrence per chunk, F = e^{G_C} I - Kh^T W:
      S1 = F S0 + Kh^T U  (forward),   dS0 = F^T dS1 + (gam q)^T dO - W^T A^T dO  (reverse);
    every other term is chunk-local:
      dVN = A^T dO + Kh dS1, dA = incl(dO VN^T), dW = -dVN S0^T, dU = dVN,
      dBv = T^-T dU, dBk = T^-T dW, dM = strict(-(dBv U^T + dBk W^T)),
    then the products' chain rules into q, k, v, beta and G, G into g by a reverse
    cumulative sum, and the L2-normalisation chain rule into the raw q and k.
    """
    qf, kf = q.float(), k.float()
    scale = q.shape[-1] ** -0.5
    rq = torch.rsqrt((qf * qf).sum(-1, keepdim=True) + 1e-6)
    rk = torch.rsqrt((kf * kf).sum(-1, keepdim=True) + 1e-6)
    qn, kn = qf * rq, kf * rk
    b, s, h, dk = k.shape
    dv = v.shape[-1]
    pad = (-s) % chunk
    n = (s + pad) // chunk

    def chunks(t):  # [b, s, h, ...] -> [b, h, n, C, ...]
        t = torch.nn.functional.pad(t, (0, 0) * (t.dim() - 3) + (0, 0, 0, pad)) if pad else t
        return t.reshape(b, n, chunk, h, *t.shape[3:]).movedim(3, 1)

    Q, K = chunks(qn * scale), chunks(kn)
    V, dO = chunks(v.float()), chunks(dout.float())
    gc, bc = chunks(g.float().unsqueeze(-1))[..., 0], chunks(beta.float().unsqueeze(-1))[..., 0]
    G = gc.cumsum(-1)
    gam = G.exp()
    incl = torch.ones(chunk, chunk, dtype=torch.bool, device=q.device).tril()
    strict = incl.tril(-1)
    zero = torch.zeros((), device=q.device)
    Gam = torch.where(incl, (G.unsqueeze(-1) - G.unsqueeze(-2)).clamp(max=0).exp(), zero)
    KK = K @ K.transpose(-1, -2)
    M = torch.where(strict, bc.unsqueeze(-1) * KK * Gam, zero)
    eye = torch.eye(chunk, device=q.device)
    Tinv = torch.linalg.solve_triangular(eye + M, eye.expand_as(M), upper=False, unitriangular=True)
    Bv, Bk = V * bc.unsqueeze(-1), K * (bc * gam).unsqueeze(-1)
    U, W = Tinv @ Bv, Tinv @ Bk
    A = torch.where(incl, (Q @ K.transpose(-1, -2)) * Gam, zero)
    GC = G[..., -1:]
    eK = (GC - G).exp()
    Kh = K * eK.unsqueeze(-1)
    gC = GC.exp().unsqueeze(-1)  # [b, h, n, 1, 1]
    F = gC * torch.eye(dk, device=q.device) - Kh.transpose(-1, -2) @ W
    # forward states entering each chunk, gradients of the states leaving each chunk
    S0 = torch.zeros(b, h, n, dk, dv, device=q.device)
    for i in range(n - 1):
        S0[:, :, i + 1] = F[:, :, i] @ S0[:, :, i] + Kh[:, :, i].transpose(-1, -2) @ U[:, :, i]
    Pc = (Q * gam.unsqueeze(-1)).transpose(-1, -2) @ dO - W.transpose(-1, -2) @ (A.transpose(-1, -2) @ dO)
    dS1 = torch.zeros(b, h, n, dk, dv, device=q.device)
    for i in range(n - 1, 0, -1):
        dS1[:, :, i - 1] = F[:, :, i].transpose(-1, -2) @ dS1[:, :, i] + Pc[:, :, i]
    # chunk-local adjoints
    VN = U - W @ S0
    dVN = A.transpose(-1, -2) @ dO + Kh @ dS1
    dA = torch.where(incl, dO @ VN.transpose(-1, -2), zero)
    dQg = dO @ S0.transpose(-1, -2)
    dKh = VN @ dS1.transpose(-1, -2)
    dW = -dVN @ S0.transpose(-1, -2)
    dBv = Tinv.transpose(-1, -2) @ dVN
    dBk = Tinv.transpose(-1, -2) @ dW
    dM = torch.where(strict, -(dBv @ U.transpose(-1, -2) + dBk @ W.transpose(-1, -2)), zero)
    dV = bc.unsqueeze(-1) * dBv
    kdk = (dBk * K).sum(-1)
    dB = (dBv * V).sum(-1) + gam * kdk
    dK = (bc * gam).unsqueeze(-1) * dBk
    dG = bc * gam * kdk
    E = dM * Gam
    dB = dB + (E * KK).sum(-1)
    dK = dK + bc.unsqueeze(-1) * (E @ K) + E.transpose(-1, -2) @ (bc.unsqueeze(-1) * K)
    MM = dM * M
    dG = dG + MM.sum(-1) - MM.sum(-2)
    Fq = dA * Gam
    dQ = Fq @ K
    dK = dK + Fq.transpose(-1, -2) @ Q
    AA = dA * A
    dG = dG + AA.sum(-1) - AA.sum(-2)
    dQ = dQ + gam.unsqueeze(-1) * dQg
    dG = dG + gam * (Q * dQg).sum(-1)
    dK = dK + eK.unsqueeze(-1) * dKh
    tk = eK * (K * dKh).sum(-1)
    dGC = tk.sum(-1) + gC[..., 0, 0] * (S0 * dS1).sum((-1, -2))
    dG = dG - tk
    dG[..., -1] = dG[..., -1] + dGC
    dg = dG.flip(-1).cumsum(-1).flip(-1)

    def unchunk(t):  # [b, h, n, C, ...] -> [b, s, h, ...]
        t = t.movedim(1, 3).reshape(b, n * chunk, h, *t.shape[4:])
        return t[:, :s]

    dqs, dkn = unchunk(dQ) * scale, unchunk(dK)
    dq = rq * (dqs - qn * (qn * dqs).sum(-1, keepdim=True))
    dk = rk * (dkn - kn * (kn * dkn).sum(-1, keepdim=True))
    return dq, dk, unchunk(dV), unchunk(dg.unsqueeze(-1))[..., 0], unchunk(dB.unsqueeze(-1))[..., 0]


def causal_attention(q, k, v):
    """Verifier attention: q [b, s, Hq, D], k/v [b, s, Hk, D]; bf16 scores + fp32 softmax."""
    g = q.shape[2] // k.shape[2]
    qt, kt, vt = q.transpose(1, 2), k.repeat_interleave(g, 2).transpose(1, 2), v.repeat_interleave(g, 2).transpose(1, 2)
    s = (qt @ kt.transpose(-1, -2)) * q.shape[-1] ** -0.5
    n = q.shape[1]
    mask = torch.ones(n, n, dtype=torch.bool, device=q.device).triu(1)
    s = s.masked_fill(mask, torch.finfo(s.dtype).min)
    p = s.softmax(-1, dtype=torch.float32).to(q.dtype)
    return (p @ vt).transpose(1, 2)


def partial_rope(x, cos, sin, rotary_dim):
    """RoPE on the first ``rotary_dim`` channels of each head. x [b, s, H, D]; cos/sin [b, s, rd]."""
    c, s_ = cos.unsqueeze(2), sin.unsqueeze(2)
    return torch.cat((rope(x[..., :rotary_dim], c, s_), x[..., rotary_dim:]), -1)


def gated_delta_rule_backward(q, k, v, g, beta, dout):
    """Gradients (dq, dk, dv, dg, dbeta) of ``gated_delta_rule_recurrent`` by autograd in fp32.

    The verifier is frozen, so training never needs this; it is the oracle of the
    backward kernel (q, k are the raw, pre-normalisation inputs).
    """
    with torch.enable_grad():
        leaves = [t.detach().float().requires_grad_(True) for t in (q, k, v, g, beta)]
        out = gated_delta_rule_recurrent(*leaves)
        out.backward(dout.float())
    return tuple(t.grad for t in leaves)
