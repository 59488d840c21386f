"""Hand-written forward/backward ops. No autograd anywhere.

Every op takes token-major tensors. On CUDA tensors it runs the sm_100a kernels of
``nanospec_b200._C`` (and raises if the extension is missing); on CPU tensors it
runs the plain PyTorch statement in ``ops.reference`` (the CPU path used by the
gloo multi-rank tests and the oracle for the kernels).

Reference ops these replace: nanospec/ops.py:34-239, nanospec/objective.py:39-80,
nanospec/shard.py:317-351.
"""

from __future__ import annotations

import torch

from . import reference as ref
from ._ext import cuda_ops


def _c():
    return cuda_ops()


# ------------------------------------------------------------------------- GEMM
def linear(x, w, out=None, residual=None):
    """``x @ w.T`` (+ ``residual``), output in x.dtype. x [..., K], w [N, K]."""
    if x.is_cuda:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        if out is None:
            out = torch.empty(x2.shape[0], w.shape[0], device=x.device, dtype=x.dtype)
        res = None if residual is None else residual.reshape(-1, w.shape[0])
        _c().linear(x2, w, out.view(-1, w.shape[0]), res)
        return out.view(*lead, w.shape[0])
    y = ref.linear(x, w)
    if residual is not None:
        y = residual + y
    if out is not None:
        out.copy_(y)
        return out
    return y


def linear_dgrad(dy, w, out=None, accumulate=False):
    """``dy @ w`` (+= into ``out`` when accumulate). dy [..., N], w [N, K]."""
    if dy.is_cuda:
        lead = dy.shape[:-1]
        d2 = dy.reshape(-1, dy.shape[-1])
        if out is None:
            out = torch.empty(d2.shape[0], w.shape[1], device=dy.device, dtype=dy.dtype)
        _c().linear_dgrad(d2, w, out.view(-1, w.shape[1]), accumulate)
        return out.view(*lead, w.shape[1])
    dx = ref.linear_dgrad(dy, w)
    if out is not None:
        if accumulate:
            out.add_(dx)
        else:
            out.copy_(dx)
        return out
    return dx


def linear_wgrad(dy, x, out, accumulate=False, norm=None):
    """``out (+)= dy^T @ x`` over all leading dims. out [N, K] in compute dtype.

    ``norm``: a ``parallel.optim.FusedGradNorm`` bound to the shard that owns ``out``
    (``FusedGradNorm.bind(shard)``); the GEMM then also writes its part of the
    squared gradient norm while it stores ``out`` (CUDA, plain overwrite only).
    """
    if dy.is_cuda:
        dy2, x2 = dy.reshape(-1, dy.shape[-1]), x.reshape(-1, x.shape[-1])
        if norm is not None and not accumulate:
            norm.launch(lambda f, part, off: _c().linear_wgrad(dy2, x2, out, False, f, part, off), out)
        else:
            _c().linear_wgrad(dy2, x2, out, accumulate)
        return out
    dw = ref.linear_wgrad(dy, x)
    if accumulate:
        out.add_(dw)
    else:
        out.copy_(dw)
    return out


# ------------------------------------------------------------------------- norms
def rms_norm(x, w, eps, out=None):
    """Returns ``(w * bf16(x * inv), inv)``; inv is fp32 ``[..., 1]``."""
    if x.is_cuda:
        x2 = x.reshape(-1, x.shape[-1])
        y = out if out is not None else torch.empty_like(x)
        inv = torch.empty(x2.shape[0], 1, device=x.device, dtype=torch.float32)
        _c().rms_norm_fwd(x2, w, float(eps), y.view(-1, x.shape[-1]), inv)
        return y, inv.view(*x.shape[:-1], 1)
    y, inv = ref.rms_norm(x, w, eps)
    if out is not None:
        out.copy_(y)
        y = out
    return y, inv


def rms_norm_backward(dy, x, inv, w, dw_out, residual=None, out=None):
    """dx of RMSNorm (+ ``residual`` gradient); writes the weight gradient into ``dw_out``."""
    if dy.is_cuda:
        n = x.shape[-1]
        dx = out if out is not None else torch.empty_like(x)
        res = None if residual is None else residual.reshape(-1, n)
        _c().rms_norm_bwd(dy.reshape(-1, n), x.reshape(-1, n), inv.reshape(-1), w,
                          dx.view(-1, n), dw_out, res)
        return dx
    dx, dw = ref.rms_norm_backward(dy, x, inv, w)
    dw_out.copy_(dw)
    if residual is not None:
        dx = residual + dx
    if out is not None:
        out.copy_(dx)
        dx = out
    return dx


def head_norm_rope(x, w, eps, cos, sin, out=None):
    """Per-head RMSNorm then RoPE. x [T, H, D] (row stride may exceed H*D); cos/sin [T, D]."""
    if x.is_cuda:
        t, h, d = x.shape
        y = out if out is not None else torch.empty(t, h, d, device=x.device, dtype=x.dtype)
        inv = torch.empty(t, h, 1, device=x.device, dtype=torch.float32)
        _c().head_norm_rope_fwd(x, w, float(eps), cos, sin, y, inv)
        return y, inv
    y, inv = ref.head_norm_rope(x, w, eps, cos, sin)
    if out is not None:
        out.copy_(y)
        y = out
    return y, inv


def head_norm_rope_backward(dy, x, inv, w, cos, sin, dw_out, out=None):
    if dy.is_cuda:
        dx = out if out is not None else torch.empty(x.shape, device=x.device, dtype=x.dtype)
        _c().head_norm_rope_bwd(dy, x, inv, w, cos, sin, dx, dw_out)
        return dx
    dx, dw = ref.head_norm_rope_backward(dy, x, inv, w, cos, sin)
    dw_out.copy_(dw)
    if out is not None:
        out.copy_(dx)
        dx = out
    return dx


def rotary_factors(positions, dim, theta, dtype):
    """cos/sin tables ``[..., dim]`` (fp32 angles, cast to dtype)."""
    return ref.rotary_factors(positions, dim, theta, dtype)


# ------------------------------------------------------------------------- MLP
def swiglu(gate_up, out=None):
    """``silu(gate) * up`` for gate_up = [gate | up] along the last dim."""
    m = gate_up.shape[-1] // 2
    if gate_up.is_cuda:
        y = out if out is not None else torch.empty(*gate_up.shape[:-1], m, device=gate_up.device,
                                                    dtype=gate_up.dtype)
        _c().swiglu_fwd(gate_up.reshape(-1, 2 * m), y.view(-1, m))
        return y
    g, u = gate_up[..., :m], gate_up[..., m:]
    y = torch.nn.functional.silu(g) * u
    if out is not None:
        out.copy_(y)
        y = out
    return y


def swiglu_backward(dp, gate_up, out=None):
    """Returns [dgate | dup] with the same layout as gate_up."""
    m = gate_up.shape[-1] // 2
    if dp.is_cuda:
        dgu = out if out is not None else torch.empty_like(gate_up)
        _c().swiglu_bwd(dp.reshape(-1, m), gate_up.reshape(-1, 2 * m), dgu.view(-1, 2 * m))
        return dgu
    dg, du = ref.swiglu_backward(dp, gate_up[..., :m], gate_up[..., m:])
    dgu = torch.cat((dg, du), -1)
    if out is not None:
        out.copy_(dgu)
        dgu = out
    return dgu


# ------------------------------------------------------------------------- attention
def _to_batched(k, b, s, td):
    """Split-layout keys [b*s + b*td, H, D] -> [b, s+td, H, D]."""
    return torch.cat((k[:b * s].reshape(b, s, *k.shape[1:]), k[b * s:].reshape(b, td, *k.shape[1:])), 1)


def _from_batched(kb, out, s):
    b = kb.shape[0]
    out[:b * s].copy_(kb[:, :s].reshape(-1, *kb.shape[2:]))
    out[b * s:].copy_(kb[:, s:].reshape(-1, *kb.shape[2:]))
    return out


def attention(q, k, v, anchors, keep, seq_len, block_size):
    """Draft attention with the anchor-prefix + own-block mask.

    q [b, Td, Hq, D]; k, v in *split layout* [b*S + b*Td, Hk, D]: the S context keys
    of every batch row first, then the Td draft keys of every batch row (rows may
    be strided). Query block j of row i sees context keys [0, anchors[i, j]) and
    its own block's draft keys; a block with keep False sees nothing and outputs
    zeros. Returns (out [b, Td, Hq, D], lse [b, Hq, Td] fp32; -inf on empty rows).
    """
    b, td, hq, d = q.shape
    if q.is_cuda:
        out = torch.empty(b, td, hq, d, device=q.device, dtype=q.dtype)
        lse = torch.empty(b, hq, td, device=q.device, dtype=torch.float32)
        _c().attn_fwd(q, k, v, anchors, keep, int(seq_len), int(block_size), out, lse)
        return out, lse
    from ..data import dense_mask
    mask = dense_mask(anchors, keep, seq_len, block_size)
    kb, vb = _to_batched(k, b, seq_len, td), _to_batched(v, b, seq_len, td)
    o, lse = ref.draft_attention(q.transpose(1, 2), kb.transpose(1, 2), vb.transpose(1, 2), mask)
    return o.transpose(1, 2).contiguous(), lse


def attention_backward(dout, q, k, v, out, lse, anchors, keep, seq_len, block_size,
                       dq=None, dk=None, dv=None):
    """Gradients of ``attention``; dk/dv in split layout (written into given views)."""
    b, td = q.shape[:2]
    if q.is_cuda:
        dq = dq if dq is not None else torch.empty_like(q)
        dk = dk if dk is not None else torch.empty(k.shape, device=k.device, dtype=k.dtype)
        dv = dv if dv is not None else torch.empty(v.shape, device=v.device, dtype=v.dtype)
        _c().attn_bwd(dout, q, k, v, out, lse, anchors, keep, int(seq_len), int(block_size),
                      dq, dk, dv)
        return dq, dk, dv
    from ..data import dense_mask
    mask = dense_mask(anchors, keep, seq_len, block_size)
    t = lambda x: x.transpose(1, 2)  # noqa: E731
    kb, vb = _to_batched(k, b, seq_len, td), _to_batched(v, b, seq_len, td)
    gq, gk, gv = ref.draft_attention_backward(t(dout), t(q), t(kb), t(vb), t(out), lse, mask)
    gq = t(gq).contiguous()
    if dq is not None:
        dq.copy_(gq)
        gq = dq
    dk = _from_batched(t(gk), dk if dk is not None else torch.empty(k.shape, dtype=k.dtype), seq_len)
    dv = _from_batched(t(gv), dv if dv is not None else torch.empty(v.shape, dtype=v.dtype), seq_len)
    return gq, dk, dv


# ------------------------------------------------------------------------- embedding
def embedding(ids, w, out=None):
    if w.is_cuda:
        flat = ids.reshape(-1)
        y = out if out is not None else torch.empty(flat.numel(), w.shape[1], device=w.device,
                                                    dtype=w.dtype)
        _c().embedding_fwd(flat, w, y.view(-1, w.shape[1]))
        return y.view(*ids.shape, w.shape[1])
    y = ref.embedding(ids, w)
    if out is not None:
        out.copy_(y)
        y = out
    return y


def embedding_backward(dy, ids, grad_out):
    """``grad_out[ids[i]] += dy[i]`` deterministically (fixed order, fp32 sums), copy semantics."""
    if dy.is_cuda:
        _c().embedding_bwd(dy.reshape(-1, dy.shape[-1]), ids.reshape(-1), grad_out)
        return grad_out
    grad_out.copy_(ref.embedding_backward(dy, ids, grad_out.shape[0]).to(grad_out.dtype))
    return grad_out
