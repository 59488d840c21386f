"""One synchronous training step: verifier -> hand-off -> draft fwd -> head -> bwd -> AdamW.

Public API (reference: nanospec/train.py:22-401):
``train(ids, drafter, objective, *, verifier=, teacher_batch=, loss_mask=,
optimizer=, anchors=, accumulation_steps=1, overlap=True, resident=None, phases=None)
-> TrainResult``.

Execution differs from the reference in layout, not in math:

* tokens are kept in a *split layout*: the ``b*S`` context rows of all batch rows
  first, then the ``b*Td`` draft rows (Td = blocks * block_size). One GEMM computes
  K and V for context and draft tokens together with the shared weights;
* adjacent weights are used as one matrix: ``[k_proj; v_proj]`` (one K/V GEMM),
  ``[gate_proj; up_proj]`` (one gate/up GEMM, SwiGLU reads both halves);
* residual adds ride in GEMM epilogues; RoPE is fused with the per-head RMSNorm;
* the head (LM head + Markov head + CE/KL) runs forward and backward back to back
  (``objective.head_loss``), so the heads unit is visited once per step;
* the context-projection input gradient is only formed when ``fc_norm`` needs it;
* with one rank and gradients written in place, the weight-gradient GEMMs also
  produce the optimizer's gradient norm (``parallel.optim.FusedGradNorm``);
* ``phases=`` marks device-timed phase boundaries (``utils.phases``).
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import torch

from . import ops
from .config import Objective
from .data import prepare
from .objective import LossMetrics, head_loss
from .parallel.node import TeacherBatch
from .utils import debug as _debug


@dataclass
class TrainResult:
    teacher: TeacherBatch | None = None
    metrics: LossMetrics | None = None
    hidden: torch.Tensor | None = None
    update: dict | None = None


def _cat_rows(a, b):
    return torch.cat((a.reshape(-1, a.shape[-1]), b.reshape(-1, b.shape[-1])), 0)


class _Grads:
    """Gradient views of one unit, bound for the duration of its backward."""

    def __init__(self, unit, buffer, sched=None, index=None):
        self.unit = unit
        self.flat = buffer
        self.views = unit.views(buffer)
        self.sched = sched
        self.index = index

    def wgrad(self, dy, x, first, last=None, norm=None):
        """``dW = dy^T x`` for parameter ``first`` (or the adjacent span ``first ..
        last``). A schedule that reduce-scatters by pushes takes it into its fused
        weight-gradient GEMM (the epilogue stores into the owners' slots); otherwise
        the GEMM writes the gradient view."""
        out = self.span(first, last) if last is not None else self.views[first]
        push = getattr(self.sched, "push_wgrad", None)
        if norm is None and push is not None and push(self.index, dy, x, self.unit.offsets[first][0], out.shape):
            return
        ops.linear_wgrad(dy, x, out, norm=norm)

    def __getitem__(self, name):
        return self.views[name]

    def span(self, first, last):
        lo = self.unit.offsets[first][0]
        hi = self.unit.offsets[last][1]
        cols = self.unit.shapes[first][-1]
        return self.flat[lo:hi].view(-1, cols)


def _span(unit, first, last):
    """2-D view over the adjacent gathered weights ``first .. last`` (same column count)."""
    lo = unit.offsets[first][0]
    hi = unit.offsets[last][1]
    cols = unit.shapes[first][-1]
    return unit.gathered[lo:hi].view(-1, cols)


def _bind_grads(sched, index, unit):
    buf = sched.gradient_buffer(index)
    if buf is None:
        if unit.world_size == 1 and getattr(unit, "grad_zero", False):
            # One rank and a zero gradient shard: write gradients straight into it.
            buf = unit.grad
            unit.direct_grad = True
            if _debug.enabled():  # copy semantics: every element must be overwritten
                _debug.poison(buf[:unit.numel])
        else:
            buf = torch.empty(unit.full_size, device=unit.param.device, dtype=unit.param.dtype)
    if buf is not unit.grad:
        # Every parameter gradient is written with copy semantics; only the padding
        # tail of the flat buffer must be cleared.
        if unit.full_size > unit.numel:
            buf[unit.numel:].zero_()
    unit.full_grad = buf
    unit.bind_gradients(buf)
    return _Grads(unit, buf, sched, index)


def _reduce(sched, index, unit):
    if getattr(unit, "direct_grad", False):
        unit.direct_grad = False
        unit.grad_zero = False
        unit.full_grad = None
        sched.release(index)
        return
    unit.grad_zero = False
    sched.reduce(index)


class DraftStep:
    """Runs the draft forward, head and backward of one step for one ``DSpark``."""

    def __init__(self, model, objective: Objective):
        self.model = model
        self.o = objective

    @torch.no_grad()
    def run(self, ids, teacher: TeacherBatch, loss_mask, anchors, accumulation_steps, overlap,
            resident=None, timer=None):
        m, o = self.model, self.o
        c = m.config
        dtype = m.dtype
        b, s = ids.shape
        hq, hk, d = c.num_attention_heads, c.num_key_value_heads, c.head_dim
        qd, kd = hq * d, hk * d
        plan = m.sharding
        if resident is None:
            resident = ids.is_cuda and plan.context.world_size > 1 and overlap
        sched = plan.schedule(overlap=overlap, resident=resident)
        nl = len(plan.layers)
        visit = 0
        # One rank, one micro-step, every shard's gradient written in place: the
        # weight-gradient GEMMs can also produce the optimizer's gradient norm.
        fuse_norm = (ids.is_cuda and plan.context.world_size == 1 and accumulation_steps == 1
                     and os.environ.get("NANOSPEC_FUSED_NORM", "1") != "0"
                     and all(getattr(u, "grad_zero", False) for u in plan))
        self.norm = None

        if loss_mask is None:
            loss_mask = torch.ones(b, s, dtype=torch.float32, device=ids.device)
        feats = [h.to(dtype) for h in teacher.hidden_states]

        # ---------------------------------------------------------- context unit
        fc_saved = []
        fused_first = not m.fc_norm and hasattr(sched, "acquire_linear")
        if fused_first:
            # the projection is the unit's first consumer: a peer schedule may gather
            # the unit inside this GEMM
            context_input = torch.cat(feats, -1).reshape(b * s, -1)
            projected = sched.acquire_linear(0, context_input, "context_proj.weight")
            sched.prefetch(1)
        else:
            sched.prefetch(0)
            sched.acquire(0)
            sched.prefetch(1)
            if m.fc_norm:
                normed = []
                for norm, f in zip(m.fc_norm, feats):
                    y, inv = ops.rms_norm(f, norm.weight, norm.eps)
                    normed.append(y)
                    fc_saved.append(inv)
                context_input = torch.cat(normed, -1)
            else:
                context_input = torch.cat(feats, -1)
            context_input = context_input.reshape(b * s, -1)
            projected = ops.linear(context_input, m.context_proj.weight)
        context, inv_ctx = ops.rms_norm(projected, m.context_norm.weight, m.context_norm.eps)
        sched.release(0)

        prep = prepare(ids, loss_mask, o, anchors)
        nb, bs = prep.anchors.shape[1], o.block_size
        td = nb * bs
        noise = torch.full((b, nb, bs), c.mask_token_id, dtype=torch.long, device=ids.device)
        noise[:, :, 0] = torch.where(prep.keep, torch.gather(ids, 1, prep.anchors), c.mask_token_id)
        x = ops.embedding(noise.reshape(b * td), m.embed_tokens.weight)
        q_cos, q_sin = ops.rotary_factors(prep.positions.reshape(-1), d, c.rope_theta, dtype)
        key_pos = torch.cat((prep.context_positions.reshape(-1), prep.positions.reshape(-1)))
        k_cos, k_sin = ops.rotary_factors(key_pos, d, c.rope_theta, dtype)

        saved = []
        for li, layer in enumerate(m.layers):
            visit = 1 + li
            unit = sched.acquire(visit)
            sched.prefetch(visit + 1)
            attn, mlp = layer.self_attn, layer.mlp
            # Input norm writes the draft rows of [context ; draft] directly.
            xin = torch.empty(b * (s + td), c.hidden_size, device=x.device, dtype=dtype)
            xin[:b * s].copy_(context)
            n, inv_in = ops.rms_norm(x, layer.input_layernorm.weight, layer.input_layernorm.eps,
                                     out=xin[b * s:])
            q = ops.linear(n, attn.q_proj.weight)
            kv = ops.linear(xin, _span(unit, "self_attn.k_proj.weight", "self_attn.v_proj.weight"))
            q_rot, inv_q = ops.head_norm_rope(q.view(-1, hq, d), attn.q_norm.weight, attn.q_norm.eps,
                                              q_cos, q_sin)
            k_rot, inv_k = ops.head_norm_rope(kv[:, :kd].view(-1, hk, d), attn.k_norm.weight,
                                              attn.k_norm.eps, k_cos, k_sin)
            v = kv[:, kd:].view(-1, hk, d)
            a_out, lse = ops.attention(q_rot.view(b, td, hq, d), _split_kv(k_rot, b, s, td),
                                       _split_kv(v, b, s, td), prep.anchors, prep.keep, s, bs)
            a_flat = a_out.reshape(b * td, qd)
            x1 = ops.linear(a_flat, attn.o_proj.weight, residual=x)
            n2, inv_2 = ops.rms_norm(x1, layer.post_attention_layernorm.weight,
                                     layer.post_attention_layernorm.eps)
            gu = ops.linear(n2, _span(unit, "mlp.gate_proj.weight", "mlp.up_proj.weight"))
            prod = ops.swiglu(gu)
            x_next = ops.linear(prod, mlp.down_proj.weight, residual=x1)
            saved.append(dict(x=x, inv_in=inv_in, xin=xin, q=q, inv_q=inv_q, kv=kv, inv_k=inv_k,
                              q_rot=q_rot, k_rot=k_rot, a_out=a_out, lse=lse, x1=x1, inv_2=inv_2,
                              n2=n2, gu=gu, prod=prod))
            x = x_next
            sched.release(visit)

        if timer is not None:
            timer.mark("draft_forward")
        # ---------------------------------------------------------- head (fwd + bwd)
        visit = 1 + nl
        unit = sched.acquire(visit)
        sched.prefetch(visit + 1)
        g = _bind_grads(sched, visit, unit)
        hidden, inv_f = ops.rms_norm(x, m.final_norm.weight, m.final_norm.eps)
        markov = m.markov_head
        e = None
        if markov is not None:
            e = ops.embedding(prep.previous.reshape(-1), markov.markov_w1.weight)
        kwargs = {}
        tidx = prep.teacher_indices  # [b, td]
        if teacher.logits is None:
            last = teacher.last_hidden.to(dtype)
            kwargs["target_hidden"] = torch.gather(
                last, 1, tidx.unsqueeze(-1).expand(-1, -1, last.shape[-1])).reshape(b * td, -1)
        else:
            tl = teacher.logits.to(dtype)
            kwargs["target_logits"] = torch.gather(
                tl, 1, tidx.unsqueeze(-1).expand(-1, -1, tl.shape[-1])).reshape(b * td, -1)
        metrics, dh, de = head_loss(
            hidden, m.lm_head.weight, e, markov.markov_w2.weight if markov is not None else None,
            prep, o, dw2_out=g["markov_head.markov_w2.weight"] if markov is not None else None,
            accumulation_steps=accumulation_steps, **kwargs)
        if fuse_norm:
            from .parallel.optim import FusedGradNorm, step_factor
            den = metrics.denominator.detach().clone().float().reshape(())
            self.norm = FusedGradNorm(step_factor(den, 1, accumulation_steps))
        if markov is not None:
            ops.embedding_backward(de, prep.previous.reshape(-1), g["markov_head.markov_w1.weight"])
        dx = ops.rms_norm_backward(dh, x, inv_f, m.final_norm.weight, g["final_norm.weight"])
        _reduce(sched, visit, unit)
        del dh, de, e

        if timer is not None:
            timer.mark("head")
        # ---------------------------------------------------------- layers, reversed
        dc = torch.zeros(b * s, c.hidden_size, device=x.device, dtype=dtype)
        for j, layer in enumerate(reversed(m.layers)):
            visit = 2 + nl + j
            unit = sched.acquire(visit)
            sched.prefetch(visit + 1)
            g = _bind_grads(sched, visit, unit)
            nrm = self.norm.bind(unit) if self.norm is not None else None
            sv = saved.pop()
            attn, mlp = layer.self_attn, layer.mlp
            dp = ops.linear_dgrad(dx, mlp.down_proj.weight)
            g.wgrad(dx, sv["prod"], "mlp.down_proj.weight", norm=nrm)
            dgu = ops.swiglu_backward(dp, sv["gu"])
            del dp
            dn2 = ops.linear_dgrad(dgu, _span(unit, "mlp.gate_proj.weight", "mlp.up_proj.weight"))
            g.wgrad(dgu, sv["n2"], "mlp.gate_proj.weight", "mlp.up_proj.weight", norm=nrm)
            del dgu
            dr = ops.rms_norm_backward(dn2, sv["x1"], sv["inv_2"], layer.post_attention_layernorm.weight,
                                       g["post_attention_layernorm.weight"], residual=dx)
            del dn2
            da = ops.linear_dgrad(dr, attn.o_proj.weight)
            g.wgrad(dr, sv["a_out"].reshape(b * td, qd), "self_attn.o_proj.weight", norm=nrm)
            dkv = torch.empty_like(sv["kv"])
            dk_rot = torch.empty(b * (s + td), hk, d, device=x.device, dtype=dtype)
            dq_rot, _, _ = ops.attention_backward(
                da.view(b, td, hq, d), sv["q_rot"].view(b, td, hq, d),
                _split_kv(sv["k_rot"], b, s, td), _split_kv(sv["kv"][:, kd:].view(-1, hk, d), b, s, td),
                sv["a_out"], sv["lse"], prep.anchors, prep.keep, s, bs,
                dk=_split_kv(dk_rot, b, s, td), dv=_split_kv(dkv[:, kd:].view(-1, hk, d), b, s, td))
            del da
            ops.head_norm_rope_backward(dk_rot, sv["kv"][:, :kd].view(-1, hk, d), sv["inv_k"],
                                        attn.k_norm.weight, k_cos, k_sin, g["self_attn.k_norm.weight"],
                                        out=dkv[:, :kd].view(-1, hk, d))
            dq = ops.head_norm_rope_backward(dq_rot.view(-1, hq, d), sv["q"].view(-1, hq, d), sv["inv_q"],
                                             attn.q_norm.weight, q_cos, q_sin,
                                             g["self_attn.q_norm.weight"])
            del dq_rot, dk_rot
            wkv = _span(unit, "self_attn.k_proj.weight", "self_attn.v_proj.weight")
            dxin = ops.linear_dgrad(dkv, wkv)
            g.wgrad(dkv, sv["xin"], "self_attn.k_proj.weight", "self_attn.v_proj.weight", norm=nrm)
            del dkv
            dq2 = dq.reshape(b * td, qd)
            n = sv["xin"][b * s:]
            dn = dxin[b * s:]
            ops.linear_dgrad(dq2, attn.q_proj.weight, out=dn, accumulate=True)
            g.wgrad(dq2, n, "self_attn.q_proj.weight", norm=nrm)
            del dq, dq2
            dx = ops.rms_norm_backward(dn, sv["x"], sv["inv_in"], layer.input_layernorm.weight,
                                       g["input_layernorm.weight"], residual=dr)
            dc.add_(dxin[:b * s])
            del dxin, dn, dr, sv
            _reduce(sched, visit, unit)

        # ---------------------------------------------------------- context, backward
        visit = 2 + 2 * nl
        unit = sched.acquire(visit)
        g = _bind_grads(sched, visit, unit)
        dproj = ops.rms_norm_backward(dc, projected, inv_ctx, m.context_norm.weight,
                                      g["context_norm.weight"])
        g.wgrad(dproj, context_input, "context_proj.weight",
                norm=self.norm.bind(unit) if self.norm is not None else None)
        if m.fc_norm:
            dcat = ops.linear_dgrad(dproj, m.context_proj.weight)
            width = c.target_hidden_size
            for i, (norm, f, inv) in enumerate(zip(m.fc_norm, feats, fc_saved)):
                ops.rms_norm_backward(dcat[:, i * width:(i + 1) * width], f.reshape(b * s, -1),
                                      inv.reshape(b * s, 1), norm.weight, g[f"fc_norm.{i}.weight"])
        _reduce(sched, visit, unit)
        sched.finish()
        if timer is not None:
            timer.mark("draft_backward")
        return metrics, hidden.view(b, td, -1)


def _split_kv(t, b, s, td):
    """Views a split-layout key tensor [b*s + b*td, H, D] as the op's key argument.

    The attention ops take keys in split layout directly (context rows of all
    batch rows first, then draft rows); this helper only checks the row count.
    """
    if t.shape[0] != b * (s + td):
        raise ValueError("key rows do not match the split layout")
    return t


@torch.no_grad()
def train(ids, drafter=None, objective=None, *, verifier=None, teacher_batch=None, loss_mask=None,
          optimizer=None, anchors=None, accumulation_steps=1, overlap=True, resident=None, phases=None):
    """One synchronous step. See the module docstring.

    ``verifier``: a ``parallel.node.Teacher``; every rank of the node calls
    ``train`` and the verifier's hidden states reach the training ranks.
    ``teacher_batch``: fixed teacher tensors instead of a verifier.
    ``optimizer``: an ``AdamW``; omit it to inspect raw gradients.
    ``overlap``: False selects the serial sharding schedule.
    ``resident``: keep gathered weights from forward to backward (default on CUDA, N>1).
    ``phases``: a ``utils.phases.PhaseTimer``; the step marks verifier, draft_forward,
    head, draft_backward and optimizer boundaries on it.

    On CUDA, the kernels' bounded-wait error word is snapshotted after each phase
    without a host wait (``utils.health``); a wait that timed out raises
    ``DeviceWaitTimeout`` at the end of this call (synchronous optimizer) or at the
    start of the next one. ``NANOSPEC_DEVICE_CHECK=0`` turns the check off.
    """
    if verifier is not None and teacher_batch is not None:
        raise ValueError("Supply a verifier or fixed teacher tensors, not both")
    health = _monitor(ids)
    if health is not None:
        health.check()  # a bounded wait of an earlier step that timed out raises here
    if verifier is not None:
        from .parallel.handoff import run_verifier
        teacher_batch, ids = run_verifier(ids, verifier)
        if phases is not None:
            phases.mark("verifier")
        if health is not None:
            health.snapshot("verifier")
            if _debug.enabled():
                health.check(block=True)
    if drafter is None:
        return TrainResult(teacher=teacher_batch)
    if teacher_batch is None or objective is None:
        raise ValueError("Draft training requires teacher tensors and an objective")
    step = getattr(drafter, "_draft_step", None)
    if step is None or step.o != objective:
        step = DraftStep(drafter, objective)
        drafter._draft_step = step
    metrics, hidden = step.run(ids, teacher_batch, loss_mask, anchors, accumulation_steps, overlap,
                               resident, timer=phases)
    if health is not None:
        health.snapshot("draft forward/backward")
        if _debug.enabled():
            health.check(block=True)
    update = None
    if optimizer is not None:
        from .parallel.optim import adamw_step
        update = adamw_step(optimizer, metrics.denominator, accumulation_steps, fused_norm=step.norm)
        if phases is not None:
            phases.mark("optimizer")
        if health is not None:
            health.snapshot("optimizer")
            # A synchronous optimizer has just waited for the device: the snapshots
            # taken so far are complete, so a timeout in this step raises now.
            health.check()
    return TrainResult(teacher_batch, metrics, hidden, update)


def _monitor(ids):
    if not (torch.is_tensor(ids) and ids.is_cuda) or os.environ.get("NANOSPEC_DEVICE_CHECK", "1") == "0":
        return None
    from .utils.health import monitor
    return monitor(ids.device)
