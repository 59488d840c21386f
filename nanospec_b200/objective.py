"""0.1 CE + 0.9 KL(target || draft) over the frozen LM head plus the Markov head.

Math and casting follow the reference (nanospec/objective.py:39-80 and the head
section of nanospec/train.py:269-311):

* draft logits ``l = h W_lm^T + E1[prev] W2^T`` in the compute dtype;
* target logits ``t = h_teacher W_lm^T`` (or given teacher logits);
* CE on the compute-dtype logits; KL = sum_v q (log q - log p) with fp32 softmaxes;
* loss weights ``valid * exp(-slot/gamma)``; ``accept_len`` = per block
  ``1 + sum_k prod_{i<=k} (sum_v min(p, q))_i * valid_i``;
* the logits gradient keeps CE at the compute-dtype boundary and KL in fp32.

``head_loss`` runs forward AND backward of the whole head: it returns the metrics
plus ``dh`` (gradient w.r.t. the final-normed hidden), ``de`` (w.r.t. the Markov
embedding rows) and writes ``dW2``. On CUDA (``ops/head.py``) the logits never
leave the GPU: with the draft's few tokens the whole ``[2T, vocab]`` block stays in
HBM for both passes; larger token counts stream the vocabulary in chunks.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .config import Objective
from .ops import reference as ref


@dataclass
class LossMetrics:
    ce: torch.Tensor
    kl: torch.Tensor
    numerator: torch.Tensor
    denominator: torch.Tensor
    accept_len_sum: torch.Tensor
    accept_len_total: torch.Tensor

    @property
    def loss(self):
        return self.numerator / self.denominator.clamp_min(1e-6)

    @property
    def accept_len(self):
        return self.accept_len_sum / self.accept_len_total.clamp_min(1.0)


def _metrics(ce, kl, weights, accept_sum, accept_total, o: Objective) -> LossMetrics:
    den = weights.sum()
    num = o.ce * ce + o.kl * kl
    d = den.clamp_min(1e-6)
    return LossMetrics(ce / d, kl / d, num, den, accept_sum, accept_total)


@torch.no_grad()
def head_loss(hidden, lm_head, markov_e, markov_w2, prepared, o: Objective, *,
              target_hidden=None, target_logits=None, dw2_out=None, accumulation_steps=1):
    """Forward + backward of LM head, Markov head and CE+KL.

    hidden [T, H] (T = b*blocks*bs, final-normed); markov_e [T, r] or None;
    target_hidden [T, H] (teacher states aligned to the draft slots) or
    target_logits [T, V]. Returns (LossMetrics, dh [T, H], de [T, r] or None).
    """
    if (target_hidden is None) == (target_logits is None):
        raise ValueError("Give exactly one of target_hidden / target_logits")
    if hidden.is_cuda:
        from .ops.head import head_loss_cuda
        return head_loss_cuda(hidden, lm_head, markov_e, markov_w2, prepared, o,
                              target_hidden=target_hidden, target_logits=target_logits,
                              dw2_out=dw2_out, accumulation_steps=accumulation_steps)
    shape = prepared.weights.shape
    logits = ref.linear(hidden, lm_head)
    if markov_e is not None:
        logits = logits + ref.linear(markov_e, markov_w2)
    if target_logits is None:
        target_logits = ref.linear(target_hidden, lm_head)
    v = logits.shape[-1]
    terms, dl = ref.ce_kl_terms(logits.view(*shape, v), target_logits.view(*shape, v),
                                prepared.target_ids, prepared.weights, prepared.valid,
                                o.ce, o.kl, accumulation_steps)
    dl = dl.view(-1, v)
    dh = dl @ lm_head
    de = None
    if markov_e is not None:
        de = dl @ markov_w2
        dw2_out.copy_(ref.linear_wgrad(dl, markov_e))
    m = _metrics(terms["ce"], terms["kl"], prepared.weights, terms["accept_sum"],
                 terms["accept_total"], o)
    return m, dh, de
