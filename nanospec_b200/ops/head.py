"""CUDA path of the fused head: LM head + Markov head + CE/KL, vocabulary streamed.

The default kernels (``head_tc_kernel`` in csrc/head.cu) never write the logits:
each 128-token x 128-vocabulary tile of the draft, Markov and target logits lives
in TMEM, and the epilogue folds it into per-token online statistics (pass 1:
log-sum-exps, the target-weighted gap, the label logit) or into the bf16 logits
gradient of one vocabulary chunk (pass 2, followed by the dh / de / dW2 GEMMs on
that chunk). They run whenever the logits would exceed 4 GiB; below that (the draft's few
hundred tokens) the form that holds the ``[2T, V]`` logits in HBM is faster and is used
(``NANOSPEC_HEAD=streamed | materialize`` overrides the choice). Both return per-token statistics (CE, KL,
sum_v min(p, q), the two log-sum-exps) and the gradients ``dh``/``de``/``dW2``;
the weighted sums and the acceptance-length metric are formed here from those
per-token values. Reference: nanospec/objective.py:39-80, nanospec/train.py:269-311.
"""

from __future__ import annotations

import os

import torch

from ._ext import cuda_ops

# Vocabulary columns per chunk; 0 = automatic. Streamed path: the whole vocabulary
# while the [T, V] bf16 gradient fits in 1 GiB, else 512 MB gradient chunks.
# Materialised path: the whole vocabulary while [R + T, V] bf16 fits in 4 GiB.
VOCAB_CHUNK = int(os.environ.get("NANOSPEC_VOCAB_CHUNK", 0))


def head_loss_cuda(hidden, lm_head, markov_e, markov_w2, prepared, o, *, target_hidden=None,
                   target_logits=None, dw2_out=None, accumulation_steps=1):
    from ..objective import _metrics

    shape = prepared.weights.shape  # [b, nb, bs]
    t = hidden.shape[0]
    if target_logits is None:
        hcat = torch.cat((hidden, target_hidden), 0)
    else:
        hcat = hidden.contiguous()
        target_logits = target_logits.contiguous()
    weights = prepared.weights.reshape(-1).contiguous().float()
    labels = prepared.target_ids.reshape(-1).contiguous()
    row, dh, de = cuda_ops().head_loss(
        hcat, t, lm_head, markov_e, markov_w2, target_logits, labels, weights, float(o.ce),
        float(o.kl), 1.0 / accumulation_steps, dw2_out, VOCAB_CHUNK)
    ce_tok = row[:, 0].view(shape)
    kl_tok = row[:, 1].view(shape)
    rate = row[:, 2].view(shape)
    ce = (ce_tok * prepared.weights).sum()
    kl = (kl_tok * prepared.weights).sum()
    valid = prepared.valid
    prefix = (rate * valid).cumprod(-1)
    block_valid = valid.any(-1)
    accept_sum = ((prefix.sum(-1) + 1.0) * block_valid).sum()
    accept_total = block_valid.float().sum()
    return _metrics(ce, kl, prepared.weights, accept_sum, accept_total, o), dh, de
