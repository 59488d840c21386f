"""Anchor sampling and draft-batch preparation.

Behaviour follows the reference's ``sample_anchors``/``prepare``
(nanospec/dspark.py:71-144): the same random stream (one ``torch.rand(b, 1)`` on
the ids' device per call) and the same selection rule, so that both projects pick
identical anchors from identical RNG state. That parity is what lets the step-level
tests compare losses and gradients with the reference.

Unlike the reference, the dense ``[b, 1, blocks*bs, S + blocks*bs]`` boolean mask
is not built on the GPU path. The attention kernels consume the *anchor layout*
(``anchors``, ``keep``) directly: a query in block ``j`` sees context keys
``[0, anchors[j])`` plus the keys of its own block, and a block with
``keep == False`` sees nothing (its output and gradients are zero).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .config import Objective


@torch.no_grad()
def sample_anchors(ids: torch.Tensor, loss_mask: torch.Tensor, o: Objective):
    """Pick ``o.num_anchors`` anchor positions per row, strided from a random offset.

    Candidate positions ``t`` need supervision at ``t`` and ``t+1``. Candidates are
    sorted ascending; anchor ``i`` is candidate ``(offset + i*stride) mod count``
    with ``stride = clamp(count // num_anchors, 1, block_size + 1)``. Slots past
    ``count`` are dropped (``keep`` False, anchor 0).
    """
    b, s = ids.shape
    dev = ids.device
    na = o.num_anchors
    if s <= o.block_size:
        zeros = torch.zeros(b, na, dtype=torch.long, device=dev)
        return zeros, torch.zeros(b, na, dtype=torch.bool, device=dev)
    limit = min(s - o.block_size + 1, s - 1)
    sup = loss_mask > 0.5
    candidate = sup[:, :limit] & sup[:, 1 : limit + 1]
    count = candidate.sum(dim=1, keepdim=True)
    pos = torch.arange(limit, device=dev).expand(b, limit)
    # Non-candidates sort to the end (value s+1), keeping candidates ascending.
    sorted_pos = torch.sort(torch.where(candidate, pos, s + 1), dim=1).values
    stride = torch.clamp(count // na, min=1, max=o.block_size + 1)
    denom = torch.clamp(count, min=1)
    start = (torch.rand(b, 1, device=dev) * denom).long()
    slots = torch.arange(na, device=dev).unsqueeze(0)
    pick = torch.remainder(start + slots * stride, denom).clamp(max=limit - 1)
    keep = slots < count
    anchors = torch.gather(sorted_pos, 1, pick)
    return torch.where(keep, anchors, torch.zeros_like(anchors)), keep


@dataclass
class PreparedBatch:
    anchors: torch.Tensor  # [b, nb] long
    keep: torch.Tensor  # [b, nb] bool
    positions: torch.Tensor  # [b, nb*bs] draft token positions a+slot
    context_positions: torch.Tensor  # [b, s]
    target_ids: torch.Tensor  # [b, nb, bs] label token ids
    previous: torch.Tensor  # [b, nb, bs] Markov previous tokens
    weights: torch.Tensor  # [b, nb, bs] fp32 loss weights
    valid: torch.Tensor  # [b, nb, bs] bool supervision prefix
    teacher_indices: torch.Tensor  # [b, nb*bs] teacher state index per draft slot
    seq_len: int
    block_size: int

    @property
    def mask(self) -> torch.Tensor:
        """Dense boolean attention mask ``[b, 1, nb*bs, s + nb*bs]`` (CPU oracle only)."""
        return dense_mask(self.anchors, self.keep, self.seq_len, self.block_size)


def dense_mask(anchors, keep, s, bs):
    b, nb = anchors.shape
    dev = anchors.device
    q_block = torch.arange(nb * bs, device=dev) // bs  # [Td]
    kv = torch.arange(s + nb * bs, device=dev)  # [S+Td]
    ctx = (kv < s).view(1, 1, -1) & (kv.view(1, 1, -1) < anchors[:, q_block].unsqueeze(-1))
    own = (kv >= s).view(1, -1) & (q_block.view(-1, 1) == ((kv - s).clamp(min=0) // bs).view(1, -1))
    m = (ctx | own.unsqueeze(0)) & keep[:, q_block].unsqueeze(-1)
    return m.unsqueeze(1)


@torch.no_grad()
def prepare(ids: torch.Tensor, loss_mask: torch.Tensor, o: Objective, anchors=None) -> PreparedBatch:
    b, s = ids.shape
    if s < 1:
        raise ValueError("Empty input sequence")
    a, keep = sample_anchors(ids, loss_mask, o) if anchors is None else anchors
    nb, bs = a.shape[1], o.block_size
    dev = ids.device
    slot = torch.arange(bs, device=dev).view(1, 1, bs)
    label_pos = a.unsqueeze(-1) + slot + 1  # slot j predicts ids[a+j+1]
    safe = torch.where(keep.unsqueeze(-1), label_pos.clamp(max=s - 1), torch.zeros_like(label_pos))
    flat_safe = safe.reshape(b, -1)
    target_ids = torch.gather(ids, 1, flat_safe).view(b, nb, bs)
    supervised = torch.gather(loss_mask, 1, flat_safe).view(b, nb, bs) > 0.5
    ok = keep.unsqueeze(-1) & (label_pos < s) & supervised
    # A gap in supervision truncates the remainder of the block.
    valid = torch.cumprod(ok.to(torch.int32), dim=-1).bool()
    weights = valid.float()
    if o.gamma > 0:
        weights = weights * torch.exp(-slot.float() / o.gamma)
    first = torch.gather(ids, 1, a).unsqueeze(-1)
    previous = torch.cat((first, target_ids[:, :, :-1]), dim=-1)
    return PreparedBatch(
        anchors=a,
        keep=keep,
        positions=(a.unsqueeze(-1) + slot).reshape(b, -1),
        context_positions=torch.arange(s, device=dev).expand(b, s),
        target_ids=target_ids,
        previous=previous,
        weights=weights,
        valid=valid,
        teacher_indices=(flat_safe - 1).clamp(min=0),
        seq_len=s,
        block_size=bs,
    )
