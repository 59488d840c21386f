"""Verifier pipeline partitions and the verifier -> trainer hand-off.

Reference behaviour (nanospec/distributed.py:41-63, nanospec/train.py:53-181): the
inference ranks own contiguous layer ranges; stage i receives the hidden state of
the whole [N, S] batch from stage i-1, runs its layers and sends to stage i+1; after
a device sync and barrier, each captured layer and the final normed hidden state are
*broadcast to all ranks* and the last stage also computes and broadcasts the full
[N, S, V] teacher logits. Trainer r keeps row r.

Here:

* stage-to-stage transfers stay NCCL point-to-point, but the batch is split into
  per-row microbatches so stage i+1 starts on row 0 while stage i runs row 1
  (a forward-only pipeline; rows are independent, the recurrence runs along tokens);
* every captured decoder output row r goes only to trainer r, as soon as the row
  exists (one send per row and capture instead of a broadcast of all rows to all
  ranks), and the final normed hidden state the same way;
* teacher logits are not formed: the trainer's head recomputes the target logits
  from ``last_hidden`` vocabulary-chunk by chunk, so the [N, S, V] tensor never exists;
* with a colocated topology (verifier partitions on the training GPUs), rows that a
  rank both produces and trains on are handed over without any transfer;
* hand-off messages use their own process group (its own NCCL communicator), and
  every trainer posts its receives before any verifier compute starts. Pipeline and
  hand-off messages therefore can neither be matched against each other (they have
  identical shapes) nor wait on each other.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn

from ..models.verifier import Checkpoint, QwenStage, random_verifier_weights, stage_forward, synthetic_hf_config
from .node import TeacherBatch


class Teacher(nn.Module):
    """The verifier as seen from one rank: partition table plus this rank's stage.

    With a replicated topology (``Topology.replicated``) every rank owns all layers
    and runs them on its own batch row; otherwise partitions are contiguous layer
    ranges over ``node.inference_ranks`` (reference: nanospec/distributed.py:41-63).
    """

    def __init__(self, node, path, capture, *, checkpoint=None, weights=None, config=None):
        super().__init__()
        self.node = node
        if weights is None:
            self.checkpoint = checkpoint or Checkpoint(path)
            self.config = self.checkpoint.text_config
        else:
            self.checkpoint = None
            self.config = config["text_config"]
        self.capture = tuple(capture)
        n = self.config["num_hidden_layers"]
        ranks = node.inference_ranks
        self.replicated = bool(getattr(node.topology, "replicate", False))
        if self.replicated:
            self.partitions = {r: (0, n) for r in ranks}
        else:
            self.partitions = {r: (i * n // len(ranks), (i + 1) * n // len(ranks)) for i, r in enumerate(ranks)}
        self.stage = None
        world = dist.get_world_size() if dist.is_initialized() else 1
        # Collective: every rank constructs its Teacher, so every rank creates this group.
        self.handoff_group = dist.new_group(list(range(world))) if world > 1 and not self.replicated else None
        if node.rank in ranks:
            start, end = self.partitions[node.rank]
            first = self.replicated or node.rank == ranks[0]
            last = self.replicated or node.rank == ranks[-1]
            self.stage = QwenStage(self.checkpoint, start, end, device=node.device, first=first, last=last,
                                   weights=weights, config=config)

    @classmethod
    def random(cls, node, text_config, capture, *, seed=0, embed=None, lm_head=None):
        """A verifier with random-init weights generated on this rank's device.

        Only this rank's layers are drawn (all of them when replicated). ``embed`` /
        ``lm_head`` let the verifier share the frozen target tensors with a draft.
        """
        n = text_config["num_hidden_layers"]
        ranks = node.inference_ranks
        weights = None
        if node.rank in ranks:
            if getattr(node.topology, "replicate", False):
                start, end, first, last = 0, n, True, True
            else:
                i = ranks.index(node.rank)
                start, end = i * n // len(ranks), (i + 1) * n // len(ranks)
                first, last = i == 0, i == len(ranks) - 1
            weights = random_verifier_weights(text_config, start, end, device=node.device, first=first,
                                              last=last, seed=seed + start, embed=embed, lm_head=lm_head)
        else:
            weights = {}
        return cls(node, None, capture, weights=weights, config=synthetic_hf_config(text_config, seed=seed))

    def owner(self, layer):
        if self.replicated:
            return self.node.rank
        return next(r for r, (a, b) in self.partitions.items() if a <= layer < b)


@torch.no_grad()
def run_verifier(ids, verifier: Teacher, microbatch_rows: int = 1):
    """Runs the verifier on the full [N, S] batch; returns (TeacherBatch | None, ids row).

    Every rank of the node calls this with the same ``ids``. Training rank r gets a
    ``TeacherBatch`` with row r of each capture and of the final normed hidden state
    (and no logits), plus ``ids[r:r+1]``; other ranks get ``(None, ids)``.
    """
    node, stage = verifier.node, verifier.stage
    if verifier.replicated:
        # Every rank runs the whole verifier on its own row: the hand-off is local.
        row = ids[node.rank:node.rank + 1] if ids.shape[0] > 1 else ids
        out, captured = stage_forward(stage, row, capture=verifier.capture)
        return TeacherBatch([captured[layer] for layer in verifier.capture], out, None), row
    ranks = node.inference_ranks
    b, s = ids.shape
    width = verifier.config["hidden_size"]
    dtype = torch.bfloat16
    ntrain = node.train_gpus
    caps = verifier.capture
    hg = verifier.handoff_group
    # Receive buffers of this trainer, posted before any compute so sends never block.
    recv_feats = {}
    recv_last = None
    recv_work = []
    if node.training:
        recv_feats = {layer: torch.empty(1, s, width, device=node.device, dtype=dtype) for layer in caps}
        recv_last = torch.empty(1, s, width, device=node.device, dtype=dtype)
        ops = [dist.P2POp(dist.irecv, recv_feats[layer], verifier.owner(layer), group=hg)
               for layer in caps if verifier.owner(layer) != node.rank]
        if ranks[-1] != node.rank:
            ops.append(dist.P2POp(dist.irecv, recv_last, ranks[-1], group=hg))
        if ops:
            recv_work = dist.batch_isend_irecv(ops)

    local_feats, local_last = {}, None
    if stage is not None:
        idx = ranks.index(node.rank)
        last_stage = idx == len(ranks) - 1
        rows = list(range(0, b, microbatch_rows))
        pending = []
        for r0 in rows:
            r1 = min(b, r0 + microbatch_rows)
            if stage.embed_tokens is not None:
                x = ids[r0:r1]
            else:
                x = torch.empty(r1 - r0, s, width, device=node.device, dtype=dtype)
                dist.recv(x, src=ranks[idx - 1])
            out, captured = stage_forward(stage, x, capture=caps)
            sends = []
            for layer, h in captured.items():
                for row in range(r0, r1):
                    if row >= ntrain:
                        continue
                    piece = h[row - r0:row - r0 + 1].contiguous()
                    if row == node.rank:
                        local_feats[layer] = piece
                    else:
                        sends.append(dist.P2POp(dist.isend, piece, row, group=hg))
            if last_stage:
                for row in range(r0, r1):
                    if row >= ntrain:
                        continue
                    piece = out[row - r0:row - r0 + 1].contiguous()
                    if row == node.rank:
                        local_last = piece
                    else:
                        sends.append(dist.P2POp(dist.isend, piece, row, group=hg))
            if sends:
                pending.extend(dist.batch_isend_irecv(sends))
            if not last_stage:
                pending.append(dist.isend(out.contiguous(), ranks[idx + 1]))
        for w in pending:
            w.wait()
    if node.training:
        for w in recv_work:
            w.wait()
        feats = [local_feats.get(layer, recv_feats[layer]) for layer in caps]
        last = local_last if local_last is not None else recv_last
        return TeacherBatch(feats, last, None), ids[node.rank:node.rank + 1]
    return None, ids
