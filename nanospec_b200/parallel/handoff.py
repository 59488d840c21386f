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
* on CUDA the hand-off is by peer stores (``HandoffWindow``): every training rank
  exposes receive slots (one per capture layer and one for the final hidden state)
  in a CUDA-IPC window, the verifier rank that produces trainer r's row stores it
  straight into r's slot over NVLink and raises a per-slot flag, and trainer r
  waits on those flags (bounded) and trains on the slots in place. Trainer r
  releases its slots at the start of the next step (a flag the producers wait on
  before storing again). ``NANOSPEC_HANDOFF=nccl`` keeps the point-to-point sends;
* NCCL hand-off messages use their own process group (its own NCCL communicator),
  and every trainer posts its receives before any verifier compute starts. Pipeline
  and hand-off messages therefore can neither be matched against each other (they
  have identical shapes) nor wait on each other.
"""

from __future__ import annotations

import os

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


class HandoffWindow:
    """Receive slots of every training rank in peer memory, and the flags around them.

    Collective over the node (all ranks create it together). Slot i of trainer r
    holds row r of capture i (i < len(capture)) or of the final normed hidden state
    (i = len(capture)), [s, width] bf16, in two sets used by alternate steps. Flags
    (``[channel][source rank]`` words in the receiver's window): channel DATA + i, set
    by the producer of slot i with the step's sequence number; channel FREE, set by a
    trainer on each producer when a step's slot set is no longer read. A producer
    writes step t's set after FREE reached t - 2, which the trainer raised at the
    start of step t - 1, so the wait never holds the verifier back in steady state.
    """

    FLAGS = 4096
    DATA, FREE = 16, 64

    def __init__(self, group, training, nslots, s, width):
        from ..ops._ext import cuda_ops
        self.C = cuda_ops()
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.s, self.width, self.nslots = s, width, nslots
        self.slot_bytes = (s * width * 2 + 255) // 256 * 256
        size = self.FLAGS + (2 * nslots * self.slot_bytes if training else 0)
        self.id, _ = self.C.window_create(size, self.rank, self.world)
        handles = [None] * self.world
        dist.all_gather_object(handles, self.C.window_ipc_handle(self.id).tolist(), group=group)
        self.C.window_open(self.id, torch.tensor(handles, dtype=torch.uint8))
        self.seq = 0
        t = float(os.environ.get("NANOSPEC_PEER_TIMEOUT_S", 60))
        self.poll_limit = int(t / 200e-9)
        torch.cuda.synchronize()
        dist.barrier(group=group)

    def offset(self, slot, seq):
        return self.FLAGS + ((seq & 1) * self.nslots + slot) * self.slot_bytes

    def view(self, slot, seq):
        return self.C.window_view(self.id, self.offset(slot, seq), self.s * self.width,
                                  torch.bfloat16).view(1, self.s, self.width)

    def put(self, dst, slot, row, seq):
        self.C.peer_put(self.id, dst, self.offset(slot, seq), row.contiguous())

    def signal(self, dst, slot, seq):
        self.C.peer_signal_to(self.id, 0, self.DATA + slot, dst, seq)

    def close(self):
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        self.C.window_close(self.id)


def _handoff_window(verifier, s, width):
    """The Teacher's hand-off window for sequence length ``s`` (re-created collectively
    when ``s`` changes), or None when the NCCL hand-off is in use."""
    node = verifier.node
    if (verifier.handoff_group is None or node.device.type != "cuda"
            or os.environ.get("NANOSPEC_HANDOFF", "peer") == "nccl"):
        return None
    win = getattr(verifier, "_handoff_window", None)
    if win is None or win.s != s or win.width != width:
        if win is not None:
            win.close()
        win = HandoffWindow(verifier.handoff_group, node.training, len(verifier.capture) + 1, s, width)
        verifier._handoff_window = win
    return win


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
    win = _handoff_window(verifier, s, width)
    if win is not None:
        return _run_verifier_peer(ids, verifier, win, microbatch_rows)
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


def _run_verifier_peer(ids, verifier, win, microbatch_rows):
    """``run_verifier`` with the hand-off by peer stores into ``win`` (see module doc).

    With one-row microbatches on a fused CUDA stage, the add+norm kernel that
    produces a captured residual or the final normed hidden state stores trainer r's
    row into r's slot from its epilogue; rows produced elsewhere are copied by
    ``peer_put`` after the stage."""
    node, stage = verifier.node, verifier.stage
    ranks = node.inference_ranks
    b, s = ids.shape
    width = verifier.config["hidden_size"]
    ntrain = node.train_gpus
    caps = verifier.capture
    last_slot = len(caps)
    C = win.C
    win.seq += 1
    seq = win.seq

    def owner(slot):
        return verifier.owner(caps[slot]) if slot < last_slot else ranks[-1]

    # The previous step's slot set is no longer read by this trainer (its kernels are
    # ordered before this signal on the stream).
    if node.training and seq > 1:
        for p in sorted({owner(i) for i in range(last_slot + 1)} - {node.rank}):
            C.peer_signal_to(win.id, 0, win.FREE, p, seq - 1)
    local = {}
    if stage is not None:
        idx = ranks.index(node.rank)
        last_stage = idx == len(ranks) - 1
        mine = [i for i in range(last_slot + 1) if owner(i) == node.rank]
        dests = [r for r in range(min(b, ntrain)) if r != node.rank] if mine else []
        if seq > 2:
            for r in dests:  # r no longer reads the set of step seq - 2
                C.peer_wait_from(win.id, 0, win.FREE, r, seq - 2, win.poll_limit)
        pending = []
        for r0 in range(0, b, microbatch_rows):
            r1 = min(b, r0 + microbatch_rows)
            if stage.embed_tokens is not None:
                x = ids[r0:r1]
            else:
                x = torch.empty(r1 - r0, s, width, device=node.device, dtype=torch.bfloat16)
                dist.recv(x, src=ranks[idx - 1])
            targets = {}
            if r1 - r0 == 1 and r0 < ntrain and r0 != node.rank:
                for i in mine:
                    key = caps[i] if i < last_slot else "final"
                    targets[key] = (win.id, r0, win.offset(i, seq))
            stored = dict(targets)
            out, captured = stage_forward(stage, x, capture=caps, handoff=targets)
            rows_of = [(i, captured[caps[i]]) for i in range(last_slot) if caps[i] in captured]
            if last_stage:
                rows_of.append((last_slot, out))
            for i, h in rows_of:
                key = caps[i] if i < last_slot else "final"
                for row in range(r0, min(r1, ntrain)):
                    piece = h[row - r0:row - r0 + 1]
                    if row == node.rank:
                        local[i] = piece
                        continue
                    if row != r0 or key in targets or key not in stored:
                        win.put(row, i, piece, seq)  # not stored by the producing kernel
                    win.signal(row, i, seq)
            if not last_stage:
                pending.append(dist.isend(out.contiguous(), ranks[idx + 1]))
        for w in pending:
            w.wait()
    if node.training:
        got = []
        for i in range(last_slot + 1):
            if i in local:
                got.append(local[i])
            else:
                C.peer_wait_from(win.id, 0, win.DATA + i, owner(i), seq, win.poll_limit)
                got.append(win.view(i, seq))
        return TeacherBatch(got[:last_slot], got[last_slot], None), ids[node.rank:node.rank + 1]
    return None, ids
