"""One training step as a CUDA graph (single training rank, fixed shapes).

``train()`` launches a few hundred kernels per step from Python; at the benchmark
shape the GPU work per kernel is often shorter than the host's launch cost. A
``GraphedStep`` captures the complete step (draft forward, head, backward, AdamW)
once and then replays it: one launch per step, no host synchronisation inside.

Inputs are copied into static device buffers before each replay (the copy is part
of the step); outputs are device tensors owned by the graph (``TrainResult`` with
0-dim metrics and a ``{"grad_norm", "updated", "denominator"}`` dict of 0-dim
tensors). Anchors are drawn inside the graph from the CUDA generator's graph-safe
stream, so consecutive replays see fresh anchors.

Each replay snapshots the kernels' bounded-wait error word (``utils.health``); a
timeout raises ``DeviceWaitTimeout`` at the next ``step``.

Restrictions: one training rank (the peer and NCCL schedules keep host-side
sequence state and are not captured), fixed shapes, no verifier in the step.
"""

from __future__ import annotations

import torch

from .engine import TrainResult, train
from .parallel.node import TeacherBatch


class GraphedStep:
    def __init__(self, model, objective, optimizer, ids, teacher_batch: TeacherBatch, loss_mask=None,
                 warmup: int = 2, accumulation_steps: int = 1, anchors=None):
        if model.sharding.context.world_size != 1:
            raise ValueError("GraphedStep captures single-rank training only")
        if not ids.is_cuda:
            raise ValueError("GraphedStep needs CUDA tensors")
        self.model, self.objective, self.optimizer = model, objective, optimizer
        self.accumulation_steps = accumulation_steps
        optimizer.sync = False
        self.ids = ids.clone()
        self.hidden_states = [h.clone() for h in teacher_batch.hidden_states]
        self.last_hidden = teacher_batch.last_hidden.clone()
        self.logits = None if teacher_batch.logits is None else teacher_batch.logits.clone()
        self.loss_mask = (torch.ones(ids.shape, device=ids.device, dtype=torch.float32)
                          if loss_mask is None else loss_mask.clone())
        # Optional fixed anchors (anchor positions, keep flags); otherwise drawn per replay.
        self.anchors = None if anchors is None else (anchors[0].clone(), anchors[1].clone())
        self.stream = torch.cuda.Stream(device=ids.device)
        self.stream.wait_stream(torch.cuda.current_stream(ids.device))
        # Warm-up on the capture stream: every lazily created resource (per-stream
        # counters, kernel attributes, the device step counter) exists before capture.
        with torch.cuda.stream(self.stream):
            for _ in range(warmup):
                self._run()
        torch.cuda.current_stream(ids.device).wait_stream(self.stream)
        torch.cuda.synchronize(ids.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self.result = self._run()

    def _run(self) -> TrainResult:
        tb = TeacherBatch(self.hidden_states, self.last_hidden, self.logits)
        return train(self.ids, self.model, self.objective, teacher_batch=tb, loss_mask=self.loss_mask,
                     optimizer=self.optimizer, accumulation_steps=self.accumulation_steps, anchors=self.anchors)

    @torch.no_grad()
    def step(self, ids=None, hidden_states=None, last_hidden=None, loss_mask=None, logits=None) -> TrainResult:
        """Copy any given inputs into the static buffers, replay, return the (static) result."""
        if ids is not None:
            self.ids.copy_(ids, non_blocking=True)
        if hidden_states is not None:
            for dst, src in zip(self.hidden_states, hidden_states):
                dst.copy_(src, non_blocking=True)
        if last_hidden is not None:
            self.last_hidden.copy_(last_hidden, non_blocking=True)
        if loss_mask is not None:
            self.loss_mask.copy_(loss_mask, non_blocking=True)
        if logits is not None:
            self.logits.copy_(logits, non_blocking=True)
        health = self._health()
        if health is not None:
            health.check()  # an earlier replay's bounded wait that timed out raises here
        self.graph.replay()
        if health is not None:
            health.snapshot("graphed training step")
        return self.result

    def _health(self):
        import os
        if os.environ.get("NANOSPEC_DEVICE_CHECK", "1") == "0":
            return None
        from .utils.health import monitor
        return monitor(self.ids.device)
