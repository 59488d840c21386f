"""Process topology: one process per GPU, training ranks and verifier partitions.

Reference: nanospec/distributed.py:14-70. Differences:

* any world size of one box (1, 2, 4, 8) with a ``Topology`` split; the reference
  requires exactly 8 ranks;
* a CPU/gloo mode (``backend="gloo"``) so the host-side logic runs in tests;
* process groups get a finite timeout (default 10 minutes, ``NANOSPEC_PG_TIMEOUT``).
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from datetime import timedelta

import torch
import torch.distributed as dist

from ..config import Topology


@dataclass
class TeacherBatch:
    """Teacher tensors handed to one training rank.

    ``hidden_states``: captured decoder outputs ``[b, S, H]`` (one per capture layer);
    ``last_hidden``: final-normed hidden ``[b, S, H]``; ``logits``: optional ``[b, S, V]``.
    """

    hidden_states: list
    last_hidden: torch.Tensor
    logits: torch.Tensor | None = None


class Node:
    """This process's place in the box.

    ``train_gpus`` training ranks are global ranks ``0..N-1`` and form
    ``train_group``. ``inference_ranks`` own verifier partitions (the training
    ranks themselves when the topology is colocated).
    """

    def __init__(self, train_gpus: int, *, topology: Topology | None = None, backend=None,
                 timeout_s: float | None = None):
        self.rank = int(os.environ.get("RANK", 0))
        self.world = int(os.environ.get("WORLD_SIZE", 1))
        local = int(os.environ.get("LOCAL_RANK", self.rank))
        self.topology = topology or Topology(world=self.world, train_gpus=train_gpus)
        if self.topology.world != self.world:
            raise ValueError("topology world size does not match WORLD_SIZE")
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        self.backend = backend
        if backend == "nccl":
            self.device = torch.device("cuda", local)
            torch.cuda.set_device(self.device)
        else:
            self.device = torch.device("cpu")
        if timeout_s is None:
            timeout_s = float(os.environ.get("NANOSPEC_PG_TIMEOUT", 600))
        if not dist.is_initialized() and self.world > 1:
            kw = dict(timeout=timedelta(seconds=timeout_s))
            if backend == "nccl":
                kw["device_id"] = self.device
            dist.init_process_group(backend, **kw)
        self.train_gpus = self.topology.train_gpus
        ranks = list(range(self.train_gpus))
        self.train_group = dist.new_group(ranks, backend=backend) if self.world > 1 else None
        if self.train_gpus == self.world:
            self.train_group = dist.group.WORLD if self.world > 1 else None
        self.training = self.rank < self.train_gpus
        self.inference_ranks = list(self.topology.inference_ranks)

    def broadcast(self, value, shape, src, dtype=torch.bfloat16):
        """Broadcast a tensor of declared shape/dtype from ``src`` over the world group."""
        if self.rank == src:
            tensor = value.contiguous()
            if tuple(tensor.shape) != tuple(shape) or tensor.dtype != dtype:
                raise ValueError("Communication buffer does not match declared shape/dtype")
        else:
            tensor = torch.empty(shape, dtype=dtype, device=self.device)
        if self.world > 1:
            dist.broadcast(tensor, src)
        return tensor

    def close(self):
        if dist.is_initialized():
            dist.barrier()
            dist.destroy_process_group()


def local_node(device="cpu") -> "Node":
    """A single-process node without a process group (tests and 1-GPU tools)."""
    node = Node.__new__(Node)
    node.rank, node.world = 0, 1
    node.topology = Topology(world=1, train_gpus=1)
    node.backend = "none"
    node.device = torch.device(device)
    node.train_gpus = 1
    node.train_group = None
    node.training = True
    node.inference_ranks = [0]
    return node
