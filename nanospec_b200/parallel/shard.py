"""Explicit FULL_SHARD units and the schedules that gather and reduce them.

A ``Shard`` is one unit's flat storage (reference layout: nanospec/shard.py:45-84):
``param`` (compute dtype), ``master``/``m``/``v`` (fp32) and ``grad`` (compute
dtype), each ``ss = ceil(numel/N)`` elements, rank r owning ``[r*ss, (r+1)*ss)``.
While a unit is *gathered*, its registered parameters' ``.data`` are views into a
full-size flat buffer; while its gradients are *bound*, ``.grad`` are views into a
full-size gradient buffer.

Schedules decide how a unit's full weights appear and how its gradients leave:

* ``SerialSchedule``: NCCL all-gather when acquired, reduce-scatter(AVG) after
  backward, all on the compute stream (reference: nanospec/shard.py:153-175).
* ``OverlapSchedule``: one side stream and two reusable slots. Unit i+1 is
  all-gathered while unit i computes; unit i's reduce-scatter runs while unit
  i-1 computes. CUDA events order slot reuse (reference semantics:
  nanospec/shard.py:178-303). Results are bitwise equal to the serial schedule.
* ``ResidentSchedule``: gathers each unit once per forward into a persistent
  buffer and keeps it for the backward (no second all-gather); 180 GB of HBM per
  B200 holds the whole gathered draft (3.5 GB for the 1.75 B-parameter model).
* the fused peer-memory schedule lives in ``parallel/fused.py``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from ..utils import debug as _debug


class ScheduleError(RuntimeError):
    """Raised when a schedule's state machine is driven out of order."""


class Shard:
    @torch.no_grad()
    def __init__(self, entries, *, device, dtype, shapes=None, group=None, world_size=1, rank=0):
        """``entries``: ``(name, Parameter, initial tensor)`` in flat-layout order.

        ``shapes`` maps names to their logical shapes (default: the initial tensors').
        """
        if world_size not in (1, 2, 4, 8):
            raise ValueError("Training supports 1, 2, 4 or 8 ranks")
        self.group, self.world_size, self.rank = group, world_size, rank
        self.names = [e[0] for e in entries]
        self.parameters = tuple(e[1] for e in entries)
        if any(p.requires_grad for p in self.parameters):
            raise ValueError("Manual sharding requires requires_grad=False parameters")
        self.shapes = {e[0]: tuple((shapes or {}).get(e[0], e[2].shape)) for e in entries}
        self.offsets = {}
        n = 0
        for name in self.names:
            size = math.prod(self.shapes[name])
            self.offsets[name] = (n, n + size)
            n += size
        self.numel = n
        self.shard_size = math.ceil(n / world_size)
        self.full_size = self.shard_size * world_size
        self.param = torch.zeros(self.shard_size, device=device, dtype=dtype)
        self.load_tensors({e[0]: e[2] for e in entries}, reset_master=False)
        self.master = self.param.float()
        self.grad = torch.zeros_like(self.param)
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)
        self.gathered = None
        self.full_grad = None
        self.grad_zero = True  # grad holds no accumulated values (set by zero_grad)
        self.direct_grad = False  # gradients bound straight onto ``grad`` (one rank)
        self.empty = torch.empty(0, device=device, dtype=dtype)
        if world_size == 1:
            self.bind(self.param)
        else:
            self.release()

    # ----------------------------------------------------------------- layout
    def local_range(self):
        start = self.rank * self.shard_size
        return start, start + self.shard_size

    @torch.no_grad()
    def load_tensors(self, tensors: dict, reset_master=True):
        """Copy this rank's slice of each named full tensor into ``param``."""
        start, end = self.local_range()
        for name, value in tensors.items():
            lo, hi = self.offsets[name]
            a, b = max(start, lo), min(end, hi)
            if a < b:
                flat = value.reshape(-1)
                self.param[a - start:b - start].copy_(flat[a - lo:b - lo])
        if reset_master:
            self.master.copy_(self.param)

    def views(self, flat) -> dict:
        return {n: flat[lo:hi].view(self.shapes[n]) for n, (lo, hi) in self.offsets.items()}

    def bind(self, flat):
        for name, p in zip(self.names, self.parameters):
            lo, hi = self.offsets[name]
            p.data = flat[lo:hi].view(self.shapes[name])

    def bind_gradients(self, flat):
        for name, p in zip(self.names, self.parameters):
            lo, hi = self.offsets[name]
            p.grad = flat[lo:hi].view(self.shapes[name])

    @torch.no_grad()
    def apply_placement(self, fn):
        """Follow ``Module.to()``; optimizer state stays fp32 on the param's device."""
        if self.gathered is not None or self.full_grad is not None:
            raise ScheduleError("Release gathered buffers before moving a sharded module")
        self.param, self.grad, self.empty = fn(self.param), fn(self.grad), fn(self.empty)
        for name in ("master", "m", "v"):
            setattr(self, name, getattr(self, name).to(device=self.param.device))
        if self.world_size == 1:
            self.bind(self.param)
        else:
            self.release()

    # ----------------------------------------------------------------- serial ops
    @torch.no_grad()
    def gather(self, out=None) -> dict:
        """All-gather the full flat weights (collective when sharded) and bind views."""
        if self.gathered is not None:
            raise ScheduleError("Gathered weights must be released before another gather")
        if self.world_size == 1:
            full = self.param
        else:
            full = out if out is not None else torch.empty(
                self.full_size, device=self.param.device, dtype=self.param.dtype)
            dist.all_gather_into_tensor(full, self.param, group=self.group)
        self.gathered = full
        self.bind(full)
        return dict(zip(self.names, self.parameters))

    def release(self):
        for p in self.parameters:
            p.grad = None
            if self.world_size > 1:
                p.data = self.empty
        self.gathered = None

    def gradient_buffers(self, buffer=None):
        if self.gathered is None:
            raise ScheduleError("Gather weights before binding gradient buffers")
        if buffer is None:
            buffer = torch.empty(self.full_size, device=self.param.device, dtype=self.param.dtype)
        buffer.zero_()
        self.full_grad = buffer
        self.bind_gradients(buffer)
        return buffer

    @torch.no_grad()
    def reduce(self):
        """Reduce-scatter(AVG) the full gradient into this rank's ``grad`` shard."""
        if self.full_grad is None:
            raise ScheduleError("No gradient buffer bound")
        if self.world_size == 1:
            self.grad.add_(self.full_grad)
        else:
            out = torch.empty_like(self.param)
            dist.reduce_scatter_tensor(out, self.full_grad, op=dist.ReduceOp.AVG, group=self.group)
            self.grad.add_(out)
        self.full_grad = None
        self.release()


@dataclass
class ShardingPlan:
    context: Shard
    layers: tuple
    heads: Shard
    _cache: dict = field(default_factory=dict, init=False, repr=False)

    def named_shards(self):
        yield "context", self.context
        for i, s in enumerate(self.layers):
            yield f"layers.{i}", s
        yield "heads", self.heads

    def __iter__(self):
        for _, s in self.named_shards():
            yield s

    def step_sequence(self):
        """Unit visits of one training step: forward units, the head, reverse units.

        The head is visited once (its forward and backward run back to back), so a
        step gathers the heads unit once instead of twice.
        """
        return (self.context, *self.layers, self.heads, *self.layers[::-1], self.context)

    def enable_peer(self, group=None, timeout_s=None):
        """Switch this plan to peer-memory communication (``parallel.fused``).

        Collective over the training ranks: moves every parameter shard into a
        CUDA-IPC window that all ranks can address.
        """
        from .fused import PeerSchedule, PeerWindow
        if "peer_window" in self._cache:
            return
        window = PeerWindow(self, group)
        self._cache["peer_window"] = window
        self._cache["peer"] = PeerSchedule(self, window, timeout_s)
        self._cache["peer_serial"] = PeerSchedule(self, window, timeout_s, serial=True)

    @property
    def peer_enabled(self):
        return "peer_window" in self._cache

    def schedule(self, sequence=None, *, overlap=True, resident=False):
        """A schedule over ``sequence`` (default: ``step_sequence()``).

        With ``enable_peer``: the peer-memory schedule (overlapped, or serial on the
        compute stream when ``overlap=False``). Otherwise ``overlap=False`` or one
        rank: ``SerialSchedule``; else the double-buffered ``OverlapSchedule``, or
        ``ResidentSchedule`` when ``resident`` (gathered weights kept from the
        forward for the backward).
        """
        seq = tuple(self.step_sequence() if sequence is None else sequence)
        if self.peer_enabled and self.context.world_size > 1:
            sched = self._cache["peer" if overlap else "peer_serial"]
            sched.begin(seq)
            return sched
        on_cpu = self.context.param.device.type != "cuda"  # side streams exist on CUDA only
        if self.context.world_size == 1 or on_cpu or (not overlap and not resident):
            return SerialSchedule(seq)
        key = "resident" if resident else "overlap"
        sched = self._cache.get(key)
        if sched is None:
            sched = (ResidentSchedule if resident else OverlapSchedule)(tuple(self))
            self._cache[key] = sched
        sched.begin(seq)
        return sched

    def reset_pipeline(self):
        if self.peer_enabled:
            raise ScheduleError("a model whose shards live in a peer window cannot be moved")
        for sched in self._cache.values():
            sched.close()
        self._cache.clear()

    def parameters_changed(self):
        """Call after writing parameter shards other than through the optimizer (a
        checkpoint restore, a manual copy): drops the next-step gathers that the peer
        schedule started when the optimizer last published the shards."""
        for key in ("peer", "peer_serial"):
            sched = self._cache.get(key)
            if sched is not None:
                sched.pregathered.clear()

    def close_peer(self):
        """Collective: release the peer window (after the last step)."""
        if self.peer_enabled:
            for key in ("peer", "peer_serial"):
                self._cache.pop(key).close()
            self._cache.pop("peer_window").close()


class SerialSchedule:
    """Gather on acquire and reduce on reduce, synchronously, on the compute stream."""

    def __init__(self, visits):
        self.visits = visits

    def prefetch(self, index):
        pass

    def acquire(self, index):
        self.visits[index].gather()
        return self.visits[index]

    def gradient_buffer(self, index):
        return None

    def release(self, index):
        self.visits[index].release()

    def reduce(self, index):
        self.visits[index].reduce()

    def finish(self):
        pass


class _Slot:
    def __init__(self, size, ref: Shard):
        kw = dict(device=ref.param.device, dtype=ref.param.dtype)
        self.weights = torch.empty(size, **kw)
        self.gradients = torch.empty(size, **kw)
        self.reduced = torch.empty(size // ref.world_size, **kw)
        self.ready = torch.cuda.Event()
        self.free = torch.cuda.Event()
        self.reduced_done = torch.cuda.Event()
        self.used_free = False
        self.used_reduce = False
        self.owner = None
        self.bound = False
        self.work = []


class OverlapSchedule:
    """Two slots, one communication stream, CUDA events for the buffer hazards.

    ``ready``: the all-gather into a slot finished (compute may read it).
    ``free``: compute finished reading the slot (the next gather may overwrite it).
    ``reduced_done``: the slot's gradients were reduce-scattered (may be rewritten).
    Visit k uses slot k % 2. Every rank enqueues the same collectives in order.
    """

    def __init__(self, units):
        first = units[0]
        self.device = first.param.device
        size = max(u.full_size for u in units)
        self.slots = [_Slot(size, first) for _ in range(2)]
        self.stream = torch.cuda.Stream(device=self.device)
        for slot in self.slots:
            for buf in (slot.weights, slot.gradients, slot.reduced):
                buf.record_stream(self.stream)
        for u in units:
            u.param.record_stream(self.stream)
            u.grad.record_stream(self.stream)
        self.done = torch.cuda.Event()
        self.active = False
        self.visits = ()

    def begin(self, visits):
        if self.active:
            raise ScheduleError("Finish the communication schedule before starting another")
        self.visits = visits
        self.compute = torch.cuda.current_stream(self.device)
        # The previous optimizer step wrote the local shards on the compute stream.
        self.stream.wait_stream(self.compute)
        self.active = True

    def _slot(self, index):
        return self.visits[index], self.slots[index % 2]

    def _gather_into(self, unit, dest):
        with torch.cuda.stream(self.stream):
            work = dist.all_gather_into_tensor(dest, unit.param, group=unit.group, async_op=True)
            work.wait()
        return work

    def prefetch(self, index):
        if index >= len(self.visits):
            return
        unit, slot = self._slot(index)
        if slot.bound or slot.owner is not None:
            raise ScheduleError("Release a slot before reusing it")
        slot.owner = index
        slot.work.clear()
        if slot.used_free:
            self.stream.wait_event(slot.free)
        slot.work.append(self._gather_into(unit, slot.weights[:unit.full_size]))
        slot.ready.record(self.stream)

    def acquire(self, index):
        unit, slot = self._slot(index)
        if slot.owner != index or slot.bound or unit.gathered is not None:
            raise ScheduleError("Acquire exactly one prefetched unit")
        self.compute.wait_event(slot.ready)
        slot.weights.record_stream(self.compute)
        unit.gathered = slot.weights[:unit.full_size]
        unit.bind(unit.gathered)
        slot.bound = True
        return unit

    def gradient_buffer(self, index):
        unit, slot = self._slot(index)
        if slot.owner != index or not slot.bound:
            raise ScheduleError("Acquire weights before requesting their gradient buffer")
        if slot.used_reduce:
            self.compute.wait_event(slot.reduced_done)
        slot.gradients.record_stream(self.compute)
        return slot.gradients[:unit.full_size]

    def release(self, index):
        unit, slot = self._slot(index)
        if slot.owner != index or not slot.bound:
            raise ScheduleError("Release exactly one acquired unit")
        if _debug.enabled():  # compute is done with the slot: stale reads become NaN
            _debug.poison(slot.weights)
        slot.free.record(self.compute)
        slot.used_free = True
        unit.release()
        slot.owner, slot.bound = None, False

    def reduce(self, index):
        unit, slot = self._slot(index)
        grads = unit.full_grad
        if grads is None:
            raise ScheduleError("No gradient buffer bound")
        self.release(index)
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(slot.free)
            out = slot.reduced[:unit.shard_size]
            work = dist.reduce_scatter_tensor(out, grads, op=dist.ReduceOp.AVG,
                                              group=unit.group, async_op=True)
            work.wait()
            slot.work.append(work)
            unit.grad.add_(out)
            slot.reduced_done.record(self.stream)
            slot.used_reduce = True
        unit.full_grad = None

    def finish(self):
        if any(s.bound or s.owner is not None for s in self.slots):
            raise ScheduleError("All scheduled units must be consumed before finishing")
        self.stream.wait_stream(self.compute)
        self.done.record(self.stream)
        self.compute.wait_event(self.done)
        self.active = False

    def close(self):
        if self.active:
            raise ScheduleError("Cannot close an active communication schedule")
        self.stream.synchronize()


class ResidentSchedule(OverlapSchedule):
    """Overlap schedule whose gathers land in persistent per-unit buffers.

    The first visit of a unit in a step all-gathers it (on the side stream, one
    visit ahead); later visits in the same step re-bind that buffer, so the
    backward pass needs no second all-gather of the model. Gradients use the two
    alternating slots and the side-stream reduce-scatter exactly as
    ``OverlapSchedule`` does, so results are bitwise equal to the serial schedule.
    """

    def __init__(self, units):
        super().__init__(units)
        for slot in self.slots:
            slot.weights = torch.empty(0, device=self.device, dtype=units[0].param.dtype)
        self.resident = {id(u): torch.empty(u.full_size, device=self.device, dtype=u.param.dtype)
                         for u in units}
        for buf in self.resident.values():
            buf.record_stream(self.stream)
        self.ready_events = {id(u): torch.cuda.Event() for u in units}
        self.gathered = set()

    def begin(self, visits):
        super().begin(visits)
        self.gathered = set()

    def prefetch(self, index):
        if index >= len(self.visits):
            return
        unit, slot = self._slot(index)
        if slot.bound or slot.owner is not None:
            raise ScheduleError("Release a slot before reusing it")
        slot.owner = index
        slot.work.clear()
        key = id(unit)
        if key in self.gathered:
            return
        self.gathered.add(key)
        slot.work.append(self._gather_into(unit, self.resident[key]))
        self.ready_events[key].record(self.stream)

    def acquire(self, index):
        unit, slot = self._slot(index)
        if slot.owner != index or slot.bound or unit.gathered is not None:
            raise ScheduleError("Acquire exactly one prefetched unit")
        key = id(unit)
        self.compute.wait_event(self.ready_events[key])
        unit.gathered = self.resident[key]
        unit.bind(unit.gathered)
        slot.bound = True
        return unit
