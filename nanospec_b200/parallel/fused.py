"""Peer-memory sharding schedule: all-gather and reduce-scatter by our own kernels.

Every training rank owns one *window* (a device allocation opened by all peers
through CUDA IPC). The window holds this rank's parameter shard of every unit, two
full-size gradient slots and a flag area; peers address it at the same offsets.

* all-gather: as soon as every rank's parameters are final, the communication
  stream pulls every unit (in forward order) out of the peers' windows over NVLink
  into persistent local buffers, by copy-engine DMA (one peer-to-peer copy per
  shard, no SMs taken from compute) or by an SM kernel; compute waits per unit on
  an event. The gathered weights stay resident for the backward pass, so the model
  is gathered once per step;
* reduce-scatter of unit i: after the backward of unit i writes its full gradient
  into a window slot, each rank signals its peers, and every owner pulls its
  shard-range of every peer's slot (copy-engine DMA into a staging buffer, or an SM
  kernel), sums the N contributions in fixed rank order, averages and adds into its
  gradient shard (deterministic, NCCL AVG semantics);
* fused variants (``NANOSPEC_PEER_GATHER=fused``, ``NANOSPEC_PEER_REDUCE=push``):
  the context unit is gathered by the first GEMM that consumes it (``ag_gemm``:
  puller warps inside the GEMM fetch the unit's chunks and the tensor-core tiles
  start on each W tile as soon as its chunks are in), and every weight-gradient
  GEMM stores its bf16 output straight into the owners' window slots from its
  epilogue (``gemm_rs``); the remaining small gradients are pushed by a copy
  kernel, and each owner sums the rows of its own slot in rank order. Values are
  the same as the pull paths';
* synchronisation is by sequence-number flags in the windows (release stores /
  acquire loads) with bounded waits: a peer that never signals makes the wait
  kernel set the device error word and return, and the host raises.

The protocol per step, all ranks in the same order:
``publish`` (from the optimizer, after each shard's update): flag "unit i final"
and gather unit i for the next step on the communication stream, overlapping the
rest of the optimizer step;
``begin``: barrier "parameters of step t final" (after the previous AdamW), then
gather every unit not gathered by ``publish``;
``prefetch/acquire``: gather + event; ``gradient_buffer``: wait until every peer
has pulled this slot's previous contents; ``reduce``: signal "slot ready", wait for
all peers' "slot ready", pull-reduce, signal "slot pulled"; ``finish``: the
compute stream waits for the communication stream.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..ops._ext import cuda_ops
from ..utils import debug as _debug
from .shard import ScheduleError

FLAGS_BYTES = 4096
CH_PARAMS, CH_PULLED, CH_READY = 0, 2, 4  # channels; PULLED/READY use +slot
CH_UNIT = 8  # CH_UNIT + i: "unit i's parameters are final" (published per unit after AdamW)


def _align(n, a=256):
    return (n + a - 1) // a * a


def _weight(unit, name):
    lo, hi = unit.offsets[name]
    return unit.gathered[lo:hi].view(unit.shapes[name])


class PeerWindow:
    """This rank's symmetric window and the peers' view of it."""

    def __init__(self, plan, group=None):
        self.C = cuda_ops()
        first = plan.context
        self.rank, self.world = first.rank, first.world_size
        self.group = group if group is not None else first.group
        units = list(plan)
        off = FLAGS_BYTES
        self.param_off = {}
        for u in units:
            self.param_off[id(u)] = off
            off += _align(u.shard_size * 2)
        self.slot_bytes = _align(max(u.full_size for u in units) * 2)
        self.slot_off = [off, off + self.slot_bytes]
        total = off + 2 * self.slot_bytes
        self.id, _ = self.C.window_create(total, self.rank, self.world)
        handle = self.C.window_ipc_handle(self.id)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.tolist(), group=self.group)
        self.C.window_open(self.id, torch.tensor(handles, dtype=torch.uint8))
        # Move every parameter shard into the window (values unchanged).
        for u in units:
            view = self.C.window_view(self.id, self.param_off[id(u)], u.shard_size, u.param.dtype)
            view.copy_(u.param)
            u.param = view
        self.slots = [self.C.window_view(self.id, o, self.slot_bytes // 2, first.param.dtype)
                      for o in self.slot_off]
        # Flag sequence numbers belong to the window: every schedule using it (the
        # overlapped and the serial one) continues the same monotonic sequences.
        self.seq = {CH_PARAMS: 0, CH_PULLED: 0, CH_PULLED + 1: 0, CH_READY: 0, CH_READY + 1: 0}
        torch.cuda.synchronize()
        dist.barrier(group=self.group)

    def close(self):
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        self.C.window_close(self.id)


class PeerSchedule:
    """Resident gathered weights + window-slot gradient reduction (see module doc)."""

    def __init__(self, plan, window: PeerWindow, timeout_s: float | None = None, serial=False):
        """``serial=True`` runs every transfer on the compute stream (no overlap):
        the same kernels in the same order, used as the bitwise reference."""
        self.C = cuda_ops()
        self.w = window
        self.serial = serial
        units = tuple(plan)
        self.device = units[0].param.device
        self.stream = torch.cuda.current_stream(self.device) if serial else torch.cuda.Stream(device=self.device)
        self.resident = {id(u): torch.empty(u.full_size, device=self.device, dtype=u.param.dtype) for u in units}
        self.ready = {id(u): torch.cuda.Event() for u in units}
        self.reduced = [torch.cuda.Event(), torch.cuda.Event()]
        self.seq = window.seq
        self.slot_owner = [None, None]
        t = timeout_s if timeout_s is not None else float(os.environ.get("NANOSPEC_PEER_TIMEOUT_S", 60))
        self.poll_limit = int(t / 200e-9)
        # "ce": copy-engine all-gather (default); "sm": the SM all-gather kernel
        self.gather_engine = os.environ.get("NANOSPEC_PEER_GATHER", "ce")
        # Reduce-scatter: "ce" DMAs the peers' slot ranges into `staging` and sums
        # locally; "sm" pulls and sums in one SM kernel. Same values either way.
        self.reduce_engine = os.environ.get("NANOSPEC_PEER_REDUCE", "ce")
        # The fused paths address 8-element (16-byte) vectors of the flat unit.
        aligned = all(u.shard_size % 8 == 0 for u in units)
        if self.reduce_engine == "push" and not aligned:
            self.reduce_engine = "ce"
        if self.gather_engine == "fused" and not aligned:
            self.gather_engine = "ce"
        self.push = self.reduce_engine == "push"
        self.local_grad = None
        self.pushed = [[], []]
        if self.push:
            # small gradients (norms, embeddings) are written here, then pushed
            size = max(u.full_size for u in units)
            self.local_grad = [torch.empty(size, device=self.device, dtype=units[0].param.dtype) for _ in range(2)]
        # fused gather: the first unit (the context projection) is gathered by its GEMM
        self.fused_keys = {id(units[0])} if self.gather_engine == "fused" else set()
        if self.fused_keys:
            chunk = min(16384, units[0].shard_size)
            self.ag_flags = torch.zeros((units[0].full_size + chunk - 1) // chunk, device=self.device,
                                        dtype=torch.int32)
            self.ag_claim = torch.zeros(1, device=self.device, dtype=torch.int32)
            self.ag_epoch = 0
        self.params_final = torch.cuda.Event()
        self.staging = None
        if self.reduce_engine == "ce":
            self.staging = torch.empty(self.w.world * max(u.shard_size for u in units), device=self.device,
                                       dtype=units[0].param.dtype)
        self.unit_index = {id(u): i for i, u in enumerate(units)}
        self.pregathered = set()
        if not serial:
            # The optimizer calls this after updating each shard: the next step's
            # gather of that unit starts while the remaining shards are updated.
            for u in units:
                u.on_updated = self.publish
        self.active = False
        self.visits = ()
        self.gathered = set()

    # ------------------------------------------------------------------ helpers
    def _signal(self, channel):
        self.seq[channel] += 1
        self.C.peer_signal(self.w.id, 0, channel, self.seq[channel])

    def _wait(self, channel, seq):
        if seq > 0:
            self.C.peer_wait(self.w.id, 0, channel, seq, self.poll_limit)

    # ------------------------------------------------------------------ schedule API
    def begin(self, visits):
        if self.active:
            raise ScheduleError("Finish the communication schedule before starting another")
        self.visits = visits
        self.compute = torch.cuda.current_stream(self.device)
        if self.serial:
            self.stream = self.compute
        self.stream.wait_stream(self.compute)  # this rank's optimizer step is done
        with torch.cuda.stream(self.stream):
            self._signal(CH_PARAMS)
            self._wait(CH_PARAMS, self.seq[CH_PARAMS])  # every peer's shards are final
            self.params_final.record(self.stream)
        self.gathered, self.pregathered = self.pregathered, set()
        self.active = True
        if not self.serial:
            # Gather every unit now, back to back, in visit order: the link never idles
            # waiting for compute, and compute waits only for the unit it needs.
            for i in range(len(visits)):
                if id(visits[i]) not in self.fused_keys:
                    self.prefetch(i)

    def prefetch(self, index):
        if index >= len(self.visits):
            return
        unit = self.visits[index]
        key = id(unit)
        if key in self.gathered:
            return
        self.gathered.add(key)
        with torch.cuda.stream(self.stream):
            gather = self.C.peer_allgather_ce if self.gather_engine == "ce" else self.C.peer_allgather
            gather(self.w.id, self.w.param_off[key], unit.shard_size, self.resident[key])
            self.ready[key].record(self.stream)

    def publish(self, unit):
        """After this rank's optimizer updated ``unit`` (on the compute stream): flag the
        unit's parameters as final to every peer and, on the communication stream,
        gather the unit for the next step once every peer has flagged it too."""
        if self.active:
            return  # an update inside a step: the next ``begin`` gathers as usual
        key = id(unit)
        if key in self.fused_keys:
            return  # gathered by its first GEMM in the next step
        ch = CH_UNIT + self.unit_index[key]
        self.seq.setdefault(ch, 0)
        self._signal(ch)
        seq = self.seq[ch]
        with torch.cuda.stream(self.stream):
            self._wait(ch, seq)
            gather = self.C.peer_allgather_ce if self.gather_engine == "ce" else self.C.peer_allgather
            gather(self.w.id, self.w.param_off[key], unit.shard_size, self.resident[key])
            self.ready[key].record(self.stream)
        self.pregathered.add(key)

    def acquire(self, index):
        unit = self.visits[index]
        key = id(unit)
        if key not in self.gathered or unit.gathered is not None:
            raise ScheduleError("Acquire exactly one prefetched unit")
        self.compute.wait_event(self.ready[key])
        unit.gathered = self.resident[key]
        unit.bind(unit.gathered)
        return unit

    def acquire_linear(self, index, x, name):
        """Acquire unit ``index`` and return ``x @ W^T`` for its parameter ``name``.

        In the fused gather mode the unit is gathered by that GEMM (``ag_gemm``):
        the GEMM waits only for the chunks of W each tile reads, and the whole unit
        is resident when it finishes. Otherwise: gather, acquire, plain GEMM."""
        from .. import ops
        unit = self.visits[index]
        key = id(unit)
        lo, hi = unit.offsets[name]
        shape = unit.shapes[name]
        if key not in self.fused_keys or key in self.gathered or lo % 8:
            self.prefetch(index)
            self.acquire(index)
            return ops.linear(x, _weight(unit, name))
        if unit.gathered is not None:
            raise ScheduleError("Acquire exactly one prefetched unit")
        self.gathered.add(key)
        x2 = x.reshape(-1, x.shape[-1])
        out = torch.empty(x2.shape[0], shape[0], device=x.device, dtype=x.dtype)
        self.compute.wait_event(self.params_final)
        self.ag_epoch += 1
        self.C.ag_gemm(self.w.id, self.w.param_off[key], unit.shard_size, self.resident[key], lo, shape[0],
                       shape[1], x2, out, self.ag_flags, self.ag_claim, self.ag_epoch, self.poll_limit)
        self.ready[key].record(self.compute)
        unit.gathered = self.resident[key]
        unit.bind(unit.gathered)
        return out.view(*x.shape[:-1], shape[0])

    def push_wgrad(self, index, dy, x, offset, shape):
        """Push mode: ``dW = dy^T x`` for the tensor at element ``offset`` of unit
        ``index``, stored by the GEMM's epilogue into the owners' slots. Returns
        False when this schedule does not push (the caller writes the view)."""
        if not self.push or offset % 8 or shape[-1] % 8:
            return False
        unit = self.visits[index]
        slot = index % 2
        if self.slot_owner[slot] != index:
            raise ScheduleError("push without a bound gradient slot")
        dy2, x2 = dy.reshape(-1, dy.shape[-1]), x.reshape(-1, x.shape[-1])
        self.C.gemm_rs(self.w.id, self.w.slot_off[slot], unit.shard_size, offset, dy2, x2)
        self.pushed[slot].append((offset, offset + shape[0] * shape[1]))
        return True

    def gradient_buffer(self, index):
        unit = self.visits[index]
        slot = index % 2
        if self.slot_owner[slot] is not None:
            raise ScheduleError("gradient slot still bound")
        # Every peer must have pulled this slot's previous contents.
        self._wait(CH_PULLED + slot, self.seq[CH_PULLED + slot])
        self.slot_owner[slot] = index
        buf = (self.local_grad[slot] if self.push else self.w.slots[slot])[:unit.full_size]
        self.pushed[slot] = []
        if _debug.enabled():  # every element must be rewritten by this unit's backward
            _debug.poison(buf)
        return buf

    def release(self, index):
        unit = self.visits[index]
        unit.release()

    def reduce(self, index):
        unit = self.visits[index]
        slot = index % 2
        if self.slot_owner[slot] != index:
            raise ScheduleError("reduce without a bound gradient slot")
        self.slot_owner[slot] = None
        unit.full_grad = None
        self.release(index)
        if self.push:
            # the gradients no GEMM pushed: the gaps between the pushed ranges
            at = 0
            for lo, hi in sorted(self.pushed[slot]) + [(unit.full_size, unit.full_size)]:
                if lo > at:
                    self.C.peer_push(self.w.id, self.w.slot_off[slot], unit.shard_size, self.local_grad[slot], at, lo)
                at = max(at, hi)
            self.pushed[slot] = []
        self._signal(CH_READY + slot)  # on compute: my slot holds unit's full gradient
        seq = self.seq[CH_READY + slot]
        self.stream.wait_stream(self.compute)
        with torch.cuda.stream(self.stream):
            self._wait(CH_READY + slot, seq)
            if self.push:
                self.C.peer_reduce_local(self.w.id, self.w.slot_off[slot], unit.shard_size, unit.grad)
            elif self.staging is not None:
                self.C.peer_reduce_avg_ce(self.w.id, self.w.slot_off[slot], unit.shard_size, unit.grad, self.staging)
            else:
                self.C.peer_reduce_avg(self.w.id, self.w.slot_off[slot], unit.shard_size, unit.grad)
            self._signal(CH_PULLED + slot)

    def finish(self):
        self.compute.wait_stream(self.stream)
        self.active = False

    def close(self):
        self.stream.synchronize()
