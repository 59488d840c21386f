"""Host-side check of the kernels' bounded waits.

Every device-side wait in this project (an mbarrier wait inside a GEMM, a peer
flag wait of the peer-memory schedule) is bounded: when it runs out it stores a
non-zero code in a per-device error word and the kernel returns instead of
hanging the GPU. This module makes such a timeout surface as a Python exception
on the host, without putting a synchronisation into the training step:

* ``snapshot(tag)`` enqueues, on the current stream, an asynchronous copy of the
  error word into pinned host memory and records an event behind it;
* ``check()`` looks at every snapshot whose event has completed (it never waits
  unless ``block=True``) and raises ``DeviceWaitTimeout`` naming the phase of the
  first snapshot that saw a non-zero word. Before raising it resets the device
  state (the split-K arrival counters and the error word), so the context stays
  usable for a retry or a clean shutdown.

``train()`` snapshots after the verifier, after the draft backward and after the
optimizer, and checks at the start of every call and after the optimizer (where
the host has already synchronised when the optimizer reads its scalars). So a
timeout raises in the same ``train()`` call with the default synchronous
optimizer, or at the start of the next call otherwise.

Codes: 1 = an mbarrier wait in a tensor-core kernel, 2 = a peer flag wait, 3 = a
token id outside the embedding table (the kernel skipped the access).
Reference policy: the reference raises on schedule misuse
(nanospec/shard.py:230-231,247-248) and relies on a finite NCCL timeout
(nanospec/distributed.py:24); it has no device-side waits of its own.
"""

from __future__ import annotations

import torch

from ..ops._ext import cuda_ops

CODES = {1: "a tensor-core kernel's mbarrier wait", 2: "a peer-memory flag wait",
         3: "an index out of range in an embedding gather or scatter (the access was skipped)"}


class DeviceWaitTimeout(RuntimeError):
    """A bounded device-side wait gave up (or a kernel skipped an out-of-range
    access); the step's results are not valid."""

    def __init__(self, code: int, tag: str):
        self.code, self.tag = code, tag
        what = CODES.get(code, f"error code {code}")
        verb = "was reported" if code == 3 else "timed out"
        super().__init__(f"{what} {verb} on the device during '{tag}'; the step's outputs are invalid "
                         f"(device state was reset)")


class _Done:
    """Stand-in for a CUDA event when the error word lives in host memory."""

    def query(self):
        return True

    def synchronize(self):
        pass


class ErrorMonitor:
    """Snapshots and checks the error word of one device (see the module doc).

    ``word`` / ``reset`` default to the CUDA extension's error word and reset
    routine; passing a CPU ``word`` tensor and a ``reset`` callable runs the same
    host logic without a GPU (the failure-path tests do this).
    """

    SLOTS = 16

    def __init__(self, device, word=None, reset=None):
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        if word is None:
            C = cuda_ops()
            with torch.cuda.device(self.device):
                word = C.device_error_tensor()

            def reset():
                with torch.cuda.device(self.device):
                    C.reset_device_error_state()
        self.word, self.reset = word, reset
        host = torch.zeros(self.SLOTS, dtype=torch.int32)
        self.host = host.pin_memory() if self.cuda else host
        self.pending = []  # (slot, event, tag)
        self.next = 0

    def snapshot(self, tag: str):
        if self.cuda and torch.cuda.is_current_stream_capturing():
            return
        if len(self.pending) >= self.SLOTS:
            self.check(block=True)
        slot = self.next
        self.next = (self.next + 1) % self.SLOTS
        self.host[slot:slot + 1].copy_(self.word, non_blocking=self.cuda)
        if self.cuda:
            ev = torch.cuda.Event()
            ev.record()
        else:
            ev = _Done()
        self.pending.append((slot, ev, tag))

    def check(self, block: bool = False):
        if self.cuda and torch.cuda.is_current_stream_capturing():
            return
        keep = []
        failed = None
        for slot, ev, tag in self.pending:
            if block:
                ev.synchronize()
            elif not ev.query():
                keep.append((slot, ev, tag))
                continue
            code = int(self.host[slot])
            if code and failed is None:
                failed = (code, tag)
        self.pending = keep
        if failed is not None:
            self.pending = []
            if self.reset is not None:
                self.reset()
            raise DeviceWaitTimeout(*failed)


_monitors: dict = {}


def monitor(device) -> ErrorMonitor | None:
    """The monitor of ``device`` (None for CPU devices)."""
    device = torch.device(device)
    if device.type != "cuda":
        return None
    key = device.index if device.index is not None else torch.cuda.current_device()
    m = _monitors.get(key)
    if m is None:
        m = _monitors[key] = ErrorMonitor(torch.device("cuda", key))
    return m
