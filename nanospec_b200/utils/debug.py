"""Debug mode (``NANOSPEC_DEBUG=1``): hazards made visible instead of silent.

* Poison fill: buffers that the schedule considers free are filled with NaN before
  their next user may touch them (a released gather slot before the next all-gather
  into it, a gradient slot before the backward binds it, a single-rank gradient shard
  before the next backward overwrites it). A read of stale data after a release, or
  a gradient element the backward failed to write, then turns into NaN, which the
  optimizer's finite check reports as a skipped update.
* Synchronous device checks: ``train()`` waits for each phase's error-word snapshot,
  so a device-side timeout or out-of-range index raises in the phase that caused it.

Results in debug mode are identical to normal mode when nothing reads freed memory
(the tests check this); the cost is one fill per buffer release and a host wait per
phase.
"""

from __future__ import annotations

import os

import torch


def enabled() -> bool:
    return os.environ.get("NANOSPEC_DEBUG", "0") not in ("", "0")


def poison(t: torch.Tensor):
    """Fill ``t`` with NaN (floating) on the current stream."""
    if t is not None and t.is_floating_point() and t.numel():
        t.fill_(float("nan"))
