"""Sharded optimizer checkpoints: staged off the GPU asynchronously, committed by metadata.

On-disk format (the reference's, nanospec/checkpoint.py:14-82, kept so that
checkpoints interchange between the two projects):

* one directory per save, ``{prefix}-step{step}-{tag}`` with a 12-hex-digit tag that
  every rank agrees on, so a complete generation is never overwritten;
* ``rank-{r}.pt`` per training rank: ``{"units": {unit: {"param", "master", "m",
  "v"}}, "optimizer_steps", "rng", "step"}``, written to a temporary name and renamed;
* ``metadata.json`` last (written by rank 0 after every rank file exists): a
  checkpoint is complete exactly when it has one.

Design here:

* ``Snapshot``: the shard tensors are copied into pinned host buffers on a side CUDA
  stream, so training continues while the copy runs; the buffers are reused by the
  next snapshot of the same model. ``save`` waits for the copy, ``save_async``
  returns a ``PendingSave`` whose file writing runs on a background thread (the
  collective parts, agreeing on the tag and the final barrier, stay on the caller's
  thread in ``PendingSave.commit``).
* ``METADATA``: a declarative schema of the metadata fields, how each is read from
  the run and whether a mismatch refuses a resume. ``restore`` compares field by
  field and raises ``CheckpointMismatch`` listing every difference (for nested
  dicts, the differing keys), instead of stopping at the first.
* ``latest(prefix)`` finds the newest complete generation; ``Periodic`` saves every
  N steps and keeps the newest K generations.
"""

from __future__ import annotations

import glob
import json
import os
import secrets
import shutil
import threading
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any, Callable

import torch
import torch.distributed as dist

from .config import TARGET_MODEL, TARGET_REVISION

SHARD_FIELDS = ("param", "master", "m", "v")
OPTIMIZER_HPARAMS = ("lr", "weight_decay", "betas", "eps", "max_grad_norm")


class CheckpointMismatch(ValueError):
    """The checkpoint was written by a run that differs from this one."""


# ---------------------------------------------------------------------------- metadata schema
@dataclass(frozen=True)
class MetaField:
    name: str
    read: Callable[[Any], Any]      # run -> value (run: a _Run)
    must_match: bool = True         # a mismatch refuses the resume
    restore: Callable[[Any, Any], None] | None = None  # (run, stored value) -> apply


def _set_hparams(run, stored):
    for k, v in stored.items():
        setattr(run.optimizer, k, tuple(v) if isinstance(v, list) else v)


METADATA = (
    MetaField("config", lambda r: r.model.config.to_dict()),
    MetaField("objective", lambda r: asdict(r.objective)),
    MetaField("world_size", lambda r: r.unit.world_size),
    MetaField("step", lambda r: r.step, must_match=False),
    MetaField("target", lambda r: TARGET_MODEL),
    MetaField("target_revision", lambda r: TARGET_REVISION),
    MetaField("dtype", lambda r: str(r.unit.param.dtype)),
    MetaField("optimizer", lambda r: {k: getattr(r.optimizer, k) for k in OPTIMIZER_HPARAMS}, must_match=False,
              restore=_set_hparams),
)


def _jsonable(v):
    return json.loads(json.dumps(v))


def _differences(name, stored, current):
    """Human-readable differences between two JSON values (nested dicts by key)."""
    stored, current = _jsonable(stored), _jsonable(current)
    if isinstance(stored, dict) and isinstance(current, dict):
        out = []
        for k in sorted(set(stored) | set(current)):
            if k not in stored:
                out.append(f"{name}.{k}: absent in the checkpoint, run has {current[k]!r}")
            elif k not in current:
                out.append(f"{name}.{k}: checkpoint has {stored[k]!r}, absent in the run")
            else:
                out.extend(_differences(f"{name}.{k}", stored[k], current[k]))
        return out
    return [] if stored == current else [f"{name}: checkpoint {stored!r}, run {current!r}"]


@dataclass
class _Run:
    model: Any
    optimizer: Any
    objective: Any
    step: int = 0

    @property
    def unit(self):
        return self.model.sharding.context


def build_metadata(run: _Run) -> dict:
    return {f.name: _jsonable(f.read(run)) for f in METADATA}


def check_metadata(meta: dict, run: _Run):
    """Raise ``CheckpointMismatch`` listing every field that refuses the resume."""
    problems = []
    for f in METADATA:
        if f.name not in meta:
            problems.append(f"{f.name}: missing from metadata.json")
        elif f.must_match:
            problems.extend(_differences(f.name, meta[f.name], f.read(run)))
    if problems:
        raise CheckpointMismatch("checkpoint does not match this run:\n  " + "\n  ".join(problems))


# ---------------------------------------------------------------------------- staging
class Snapshot:
    """Pinned host copies of this rank's shards (reused between saves of one model)."""

    def __init__(self, model):
        self.model = model
        self.host = {}
        for name, unit in model.sharding.named_shards():
            self.host[name] = {}
            for f in SHARD_FIELDS:
                t = getattr(unit, f)
                buf = torch.empty(t.shape, dtype=t.dtype)
                self.host[name][f] = buf.pin_memory() if t.is_cuda else buf
        dev = model.sharding.context.param.device
        self.stream = torch.cuda.Stream(device=dev) if dev.type == "cuda" else None
        self.done = None

    def stage(self):
        """Start the device-to-host copies; training may continue right away."""
        units = dict(self.model.sharding.named_shards())
        if self.stream is None:
            for name, fields in self.host.items():
                for f, buf in fields.items():
                    buf.copy_(getattr(units[name], f))
            return
        self.stream.wait_stream(torch.cuda.current_stream(self.stream.device))
        with torch.cuda.stream(self.stream):
            for name, fields in self.host.items():
                for f, buf in fields.items():
                    src = getattr(units[name], f)
                    buf.copy_(src, non_blocking=True)
                    src.record_stream(self.stream)
        self.done = torch.cuda.Event()
        self.done.record(self.stream)

    def wait(self):
        if self.done is not None:
            self.done.synchronize()


def _rng_state(device):
    return torch.cuda.get_rng_state(device) if device.type == "cuda" else torch.get_rng_state()


def _set_rng_state(state, device):
    if device.type == "cuda":
        torch.cuda.set_rng_state(state, device)
    else:
        torch.set_rng_state(state)


def _agree_on_tag(unit) -> str:
    """12 hex digits drawn on rank 0 and broadcast as bytes to the other ranks."""
    raw = torch.zeros(6, dtype=torch.uint8)
    if unit.rank == 0:
        raw = torch.frombuffer(bytearray(secrets.token_bytes(6)), dtype=torch.uint8).clone()
    if unit.world_size > 1:
        dev = unit.param.device if dist.get_backend(unit.group) == "nccl" else torch.device("cpu")
        t = raw.to(dev)
        dist.broadcast(t, src=0, group=unit.group)
        raw = t.cpu()
    return bytes(raw.tolist()).hex()


def _write_atomic(target: Path, write):
    tmp = target.with_suffix(".tmp")
    write(tmp)
    tmp.replace(target)


# ---------------------------------------------------------------------------- save / restore
class PendingSave:
    """A save whose rank file is being written on a background thread.

    ``commit()`` (collective) waits for this rank's file, then rank 0 writes the
    metadata once every rank's file exists; returns the checkpoint directory.
    """

    def __init__(self, directory: Path, run: _Run, snapshot: Snapshot, rng):
        self.dir, self.run, self.snap = directory, run, snapshot
        self.error = None
        unit = run.unit
        payload_rank = unit.rank
        optimizer_steps = run.optimizer.steps

        def work():
            try:
                snapshot.wait()
                payload = {"units": {n: dict(f) for n, f in snapshot.host.items()},
                           "optimizer_steps": optimizer_steps, "rng": rng, "step": run.step}
                _write_atomic(directory / f"rank-{payload_rank}.pt", lambda p: torch.save(payload, p))
            except BaseException as exc:  # surfaced by commit()
                self.error = exc

        self.thread = threading.Thread(target=work, name="nanospec-ckpt", daemon=True)
        self.thread.start()

    def commit(self) -> str:
        self.thread.join()
        unit = self.run.unit
        ok = torch.tensor([0 if self.error is None else 1], dtype=torch.int32)
        if unit.world_size > 1:
            dev = unit.param.device if dist.get_backend(unit.group) == "nccl" else torch.device("cpu")
            okd = ok.to(dev)
            dist.all_reduce(okd, group=unit.group)
            ok = okd.cpu()
        if int(ok) != 0:
            raise RuntimeError(f"checkpoint rank file write failed on a rank: {self.error!r}")
        if unit.rank == 0:
            meta = build_metadata(self.run)
            _write_atomic(self.dir / "metadata.json", lambda p: p.write_text(json.dumps(meta, indent=2)))
        if unit.world_size > 1:
            dist.barrier(group=unit.group)
        return str(self.dir)


def save_async(path, model, optimizer, objective, step, snapshot: Snapshot | None = None) -> PendingSave:
    """Stage this rank's shards to host memory and write them in the background.

    Collective over the training ranks (the tag). Call ``commit()`` on the result on
    every rank before the next save.
    """
    run = _Run(model, optimizer, objective, step)
    unit = run.unit
    tag = _agree_on_tag(unit)
    directory = Path(f"{path}-step{step}-{tag}")
    directory.mkdir(parents=True, exist_ok=True)
    snap = snapshot or Snapshot(model)
    snap.stage()
    return PendingSave(directory, run, snap, _rng_state(unit.param.device))


def save(path, model, optimizer, objective, step) -> str:
    """Synchronous save (collective over the training ranks); returns the directory."""
    return save_async(path, model, optimizer, objective, step).commit()


def restore(path, model, optimizer, objective) -> int:
    """Load this rank's shards, optimizer step count, hyper-parameters and CUDA RNG.

    Refuses (``CheckpointMismatch`` / ``ValueError``) incomplete or unreadable
    checkpoints and any run whose config, objective, world size, dtype or target
    differs from the checkpoint's. Returns the saved step.
    """
    run = _Run(model, optimizer, objective)
    unit = run.unit
    path = Path(path)
    meta_file = path / "metadata.json"
    if not meta_file.exists():
        raise ValueError(f"{path} is not a complete checkpoint (no metadata.json)")
    meta = json.loads(meta_file.read_text())
    check_metadata(meta, run)
    rank_file = path / f"rank-{unit.rank}.pt"
    try:
        state = torch.load(rank_file, map_location="cpu", weights_only=True)
    except Exception as exc:  # truncated or corrupt file
        raise ValueError(f"Unreadable checkpoint shard {rank_file}: {exc}") from exc
    if state.get("step") != meta["step"]:
        raise ValueError(f"{rank_file} holds step {state.get('step')}, metadata.json step {meta['step']}")
    stored_units = state.get("units", {})
    for name, shard in model.sharding.named_shards():
        if name not in stored_units:
            raise ValueError(f"{rank_file} has no unit {name!r}")
        for f in SHARD_FIELDS:
            src, dst = stored_units[name][f], getattr(shard, f)
            if tuple(src.shape) != tuple(dst.shape):
                raise ValueError(f"{rank_file}: {name}.{f} is {tuple(src.shape)}, the run has {tuple(dst.shape)}")
            dst.copy_(src)
    for f in METADATA:
        if f.restore is not None:
            f.restore(run, meta[f.name])
    optimizer.steps = state["optimizer_steps"]
    model.sharding.parameters_changed()
    _set_rng_state(state["rng"], unit.param.device)
    return int(state["step"])


def latest(prefix) -> str | None:
    """Newest complete generation ``{prefix}-step*-*`` (by step), or None."""
    found = []
    for d in glob.glob(f"{prefix}-step*-*"):
        try:
            found.append((json.loads(Path(d, "metadata.json").read_text())["step"], d))
        except (OSError, ValueError, KeyError):
            continue  # incomplete or unreadable generation
    return max(found)[1] if found else None


class Periodic:
    """Save every ``every`` steps, asynchronously, keeping the newest ``keep`` generations.

    ``step(step)`` after an optimizer step: commits the previous pending save (if any),
    then starts a new one when ``step % every == 0``. ``close()`` commits the last one.
    Collective: every training rank calls it with the same steps.
    """

    def __init__(self, prefix, model, optimizer, objective, every: int, keep: int = 2):
        if every < 1 or keep < 1:
            raise ValueError("every and keep must be positive")
        self.prefix, self.model, self.optimizer, self.objective = prefix, model, optimizer, objective
        self.every, self.keep = every, keep
        self.pending = None
        self.snapshot = None

    def step(self, step: int):
        self.close()
        if step % self.every:
            return
        if self.snapshot is None:
            self.snapshot = Snapshot(self.model)
        self.pending = save_async(self.prefix, self.model, self.optimizer, self.objective, step, self.snapshot)

    def close(self) -> str | None:
        if self.pending is None:
            return None
        out = self.pending.commit()
        self.pending = None
        if self.model.sharding.context.rank == 0:
            gens = []
            for d in glob.glob(f"{self.prefix}-step*-*"):
                try:
                    gens.append((json.loads(Path(d, "metadata.json").read_text())["step"], d))
                except (OSError, ValueError, KeyError):
                    continue
            for _, d in sorted(gens)[:-self.keep]:
                shutil.rmtree(d, ignore_errors=True)
        return out
