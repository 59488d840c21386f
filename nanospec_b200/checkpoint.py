"""Per-rank optimizer checkpoints, complete once ``metadata.json`` exists.

On-disk layout (shared with the reference, nanospec/checkpoint.py:14-82, so
checkpoints interchange):

``{path}-step{step}-{tag12}/rank-{r}.pt`` =
``{"units": {unit: {"param", "master", "m", "v"}}, "optimizer_steps", "rng", "step"}``
written as ``rank-{r}.tmp`` then renamed; after a barrier rank 0 writes
``metadata.json`` (config, objective, world_size, step, target, target_revision,
dtype, optimizer hyper-parameters) through a temporary file. A new directory per
save means a complete generation is never overwritten.

Addition: ``latest(path_prefix)`` finds the newest complete generation.
"""

from __future__ import annotations

import glob
import json
import os
import uuid
from dataclasses import asdict
from pathlib import Path

import torch
import torch.distributed as dist

from .config import TARGET_MODEL, TARGET_REVISION

FIELDS = ("param", "master", "m", "v")


def _rng_state(device):
    if device.type == "cuda":
        return torch.cuda.get_rng_state(device)
    return torch.get_rng_state()


def _set_rng_state(state, device):
    if device.type == "cuda":
        torch.cuda.set_rng_state(state, device)
    else:
        torch.set_rng_state(state)


def save(path, model, optimizer, objective, step) -> str:
    first = model.sharding.context
    tag = [uuid.uuid4().hex[:12] if first.rank == 0 else None]
    if first.world_size > 1:
        dist.broadcast_object_list(tag, src=_group_src(first), group=first.group)
    out = Path(f"{path}-step{step}-{tag[0]}")
    out.mkdir(parents=True, exist_ok=True)
    units = {}
    for name, unit in model.sharding.named_shards():
        units[name] = {f: getattr(unit, f).detach().to("cpu", copy=True) for f in FIELDS}
    payload = {"units": units, "optimizer_steps": optimizer.steps,
               "rng": _rng_state(first.param.device), "step": step}
    tmp = out / f"rank-{first.rank}.tmp"
    torch.save(payload, tmp)
    tmp.replace(out / f"rank-{first.rank}.pt")
    if first.world_size > 1:
        dist.barrier(group=first.group)
    if first.rank == 0:
        meta = {
            "config": model.config.to_dict(),
            "objective": asdict(objective),
            "world_size": first.world_size,
            "step": step,
            "target": TARGET_MODEL,
            "target_revision": TARGET_REVISION,
            "dtype": str(first.param.dtype),
            "optimizer": {k: getattr(optimizer, k)
                          for k in ("lr", "weight_decay", "betas", "eps", "max_grad_norm")},
        }
        tmpm = out / "metadata.tmp"
        tmpm.write_text(json.dumps(meta, indent=2))
        tmpm.replace(out / "metadata.json")
    if first.world_size > 1:
        dist.barrier(group=first.group)
    return str(out)


def _group_src(unit):
    # Training ranks are 0..N-1 and rank 0 is in the group.
    return 0


def restore(path, model, optimizer, objective) -> int:
    first = model.sharding.context
    path = Path(path)
    meta_file = path / "metadata.json"
    if not meta_file.exists():
        raise ValueError(f"{path} is not a complete checkpoint (no metadata.json)")
    meta = json.loads(meta_file.read_text())
    if meta["world_size"] != first.world_size or meta["dtype"] != str(first.param.dtype):
        raise ValueError("Resume requires the same training GPU count and dtype")
    if json.dumps(meta["config"], sort_keys=True) != json.dumps(model.config.to_dict(), sort_keys=True):
        raise ValueError("Checkpoint configuration mismatch")
    if meta["objective"] != asdict(objective):
        raise ValueError("Checkpoint objective mismatch")
    if meta["target"] != TARGET_MODEL or meta["target_revision"] != TARGET_REVISION:
        raise ValueError("Checkpoint teacher revision mismatch")
    rank_file = path / f"rank-{first.rank}.pt"
    try:
        state = torch.load(rank_file, map_location="cpu", weights_only=True)
    except Exception as exc:  # truncated or corrupt file
        raise ValueError(f"Unreadable checkpoint shard {rank_file}: {exc}") from exc
    if state["step"] != meta["step"]:
        raise ValueError("Checkpoint rank file does not match its metadata")
    for name, unit in model.sharding.named_shards():
        stored = state["units"].get(name)
        if stored is None:
            raise ValueError(f"Checkpoint misses unit {name}")
        for f in FIELDS:
            value = stored[f]
            target = getattr(unit, f)
            if value.shape != target.shape:
                raise ValueError(f"Checkpoint unit {name}.{f} has shape {tuple(value.shape)}")
            target.copy_(value)
    for k, v in meta["optimizer"].items():
        setattr(optimizer, k, tuple(v) if k == "betas" else v)
    optimizer.steps = state["optimizer_steps"]
    model.sharding.parameters_changed()
    _set_rng_state(state["rng"], first.param.device)
    return state["step"]


def latest(prefix) -> str | None:
    """Newest complete generation ``{prefix}-step*-*`` (by step), or None."""
    best, best_step = None, -1
    for d in glob.glob(f"{prefix}-step*-*"):
        if not os.path.exists(os.path.join(d, "metadata.json")):
            continue
        try:
            step = json.loads(Path(d, "metadata.json").read_text())["step"]
        except (ValueError, KeyError):
            continue
        if step > best_step:
            best, best_step = d, step
    return best
