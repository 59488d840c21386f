"""Preflight checks of the box and provenance records for run reports.

Reference: the Modal launcher checks the GPU count, all-to-all CUDA peer access
and NVLink before it starts torchrun, and stamps each report with the topology,
device names, peer-access matrix and a sha256 per source file
(modal_app.py:133-155, 199-210). Here the same checks are a library call that the
CLI and the benchmark run on the box itself:

* ``preflight(world)`` raises ``PreflightError`` when fewer than ``world`` GPUs are
  visible, when two of the first ``world`` GPUs cannot access each other's memory
  (the peer-memory schedule needs it), or when ``nvidia-smi topo -m`` shows no
  NVLink between them; ``require_nvlink=False`` relaxes the last check.
* ``provenance()`` returns a JSON-able dict: devices, peer access, NVLink topology
  text, driver / CUDA / torch / NCCL versions, the git head if any, and sha256 of
  every product source file (the package, the CUDA sources, ``bench.py``).
"""

from __future__ import annotations

import hashlib
import subprocess
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[2]


class PreflightError(RuntimeError):
    pass


def _run(cmd) -> tuple[int, str]:
    try:
        p = subprocess.run(cmd, text=True, capture_output=True, check=False, timeout=30)
        return p.returncode, p.stdout + p.stderr
    except (OSError, subprocess.TimeoutExpired) as exc:
        return -1, str(exc)


def topology_text() -> str:
    rc, out = _run(["nvidia-smi", "topo", "-m"])
    if rc != 0:
        rc2, out2 = _run(["nvidia-smi", "nvlink", "--status"])
        out += out2
    return out


def peer_matrix(n: int) -> list[list[bool]]:
    return [[True if i == j else bool(torch.cuda.can_device_access_peer(i, j)) for j in range(n)] for i in range(n)]


def preflight(world: int, *, require_peer: bool = True, require_nvlink: bool = True) -> dict:
    """Check that this box can run ``world`` GPUs of one job; returns what it saw."""
    if not torch.cuda.is_available():
        raise PreflightError("no CUDA device is visible")
    count = torch.cuda.device_count()
    devices = [torch.cuda.get_device_name(i) for i in range(count)]
    if count < world:
        raise PreflightError(f"{world} GPUs requested, {count} visible: {devices}")
    peers = peer_matrix(world)
    if require_peer and world > 1 and not all(map(all, peers)):
        raise PreflightError(f"CUDA peer access is not all-to-all among GPUs 0..{world - 1}: {peers}")
    topo = topology_text() if world > 1 else ""
    if require_nvlink and world > 1 and "NV" not in topo and "GB/s" not in topo:
        raise PreflightError("could not verify NVLink connectivity (nvidia-smi topo -m shows no NV links)")
    return {"devices": devices[:world], "peer_access": peers, "topology": topo}


def source_hashes() -> dict:
    files = sorted(list((ROOT / "nanospec_b200").rglob("*.py")) + list((ROOT / "nanospec_b200").rglob("*.json")) +
                   list((ROOT / "csrc").rglob("*.cu")) + list((ROOT / "csrc").rglob("*.cuh")) +
                   list((ROOT / "csrc").rglob("*.h")) + list((ROOT / "csrc").rglob("*.cpp")) +
                   [ROOT / "bench.py", ROOT / "setup.py"])
    return {str(p.relative_to(ROOT)): hashlib.sha256(p.read_bytes()).hexdigest() for p in files if p.exists()}


def provenance(world: int | None = None) -> dict:
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    world = n if world is None else min(world, n)
    rc, head = _run(["git", "-C", str(ROOT), "rev-parse", "HEAD"])
    rc_d, drv = _run(["nvidia-smi", "--query-gpu=driver_version", "--format=csv,noheader"])
    hashes = source_hashes()
    combined = hashlib.sha256("".join(f"{k}:{v}\n" for k, v in sorted(hashes.items())).encode()).hexdigest()
    out = {
        "devices": [torch.cuda.get_device_name(i) for i in range(world)],
        "peer_access": peer_matrix(world) if world else [],
        "topology": topology_text() if world > 1 else "",
        "driver": drv.strip().splitlines()[0] if rc_d == 0 and drv.strip() else None,
        "cuda": torch.version.cuda,
        "torch": torch.__version__,
        "nccl": ".".join(map(str, torch.cuda.nccl.version())) if torch.cuda.is_available() else None,
        "git_head": head.strip() if rc == 0 else None,
        "source_sha256": combined,
        "source_files": hashes,
    }
    return out
