"""Provenance records and preflight refusals (no GPU needed)."""

import pytest

from nanospec_b200.utils import provenance as pv


def test_source_hashes_cover_product_sources():
    h = pv.source_hashes()
    assert "bench.py" in h and "csrc/gemm.cu" in h and "nanospec_b200/engine.py" in h
    assert all(len(v) == 64 for v in h.values())
    assert not any(k.startswith(("_work", "baseline", "tests")) for k in h)


def test_preflight_refuses_without_enough_gpus(monkeypatch):
    monkeypatch.setattr(pv.torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(pv.torch.cuda, "device_count", lambda: 2)
    monkeypatch.setattr(pv.torch.cuda, "get_device_name", lambda i: "NVIDIA B200")
    monkeypatch.setattr(pv.torch.cuda, "can_device_access_peer", lambda i, j: True)
    monkeypatch.setattr(pv, "topology_text", lambda: "GPU0 X NV18\nGPU1 NV18 X")
    with pytest.raises(pv.PreflightError, match="4 GPUs requested, 2 visible"):
        pv.preflight(4)
    assert pv.preflight(2)["devices"] == ["NVIDIA B200", "NVIDIA B200"]
    monkeypatch.setattr(pv.torch.cuda, "can_device_access_peer", lambda i, j: not (i == 1 and j == 0))
    with pytest.raises(pv.PreflightError, match="peer access"):
        pv.preflight(2)
    monkeypatch.setattr(pv.torch.cuda, "can_device_access_peer", lambda i, j: True)
    monkeypatch.setattr(pv, "topology_text", lambda: "GPU0 X PIX\nGPU1 PIX X")
    with pytest.raises(pv.PreflightError, match="NVLink"):
        pv.preflight(2)
    assert pv.preflight(2, require_nvlink=False)["peer_access"] == [[True, True], [True, True]]
