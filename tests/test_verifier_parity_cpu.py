"""The verifier (our stage forward on CPU) vs the reference's own verifier path.

The reference runs its verifier inside ``train(ids, verifier=teacher)`` and needs a
process group; here that is a one-rank gloo group and a minimal node object, on a
synthetic FP8 checkpoint written by this project (the reference loads it as is).
"""

import os
import socket
import types

import pytest
import torch
import torch.distributed as dist

from nanospec_b200.models.verifier import (Checkpoint, QwenStage, stage_forward, tiny_hybrid_text_config,
                                           write_synthetic_checkpoint)


@pytest.fixture()
def one_rank_group():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    yield
    dist.destroy_process_group()


def _cos(a, b):
    return torch.nn.functional.cosine_similarity(a.float().flatten(), b.float().flatten(), dim=0).item()


def test_verifier_matches_reference(reference, tmp_path, one_rank_group, monkeypatch):
    tc = tiny_hybrid_text_config(hidden=128, vocab=384, heads=4, head_dim=32, ffn=256)
    path = write_synthetic_checkpoint(tmp_path / "ck", tc, seed=3, fp8=True)
    capture = (1, 3)
    ids = torch.randint(0, tc["vocab_size"], (2, 70), generator=torch.Generator().manual_seed(0))

    # reference: its Teacher + train(verifier=...) on a one-rank node
    node = types.SimpleNamespace(rank=0, world=1, device=torch.device("cpu"), train_gpus=1, training=True,
                                 inference_ranks=[0], train_group=None)
    node.broadcast = types.MethodType(reference.distributed.Node.broadcast, node)
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a, **k: None)
    teacher = reference.distributed.Teacher(node, str(path), capture)
    ref = reference.train.train(ids, verifier=teacher).teacher

    ours = QwenStage(Checkpoint(path), 0, tc["num_hidden_layers"], device="cpu", first=True, last=True)
    final, caps = stage_forward(ours, ids, capture=capture)
    # The reference keeps row 0 for the (single) trainer.
    for got, layer in zip(ref.hidden_states, capture):
        assert _cos(caps[layer][0:1], got) > 0.999, layer
    assert _cos(final[0:1], ref.last_hidden) > 0.999
    # Layer 1 is two gated-DeltaNet layers in: within a few bf16 ulps.
    assert (caps[1][0:1].float() - ref.hidden_states[0].float()).abs().max().item() < 0.05
    # Teacher logits: the reference broadcasts them; ours recomputes them in the head.
    logits = final[0:1] @ ours.lm_head.weight.t()
    assert _cos(logits, ref.logits) > 0.999
