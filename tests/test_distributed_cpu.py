"""Multi-rank host logic on CPU (gloo): sharding, pooled normalisation, checkpoints,
the verifier pipeline and the trainer hand-off. No GPU involved."""

import os
import socket
import tempfile
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import nanospec_b200 as N


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fn, args, errq):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.set_num_threads(1)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        fn(rank, world, *args)
        if dist.is_initialized():
            dist.barrier()
    except BaseException:  # report to the parent, never hang it
        errq.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def run_ranks(world, fn, *args, timeout=240):
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fn, args, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not alive, "ranks timed out"
    assert not errors, errors[0][1]
    assert all(p.exitcode == 0 for p in procs)


# ---------------------------------------------------------------------------- draft sharding
def _tiny_model(rank, world, dtype=torch.float32, name="tiny"):
    c = N.DraftConfig.load(N.config_path(name))
    g = torch.Generator().manual_seed(43)
    emb = (torch.randn(c.vocab_size, c.hidden_size, generator=g) * 0.1).to(dtype)
    head = (torch.randn(c.vocab_size, c.hidden_size, generator=g) * 0.1).to(dtype)
    group = dist.group.WORLD if world > 1 else None
    return c, N.DSpark(c, N.initialize(c, 42, dtype), emb, head, device="cpu", dtype=dtype,
                       group=group, world_size=world, rank=rank)


def _batch(c, b=2, s=64):
    g = torch.Generator().manual_seed(9)
    ids = torch.randint(0, c.vocab_size, (b, s), generator=g)
    hs = [torch.randn(b, s, c.hidden_size, generator=g) for _ in range(c.num_target_layers)]
    last = torch.randn(b, s, c.hidden_size, generator=g)
    mask = torch.ones(b, s)
    mask[1, 20:23] = 0  # unequal supervision on the second row
    return ids, hs, last, mask


def _sharded_step(rank, world, outdir):
    c, m = _tiny_model(rank, world)
    o = N.Objective(num_anchors=4)
    ids, hs, last, mask = _batch(c)
    torch.manual_seed(5)
    anchors, keep = N.sample_anchors(ids, mask, o)
    rows = slice(rank, rank + 1) if world > 1 else slice(0, 2)
    opt = N.AdamW(m.sharding, lr=1e-3, weight_decay=0.01)
    for _ in range(2):
        r = N.train(ids[rows], m, o, teacher_batch=N.TeacherBatch([h[rows] for h in hs], last[rows]),
                    loss_mask=mask[rows], anchors=(anchors[rows], keep[rows]), optimizer=opt)
    state = m.draft_state_dict()
    pooled = torch.stack((r.metrics.numerator, r.metrics.denominator))
    if world > 1:
        dist.all_reduce(pooled)
    if rank == 0:
        torch.save({"state": state, "loss": (pooled[0] / pooled[1]).item(), "update": r.update},
                   os.path.join(outdir, f"w{world}.pt"))


def test_sharded_training_matches_single_rank():
    with tempfile.TemporaryDirectory() as d:
        run_ranks(1, _sharded_step, d)
        run_ranks(2, _sharded_step, d)
        a = torch.load(os.path.join(d, "w1.pt"))
        b = torch.load(os.path.join(d, "w2.pt"))
    assert abs(a["loss"] - b["loss"]) < 1e-5
    assert abs(a["update"]["grad_norm"] - b["update"]["grad_norm"]) < 1e-5 * a["update"]["grad_norm"]
    assert abs(a["update"]["denominator"] - b["update"]["denominator"]) < 1e-6 * a["update"]["denominator"]
    for k in a["state"]:
        assert torch.allclose(a["state"][k], b["state"][k], atol=2e-6, rtol=1e-5), k


def _shard_layout(rank, world):
    c, m = _tiny_model(rank, world)
    full = N.initialize(c, 42, torch.float32)
    for name, unit in m.sharding.named_shards():
        assert unit.shard_size == -(-unit.numel // world)
        lo = rank * unit.shard_size
        flat = torch.cat([full[(name + "." if name.startswith("layers.") else "") + k].reshape(-1)
                          for k in unit.names])
        flat = torch.cat((flat, torch.zeros(unit.full_size - unit.numel)))
        assert torch.equal(unit.param, flat[lo:lo + unit.shard_size])
    exported = m.draft_state_dict()
    assert list(exported) == list(N.parameter_shapes(c))
    assert all(torch.equal(exported[k], full[k]) for k in full)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_shard_layout_and_export(world):
    run_ranks(world, _shard_layout)


def _ckpt(rank, world, path):
    from nanospec_b200 import checkpoint
    c, m = _tiny_model(rank, world)
    o = N.Objective(num_anchors=4)
    opt = N.AdamW(m.sharding, lr=1e-3)
    ids, hs, last, mask = _batch(c)
    rows = slice(rank, rank + 1)
    torch.manual_seed(rank)
    N.train(ids[rows], m, o, teacher_batch=N.TeacherBatch([h[rows] for h in hs], last[rows]),
            loss_mask=mask[rows], optimizer=opt)
    saved = checkpoint.save(path, m, opt, o, step=1)
    ref = {n: (u.param.clone(), u.master.clone(), u.m.clone(), u.v.clone()) for n, u in m.sharding.named_shards()}
    for u in m.sharding:  # clobber, then restore
        u.param.zero_(), u.master.zero_(), u.m.zero_(), u.v.zero_()
    opt.steps, opt.lr = 0, 5.0
    step = checkpoint.restore(saved, m, opt, o)
    assert step == 1 and opt.steps == 1 and opt.lr == 1e-3
    for n, u in m.sharding.named_shards():
        for a, b in zip((u.param, u.master, u.m, u.v), ref[n]):
            assert torch.equal(a, b)
    if rank == 0:
        assert os.path.exists(os.path.join(saved, "metadata.json"))
        assert sorted(os.listdir(saved)) == ["metadata.json"] + [f"rank-{r}.pt" for r in range(world)]
    with pytest.raises(ValueError):
        checkpoint.restore(saved, m, opt, N.Objective(num_anchors=5))


def test_sharded_checkpoint_roundtrip():
    with tempfile.TemporaryDirectory() as d:
        run_ranks(2, _ckpt, os.path.join(d, "ck"))


# ---------------------------------------------------------------------------- verifier pipeline
def _verifier(rank, world, ckpt_path, train_gpus, outdir):
    from nanospec_b200.config import Topology
    from nanospec_b200.models.verifier import Checkpoint, QwenStage, stage_forward
    from nanospec_b200.parallel.handoff import Teacher
    node = N.Node(train_gpus, topology=Topology(world=world, train_gpus=train_gpus), backend="gloo")
    capture = (1, 3)
    teacher = Teacher(node, ckpt_path, capture)
    ids = torch.randint(0, 512, (train_gpus, 40), generator=torch.Generator().manual_seed(3))
    res = N.train(ids, verifier=teacher)
    if node.training:
        full = QwenStage(Checkpoint(ckpt_path), 0, 4, device="cpu", first=True, last=True)
        x, cap = stage_forward(full, ids[rank:rank + 1], capture=capture)
        tb = res.teacher
        assert tb.logits is None
        for got, layer in zip(tb.hidden_states, capture):
            assert torch.equal(got, cap[layer]), layer
        assert torch.equal(tb.last_hidden, x)


@pytest.mark.parametrize("world,train_gpus", [(3, 1), (4, 2), (2, 2)])
def test_verifier_pipeline_handoff(world, train_gpus):
    from nanospec_b200.models.verifier import tiny_hybrid_text_config, write_synthetic_checkpoint
    with tempfile.TemporaryDirectory() as d:
        path = write_synthetic_checkpoint(os.path.join(d, "ck"), tiny_hybrid_text_config(), fp8=False, seed=2)
        run_ranks(world, _verifier, str(path), train_gpus, d)


# ---------------------------------------------------------------------------- CLI
def _cli(rank, world, outdir, extra):
    from nanospec_b200.cli import main
    rows = main(["--config", "tiny-hybrid", "--steps", "2", "--seq-len", "64", "--anchors", "4",
                 "--dtype", "float32", "--output", os.path.join(outdir, "run.json"), "--backend", "gloo",
                 "--learning-rate", "1e-3"] + extra)
    if rank == 0:
        assert len(rows) == 2 and all(r["updated"] for r in rows)


def test_cli_with_synthetic_verifier_and_resume():
    import glob
    import json
    with tempfile.TemporaryDirectory() as d:
        run_ranks(2, _cli, d, ["--train-gpus", "1", "--synthetic-target", "tiny"])
        report = json.load(open(os.path.join(d, "run.json")))
        assert report["verifier"] and len(report["steps"]) == 2
        ck = report["checkpoint"]
        assert os.path.exists(os.path.join(ck, "metadata.json"))
        run_ranks(2, _cli, d, ["--train-gpus", "1", "--synthetic-target", "tiny", "--checkpoint", ck])
        report2 = json.load(open(os.path.join(d, "run.json")))
        assert [r["step"] for r in report2["steps"]] == [3, 4]
        assert len(glob.glob(os.path.join(d, "run-checkpoint-step*"))) == 2


def test_cli_without_verifier_single_process():
    with tempfile.TemporaryDirectory() as d:
        from nanospec_b200.cli import main
        os.environ.pop("WORLD_SIZE", None)
        rows = main(["--config", "tiny", "--steps", "2", "--seq-len", "48", "--anchors", "4", "--dtype", "float32",
                     "--output", os.path.join(d, "r.json"), "--no-verifier", "--backend", "gloo"])
        assert len(rows) == 2
        for r in rows:  # per-phase timing of every step
            assert set(r["phase_ms"]) == {"draft_forward", "head", "draft_backward", "optimizer"}
            assert all(v >= 0 for v in r["phase_ms"].values())


# ---------------------------------------------------------------------------- replicated verifier
def _replicated(rank, world, outdir):
    import math

    from nanospec_b200.config import Topology
    from nanospec_b200.models.verifier import QwenStage, stage_forward, synthetic_hf_config, tiny_hybrid_text_config
    from nanospec_b200.parallel.handoff import Teacher
    tc = tiny_hybrid_text_config()
    node = N.Node(world, topology=Topology.replicated(world), backend="gloo")
    assert node.training and node.inference_ranks == list(range(world))
    c = N.DraftConfig.load(N.config_path("tiny-hybrid"))
    g = torch.Generator().manual_seed(5)
    emb = (torch.randn(c.vocab_size, c.hidden_size, generator=g) * 0.1).bfloat16()
    head = (torch.randn(c.vocab_size, c.hidden_size, generator=g) * 0.1).bfloat16()
    teacher = Teacher.random(node, tc, c.target_layer_ids, seed=11, embed=emb, lm_head=head)
    assert teacher.stage.start == 0 and teacher.stage.end == 4 and teacher.handoff_group is None
    # the verifier and the draft share the frozen target tensors
    assert teacher.stage.embed_tokens.weight.data_ptr() == emb.data_ptr()
    ids = torch.randint(0, c.vocab_size, (world, 48), generator=torch.Generator().manual_seed(3))
    res = N.train(ids, verifier=teacher)
    x, cap = stage_forward(teacher.stage, ids[rank:rank + 1], capture=c.target_layer_ids)
    for got, layer in zip(res.teacher.hidden_states, c.target_layer_ids):
        assert torch.equal(got, cap[layer])
    assert torch.equal(res.teacher.last_hidden, x)
    # every replica holds the same weights: one seed, one draw
    w = teacher.stage.layers[0].mlp.gate_proj.weight.float().sum().reshape(1)
    ws = [torch.zeros(1) for _ in range(world)]
    dist.all_gather(ws, w)
    assert all(torch.equal(ws[0], t) for t in ws)
    model = N.DSpark(c, N.initialize(c, 1, torch.float32), emb, head, device="cpu", dtype=torch.float32,
                     group=node.train_group, world_size=world, rank=rank)
    opt = N.AdamW(model.sharding, lr=1e-3)
    torch.manual_seed(rank)
    r = N.train(ids, model, N.Objective(num_anchors=4, block_size=4), verifier=teacher, optimizer=opt)
    assert r.update["updated"] and math.isfinite(float(r.metrics.loss))


@pytest.mark.parametrize("world", [1, 2])
def test_replicated_verifier_topology(world):
    with tempfile.TemporaryDirectory() as d:
        run_ranks(world, _replicated, d)
