"""Multi-GPU schedules on B200 (2+ GPUs; spawned NCCL ranks), plus the bounded-wait
timeout of the peer flag protocol (1 GPU, a flag that nothing sets)."""

import os
import socket
import tempfile
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import nanospec_b200 as N

pytestmark = pytest.mark.gpu
ngpu = torch.cuda.device_count() if torch.cuda.is_available() else 0
two_gpus = pytest.mark.skipif(ngpu < 2, reason="needs 2 GPUs")


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fn, args, errq):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    try:
        from datetime import timedelta
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", rank))
        fn(rank, world, *args)
        torch.cuda.synchronize()
        dist.barrier()
    except BaseException:
        errq.put((rank, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def run_ranks(world, fn, *args, timeout=600):
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


def _model(rank, world, name="tiny-hybrid"):
    c = N.DraftConfig.load(N.config_path(name))
    g = torch.Generator().manual_seed(43)
    emb = torch.randn(c.vocab_size, c.hidden_size, generator=g) * 0.1
    head = torch.randn(c.vocab_size, c.hidden_size, generator=g) * 0.1
    dev = torch.device("cuda", rank)
    m = N.DSpark(c, N.initialize(c, 42, torch.bfloat16), emb, head, device=dev, dtype=torch.bfloat16,
                 group=dist.group.WORLD, world_size=world, rank=rank)
    return c, m


def _data(c, rank, b=8, s=512):
    dev = torch.device("cuda", rank)
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    ids = torch.randint(0, c.vocab_size, (b, s), device=dev, generator=g)
    hs = [torch.randn(b, s, c.hidden_size, device=dev, generator=g).bfloat16() for _ in range(c.num_target_layers)]
    last = torch.randn(b, s, c.hidden_size, device=dev, generator=g).bfloat16()
    mask = torch.ones(b, s, device=dev)
    if rank % 2:
        mask[:, 100:103] = 0
    return ids, hs, last, mask


def _digest(m):
    return [t.clone() for s in m.sharding for t in (s.param, s.master, s.m, s.v)]


def _schedules(rank, world, outdir):
    c, m = _model(rank, world)
    o = N.Objective(num_anchors=8)
    ids, hs, last, mask = _data(c, rank)
    init = [s.param.clone() for s in m.sharding]
    results = {}
    for mode in ("nccl_serial", "nccl_overlap", "peer_serial", "peer_overlap"):
        if mode.startswith("peer"):
            m.sharding.enable_peer()
        for s, p0 in zip(m.sharding, init):
            s.param.copy_(p0)
            s.master.copy_(s.param)
            s.m.zero_(), s.v.zero_(), s.grad.zero_()
        m.sharding.parameters_changed()
        opt = N.AdamW(m.sharding, lr=1e-3, weight_decay=0.01)
        rows = []
        for _ in range(3):
            torch.manual_seed(7 + rank)
            r = N.train(ids, m, o, teacher_batch=N.TeacherBatch(hs, last), loss_mask=mask, optimizer=opt,
                        overlap=mode.endswith("overlap"))
            rows.append((r.metrics.loss.item(), r.update["grad_norm"], r.hidden.clone()))
        results[mode] = (rows, _digest(m))
    m.sharding.close_peer()
    a, b = results["peer_serial"], results["peer_overlap"]
    for ra, rb in zip(a[0], b[0]):
        assert ra[0] == rb[0] and ra[1] == rb[1] and torch.equal(ra[2], rb[2])
    for x, y in zip(a[1], b[1]):
        assert torch.equal(x, y), "peer serial vs overlap must be bitwise equal"
    a, b = results["nccl_serial"], results["nccl_overlap"]
    for x, y in zip(a[1], b[1]):
        assert torch.equal(x, y), "NCCL serial vs overlap must be bitwise equal"
    # peer vs NCCL: same math, different reduction order
    for ra, rb in zip(results["nccl_serial"][0], results["peer_serial"][0]):
        assert abs(ra[0] - rb[0]) <= 1e-3 * abs(ra[0])
    # NCCL's ring reduce-scatter rounds to bf16 after each of its world - 1 additions;
    # the peer reduce sums in fp32 and rounds once, so the gap grows with the ranks.
    tol = 1.5e-3 * world
    for x, y in zip(results["nccl_serial"][1], results["peer_serial"][1]):
        rel = ((x.float() - y.float()).norm() / x.float().norm().clamp_min(1e-12)).item()
        assert rel < tol, rel


@two_gpus
def test_schedules_bitwise_and_peer_matches_nccl():
    with tempfile.TemporaryDirectory() as d:
        run_ranks(2, _schedules, d)


@pytest.mark.skipif(ngpu < 4, reason="needs 4 GPUs")
def test_schedules_four_ranks():
    with tempfile.TemporaryDirectory() as d:
        run_ranks(4, _schedules, d)


@pytest.mark.skipif(ngpu < 1, reason="needs a GPU")
def test_peer_wait_times_out_without_hanging():
    """A wait on a flag that no rank ever sets returns with an error status."""
    from nanospec_b200.ops._ext import cuda_ops
    C = cuda_ops()
    C.clear_device_error()
    wid, _ = C.window_create(1 << 20, 0, 1)
    C.window_open(wid, C.window_ipc_handle(wid).view(1, -1))
    C.peer_wait(wid, 0, 5, 1, 2000)  # ~0.4 ms of polling, then give up
    torch.cuda.synchronize()
    assert C.device_error() == 2
    C.clear_device_error()
    # the context stays usable
    x = torch.ones(4, device="cuda")
    assert (x + 1).sum().item() == 8
    C.window_close(wid)


def _open_window(C, rank, world, nbytes):
    wid, _ = C.window_create(nbytes, rank, world)
    handles = [None] * world
    dist.all_gather_object(handles, C.window_ipc_handle(wid).tolist())
    C.window_open(wid, torch.tensor(handles, dtype=torch.uint8))
    return wid


def _fused_kernels(rank, world):
    """ag_gemm gathers the whole unit and multiplies by its W; gemm_rs + peer_push +
    peer_reduce_local produce the averaged gradient shard of every rank."""
    from nanospec_b200.ops._ext import cuda_ops
    C = cuda_ops()
    dev = torch.device("cuda", rank)
    Nw, K, M, T, pre, post = 384, 512, 300, 200, 1000, 2000
    total = pre + Nw * K + post
    ss = -(-total // (8 * world)) * 8
    full_n = ss * world
    g = torch.Generator(device=dev).manual_seed(1)
    unit = (torch.randn(full_n, device=dev, generator=g) * 0.05).bfloat16()
    param_off, slot_off = 4096, 4096 + ((ss * 2 + 255) // 256) * 256
    wid = _open_window(C, rank, world, slot_off + full_n * 2)
    C.window_view(wid, param_off, ss, torch.bfloat16).copy_(unit[rank * ss:(rank + 1) * ss])
    torch.cuda.synchronize()
    dist.barrier()

    # ---- all-gather -> GEMM, twice (the flags advance by epoch)
    W = unit[pre:pre + Nw * K].view(Nw, K)
    x = (torch.randn(M, K, device=dev, generator=g) * 0.5).bfloat16()
    flags = torch.zeros(-(-full_n // min(16384, ss)), device=dev, dtype=torch.int32)
    claim = torch.zeros(1, device=dev, dtype=torch.int32)
    ref = x.float() @ W.float().t()
    for epoch in (1, 2):
        resident = torch.full((full_n,), float("nan"), device=dev, dtype=torch.bfloat16)
        out = torch.empty(M, Nw, device=dev, dtype=torch.bfloat16)
        C.ag_gemm(wid, param_off, ss, resident, pre, Nw, K, x, out, flags, claim, epoch, 50_000_000)
        torch.cuda.synchronize()
        assert C.device_error() == 0
        assert torch.equal(resident, unit), "the gathered unit must equal every rank's shards"
        err = (out.float() - ref).abs().max().item()
        assert err <= 2e-2 * ref.abs().max().item(), err

    # ---- weight-gradient GEMM -> reduce-scatter (push), then the local sum
    gr = torch.Generator(device=dev).manual_seed(50 + rank)
    dy = (torch.randn(T, Nw, device=dev, generator=gr) * 0.5).bfloat16()
    xx = (torch.randn(T, K, device=dev, generator=gr) * 0.5).bfloat16()
    local = (torch.randn(full_n, device=dev, generator=gr) * 0.01).bfloat16()  # this rank's small grads
    C.gemm_rs(wid, slot_off, ss, pre, dy, xx)
    C.peer_push(wid, slot_off, ss, local, 0, pre)
    C.peer_push(wid, slot_off, ss, local, pre + Nw * K, full_n)
    C.peer_signal(wid, 0, 4, 1)
    C.peer_wait(wid, 0, 4, 1, 50_000_000)
    grad = torch.zeros(ss, device=dev, dtype=torch.bfloat16)
    C.peer_reduce_local(wid, slot_off, ss, grad)
    torch.cuda.synchronize()
    assert C.device_error() == 0
    # every rank's full contribution, to build the expected shard on the host
    mine = local.clone()
    mine[pre:pre + Nw * K] = (dy.float().t() @ xx.float()).bfloat16().reshape(-1)
    parts = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(parts, mine)
    acc = parts[0][rank * ss:(rank + 1) * ss].float()
    for q in range(1, world):
        acc = acc + parts[q][rank * ss:(rank + 1) * ss].float()
    want = (acc * (1.0 / world)).bfloat16().float()
    lo, hi = max(pre - rank * ss, 0), min(pre + Nw * K - rank * ss, ss)
    outside = torch.ones(ss, dtype=torch.bool, device=dev)
    if hi > lo:
        outside[lo:hi] = False
    # pushed copies are exact; GEMM outputs may differ from torch's fp32 GEMM by an ulp
    assert torch.equal(grad.float()[outside], want[outside])
    if hi > lo:
        d = (grad.float()[lo:hi] - want[lo:hi]).abs().max().item()
        assert d <= 2e-2 * want[lo:hi].abs().max().item(), d
    torch.cuda.synchronize()
    dist.barrier()
    C.window_close(wid)


def _fused_schedules(rank, world):
    """The fused paths (gather inside the context GEMM, reduce-scatter from the
    weight-gradient epilogues): serial and overlapped are bitwise equal, and they
    match the NCCL schedule as closely as the pull-based peer schedule does."""
    os.environ["NANOSPEC_PEER_GATHER"] = "fused"
    os.environ["NANOSPEC_PEER_REDUCE"] = "push"
    c, m = _model(rank, world)
    o = N.Objective(num_anchors=8)
    ids, hs, last, mask = _data(c, rank)
    init = [s.param.clone() for s in m.sharding]
    results = {}
    for mode in ("nccl_serial", "peer_serial", "peer_overlap"):
        if mode.startswith("peer"):
            m.sharding.enable_peer()
            sched = m.sharding._cache["peer"]
            assert sched.push and sched.fused_keys, "fused paths not selected"
        for s, p0 in zip(m.sharding, init):
            s.param.copy_(p0)
            s.master.copy_(s.param)
            s.m.zero_(), s.v.zero_(), s.grad.zero_()
        m.sharding.parameters_changed()
        opt = N.AdamW(m.sharding, lr=1e-3, weight_decay=0.01)
        rows = []
        for _ in range(3):
            torch.manual_seed(7 + rank)
            r = N.train(ids, m, o, teacher_batch=N.TeacherBatch(hs, last), loss_mask=mask, optimizer=opt,
                        overlap=mode.endswith("overlap"))
            rows.append((r.metrics.loss.item(), r.update["grad_norm"], r.hidden.clone()))
        results[mode] = (rows, _digest(m))
    from nanospec_b200.ops._ext import cuda_ops
    assert cuda_ops().device_error() == 0
    m.sharding.close_peer()
    a, b = results["peer_serial"], results["peer_overlap"]
    for ra, rb in zip(a[0], b[0]):
        assert ra[0] == rb[0] and ra[1] == rb[1] and torch.equal(ra[2], rb[2])
    for x, y in zip(a[1], b[1]):
        assert torch.equal(x, y), "fused serial vs overlap must be bitwise equal"
    for ra, rb in zip(results["nccl_serial"][0], results["peer_serial"][0]):
        assert abs(ra[0] - rb[0]) <= 1e-3 * abs(ra[0])
    tol = 1.5e-3 * world
    for x, y in zip(results["nccl_serial"][1], results["peer_serial"][1]):
        rel = ((x.float() - y.float()).norm() / x.float().norm().clamp_min(1e-12)).item()
        assert rel < tol, rel


@two_gpus
def test_fused_allgather_gemm_and_gemm_reduce_scatter_kernels():
    run_ranks(2, _fused_kernels)


@two_gpus
def test_fused_schedules_bitwise_and_match_nccl():
    run_ranks(2, _fused_schedules)


@pytest.mark.skipif(ngpu < 4, reason="needs 4 GPUs")
def test_fused_kernels_four_ranks():
    run_ranks(4, _fused_kernels)


def _handoff(rank, world, ckpt_path, train_gpus, fused=False):
    """Peer-store hand-off of the split layout over three steps (both slot sets and
    the release protocol): every trainer row equals the whole verifier run on that
    GPU. ``fused``: the stages run the fused FP8 path, whose add+norm epilogues store
    the captured residuals and the final normed hidden state into the trainers'
    slots."""
    from nanospec_b200.config import Topology
    from nanospec_b200.models.verifier import Checkpoint, QwenStage, stage_forward
    from nanospec_b200.ops._ext import cuda_ops
    from nanospec_b200.parallel.handoff import Teacher
    node = N.Node(train_gpus, topology=Topology(world=world, train_gpus=train_gpus))
    capture = (1, 3)
    teacher = Teacher(node, ckpt_path, capture)
    if teacher.stage is not None:
        assert teacher.stage.fused == fused
    full = QwenStage(Checkpoint(ckpt_path), 0, 4, device=node.device, first=True, last=True) if node.training else None
    for step in range(3):
        ids = torch.randint(0, 512, (train_gpus, 40), generator=torch.Generator().manual_seed(3 + step)).to(node.device)
        res = N.train(ids, verifier=teacher)
        assert getattr(teacher, "_handoff_window", None) is not None, "peer hand-off not in use"
        if node.training:
            x, cap = stage_forward(full, ids[rank:rank + 1], capture=capture)
            tb = res.teacher
            for got, layer in zip(tb.hidden_states, capture):
                assert torch.equal(got, cap[layer]), (step, layer)
            assert torch.equal(tb.last_hidden, x), step
        torch.cuda.synchronize()
    assert cuda_ops().device_error() == 0
    teacher._handoff_window.close()


@two_gpus
@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("train_gpus", [1, 2])
def test_verifier_handoff_by_peer_stores(train_gpus, fused):
    from nanospec_b200.models.verifier import tiny_hybrid_text_config, write_synthetic_checkpoint
    with tempfile.TemporaryDirectory() as d:
        if fused:  # the 27B head geometry at small width: FP8 projections, d_v = 128
            cfg = tiny_hybrid_text_config(hidden=256, vocab=512, heads=2, head_dim=128, ffn=512)
            cfg.update(linear_num_key_heads=1, linear_num_value_heads=2, linear_key_head_dim=128,
                       linear_value_head_dim=128, num_key_value_heads=1)
        else:
            cfg = tiny_hybrid_text_config()
            cfg["head_dim"] = 32  # the tcgen05 verifier attention takes head dims 32..256
        path = write_synthetic_checkpoint(os.path.join(d, "ck"), cfg, fp8=fused, seed=2)
        run_ranks(2, _handoff, str(path), train_gpus, fused)
