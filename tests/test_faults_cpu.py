"""Failure paths, injected on the host (no GPU, nothing faults or hangs a device).

- a non-finite gradient skips the optimizer update and zeroes the gradients;
- incomplete / corrupt / mismatched checkpoints are refused with ValueError;
- a rank that raises inside a step makes the other rank's next collective fail
  with an error (finite process-group timeout) instead of waiting for ever.

Reference behaviour: nanospec/shard.py:336-338 (skip on a non-finite norm),
nanospec/checkpoint.py (tmp+rename, metadata written last, mismatch errors).
"""

import json
import os
import socket
import tempfile
import time
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import nanospec_b200 as N
from nanospec_b200 import checkpoint


def _model(dtype=torch.float32):
    c = N.DraftConfig.load(N.config_path("tiny"))
    g = torch.Generator().manual_seed(43)
    emb = (torch.randn(c.vocab_size, c.hidden_size, generator=g) * 0.1).to(dtype)
    head = (torch.randn(c.vocab_size, c.hidden_size, generator=g) * 0.1).to(dtype)
    return c, N.DSpark(c, N.initialize(c, 42, dtype), emb, head, device="cpu", dtype=dtype)


def _step(c, m, opt=None):
    g = torch.Generator().manual_seed(9)
    ids = torch.randint(0, c.vocab_size, (1, 48), generator=g)
    hs = [torch.randn(1, 48, c.hidden_size, generator=g) for _ in range(c.num_target_layers)]
    last = torch.randn(1, 48, c.hidden_size, generator=g)
    torch.manual_seed(1)
    return N.train(ids, m, N.Objective(num_anchors=4), teacher_batch=N.TeacherBatch(hs, last), optimizer=opt)


def test_nonfinite_gradient_skips_update():
    c, m = _model()
    opt = N.AdamW(m.sharding, lr=1e-3)
    r = _step(c, m)
    masters = [s.master.clone() for s in m.sharding]
    first = next(iter(m.sharding))
    first.grad[3] = float("nan")
    u = N.adamw_step(opt, r.metrics.denominator)
    assert not u["updated"]
    assert opt.steps == 0
    for s, m0 in zip(m.sharding, masters):
        assert torch.equal(s.master, m0)
        assert s.grad.abs().max().item() == 0
    # the next finite step updates normally
    r = _step(c, m)
    assert N.adamw_step(opt, r.metrics.denominator)["updated"] and opt.steps == 1


@pytest.fixture
def saved():
    c, m = _model()
    opt = N.AdamW(m.sharding, lr=1e-3)
    _step(c, m, opt)
    with tempfile.TemporaryDirectory() as d:
        path = checkpoint.save(os.path.join(d, "ck"), m, opt, N.Objective(num_anchors=4), 1)
        yield path


def _restore(path, dtype=torch.float32, objective=None):
    c, m = _model(dtype)
    return checkpoint.restore(path, m, N.AdamW(m.sharding, lr=1e-3), objective or N.Objective(num_anchors=4))


def test_checkpoint_roundtrip_ok(saved):
    assert _restore(saved) == 1


def test_checkpoint_without_metadata_is_refused(saved):
    os.remove(os.path.join(saved, "metadata.json"))
    with pytest.raises(ValueError, match="metadata"):
        _restore(saved)
    assert checkpoint.latest(os.path.dirname(saved) + "/ck") is None


def test_truncated_rank_file_is_refused(saved):
    f = os.path.join(saved, "rank-0.pt")
    data = open(f, "rb").read()
    with open(f, "wb") as out:
        out.write(data[: len(data) // 3])
    with pytest.raises(ValueError, match="Unreadable"):
        _restore(saved)


def test_mismatched_dtype_objective_or_config_is_refused(saved):
    with pytest.raises(checkpoint.CheckpointMismatch, match="dtype: checkpoint 'torch.float32', run 'torch.bfloat16'"):
        _restore(saved, dtype=torch.bfloat16)
    with pytest.raises(checkpoint.CheckpointMismatch, match="objective.num_anchors: checkpoint 4, run 5"):
        _restore(saved, objective=N.Objective(num_anchors=5))
    meta_path = os.path.join(saved, "metadata.json")
    meta = json.load(open(meta_path))
    meta["config"]["hidden_size"] += 1
    meta["target_revision"] = "other"
    json.dump(meta, open(meta_path, "w"))
    with pytest.raises(ValueError) as e:  # every mismatched field is listed
        _restore(saved)
    assert "config.hidden_size: checkpoint 65, run 64" in str(e.value)
    assert "target_revision: checkpoint 'other'" in str(e.value)


def test_async_and_periodic_saves_roundtrip():
    c, m = _model()
    opt = N.AdamW(m.sharding, lr=1e-3)
    o = N.Objective(num_anchors=4)
    with tempfile.TemporaryDirectory() as d:
        prefix = os.path.join(d, "run")
        per = checkpoint.Periodic(prefix, m, opt, o, every=2, keep=2)
        masters = {}
        for step in range(1, 7):
            r = _step(c, m, opt)
            assert bool(r.update["updated"])
            per.step(step)
            masters[step] = [s.master.clone() for s in m.sharding]
        per.close()
        import glob
        gens = sorted(glob.glob(prefix + "-step*"))
        assert len(gens) == 2  # steps 4 and 6 kept, step 2 pruned
        newest = checkpoint.latest(prefix)
        assert json.load(open(os.path.join(newest, "metadata.json")))["step"] == 6
        c2, m2 = _model()
        opt2 = N.AdamW(m2.sharding, lr=1e-3)
        assert checkpoint.restore(newest, m2, opt2, o) == 6
        assert opt2.steps == opt.steps
        for a, b in zip(m2.sharding, masters[6]):
            assert torch.equal(a.master, b)


# ---------------------------------------------------------------------------- a rank dies
def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.set_num_threads(1)
    t0 = time.time()
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=8))
        c = N.DraftConfig.load(N.config_path("tiny"))
        m = N.DSpark(c, N.initialize(c, 42, torch.float32), torch.randn(c.vocab_size, c.hidden_size) * 0.1,
                     torch.randn(c.vocab_size, c.hidden_size) * 0.1, device="cpu", dtype=torch.float32,
                     group=dist.group.WORLD, world_size=world, rank=rank)
        if rank == 1:
            raise RuntimeError("injected failure inside the step")
        _step(c, m, N.AdamW(m.sharding, lr=1e-3))  # needs rank 1 in its first all-gather
        q.put((rank, "finished", time.time() - t0))
    except BaseException as exc:  # noqa: BLE001 - reported to the parent
        q.put((rank, type(exc).__name__ + ": " + str(exc).splitlines()[0] if str(exc) else type(exc).__name__,
               time.time() - t0))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001
                pass


def test_failed_rank_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung after its peer failed"
    reports = {}
    while not q.empty():
        rank, what, secs = q.get()
        reports[rank] = (what, secs)
    assert "injected failure" in reports[1][0]
    assert reports[0][0] != "finished", reports  # the surviving rank's collective failed
    assert reports[0][1] < 100


# ---------------------------------------------------------------------------- device wait timeouts
class _FlakyWord:
    """A host error word that a 'kernel' sets during one phase of the step.

    ``lag=True`` makes every snapshot look still in flight until ``land()`` is
    called, like a device copy that the host has not waited for.
    """

    def __init__(self, phase, lag=False):
        self.word = torch.zeros(1, dtype=torch.int32)
        self.phase = phase
        self.resets = 0
        self.lag = lag
        self.landed = not lag

    def land(self):
        self.landed = True

    def monitor(self):
        from nanospec_b200.utils.health import ErrorMonitor
        mon = ErrorMonitor("cpu", word=self.word, reset=self._reset)
        snap = mon.snapshot
        flaky = self

        class _Later:
            def query(self):
                return flaky.landed

            def synchronize(self):
                flaky.landed = True

        def snapshot(tag):
            if tag == self.phase:
                self.word.fill_(2)  # a peer flag wait gave up during this phase
            snap(tag)
            if self.lag:
                slot, _, t = mon.pending[-1]
                mon.pending[-1] = (slot, _Later(), t)
        mon.snapshot = snapshot
        return mon

    def _reset(self):
        self.resets += 1
        self.word.zero_()


@pytest.mark.parametrize("lag", [False, True])
def test_device_wait_timeout_raises_on_host(monkeypatch, lag):
    """A bounded device wait that gave up (code in the error word) becomes a Python
    exception naming the phase: in the same call when the snapshot has landed (a
    synchronous optimizer waited), else at the start of the next call."""
    from nanospec_b200 import engine
    from nanospec_b200.utils.health import DeviceWaitTimeout
    c, m = _model()
    opt = N.AdamW(m.sharding, lr=1e-3)
    flaky = _FlakyWord("draft forward/backward", lag=lag)
    mon = flaky.monitor()
    monkeypatch.setattr(engine, "_monitor", lambda ids: mon)
    if not lag:
        with pytest.raises(DeviceWaitTimeout, match="peer-memory flag wait.*draft forward/backward"):
            _step(c, m, opt)
    else:
        _step(c, m, opt)  # the snapshots are still "in flight": no wait, no raise
        flaky.land()
        with pytest.raises(DeviceWaitTimeout, match="draft forward/backward"):
            _step(c, m, opt)
    assert flaky.resets == 1 and int(flaky.word) == 0
    flaky.phase, flaky.lag, flaky.landed = None, False, True  # the next step is clean again
    r = _step(c, m, opt)
    assert bool(r.update["updated"])


def test_debug_mode_poison_leaves_results_unchanged(monkeypatch):
    """NANOSPEC_DEBUG=1 fills every gradient shard the backward is about to overwrite
    with NaN; if any element were not rewritten the update would turn non-finite. The
    results must equal the normal mode bitwise."""
    def run():
        c, m = _model()
        opt = N.AdamW(m.sharding, lr=1e-3, lazy_zero=True)
        out = []
        for _ in range(3):
            r = _step(c, m, opt)
            out.append((float(r.metrics.loss), bool(r.update["updated"]), r.update["grad_norm"]))
        return out, [s.master.clone() for s in m.sharding]
    monkeypatch.setenv("NANOSPEC_DEBUG", "0")
    ref, ref_m = run()
    monkeypatch.setenv("NANOSPEC_DEBUG", "1")
    got, got_m = run()
    assert got == ref and all(u for _, u, _ in got)
    for a, b in zip(ref_m, got_m):
        assert torch.equal(a, b)
