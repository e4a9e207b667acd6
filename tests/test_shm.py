"""Shared-memory host store: segments, coordinator protocol v4, FTTS store, shared sessions.

Multi-process cases run real processes on one host. Failures are injected on
the host only: a creator that raises, a creator killed mid-initialisation,
a follower whose wait runs out.
"""

import multiprocessing as mp
import os
import signal
import time
import uuid

import pytest
import torch
from torch import nn

from flextensor_b200.shm import coordinator as C
from flextensor_b200.shm.segment import ShmSegment, shm_exists
from flextensor_b200.shm.tensor_store import SharedTensorStore

CTX = mp.get_context("spawn")
LEASE = 1.0


def ns():
    return f"fttest_{uuid.uuid4().hex[:10]}"


def test_segment_roundtrip():
    n = ns()
    a = ShmSegment.create(n + "_x", 4096)
    a.tensor()[:4] = torch.tensor([1, 2, 3, 4], dtype=torch.uint8)
    b = ShmSegment.attach(n + "_x")
    assert b.tensor()[:4].tolist() == [1, 2, 3, 4]
    with pytest.raises(FileExistsError):
        ShmSegment.create(n + "_x", 10)
    a.close(), b.close(), a.unlink()
    assert not shm_exists(n + "_x")


def test_header_layout():
    buf = bytearray(C.COORD_HEADER_SIZE)
    assert C.COORD_HEADER_SIZE == 4 + 64 + 4 + 8 + 4 + 4 + 160
    h = C.CoordBlockHeader("1.2.3", 4, 77, C.CoordinatorState.FAILED, "boom é")
    h.write_to(buf)
    g = C.CoordBlockHeader.read_from(buf)
    assert (g.flextensor_version, g.protocol_version, g.creator_pid, g.state, g.failure_message) == (
        "1.2.3", 4, 77, C.CoordinatorState.FAILED, "boom é")
    with pytest.raises(RuntimeError):
        g.validate("9.9", 4)


def _creator(name, q, mode, done=None):
    from flextensor_b200.core.state import TensorManagerState  # noqa: F401
    from flextensor_b200.shm import coordinator as C2

    c = C2.ShmCoordinator(name, lease_s=LEASE)
    q.put(("role", c.is_creator))
    if mode == "ready":
        c.write_profile(b"\x00\x00\x00\x02{}")
        c.notify_ready()
        done.wait(60)  # a creator stays alive while followers attach
        c.close()
    elif mode == "fail":
        c.mark_failed("factory raised ValueError: bad checkpoint")
        done.wait(60)  # waiting followers must see FAILED (late arrivals start a new generation)
        c.close(unlink_if_last=False)
    elif mode == "hang":
        time.sleep(60)  # killed by the test while INITIALIZING


def _follower(name, q, timeout):
    from flextensor_b200.shm import coordinator as C2

    try:
        c = C2.ShmCoordinator(name, lease_s=LEASE)
        q.put(("role", c.is_creator))
        c.wait_for_ready(timeout)
        q.put(("ready", None))
    except Exception as e:  # noqa: BLE001
        q.put(("error", type(e).__name__))


_LAST: dict = {}


def _run(mode, follower_timeout=20.0, kill_after=None):
    name = ns()
    q = CTX.Queue()
    done = CTX.Event()
    cr = CTX.Process(target=_creator, args=(name, q, mode, done))
    cr.start()
    assert q.get(timeout=60) == ("role", True)
    fo = CTX.Process(target=_follower, args=(name, q, follower_timeout))
    fo.start()
    got = [q.get(timeout=60)]  # follower joined (and is waiting) before any fault is injected
    t_kill = None
    if kill_after is not None:
        time.sleep(kill_after)
        os.kill(cr.pid, signal.SIGKILL)
        t_kill = time.monotonic()
    got.append(q.get(timeout=60))
    if t_kill is not None:
        _LAST["detect_s"] = time.monotonic() - t_kill  # kill -> follower's verdict arrived
    done.set()
    fo.join(30)
    cr.join(30)
    if cr.is_alive():
        cr.kill()
    C.cleanup_namespace(name)
    return got


def test_creator_follower_ready():
    assert _run("ready") == [("role", False), ("ready", None)]


def test_creator_failed_is_reported():
    assert _run("fail") == [("role", False), ("error", "ShmCreatorFailedError")]


def test_creator_death_detected():
    got = _run("hang", follower_timeout=30.0, kill_after=0.5)
    assert got == [("role", False), ("error", "ShmCreatorDiedError")]
    # measured from the kill, so process start-up under load does not count: a lapsed 1 s
    # heartbeat lease is noticed well inside the follower's 30 s wait
    assert _LAST["detect_s"] < 15


def test_follower_timeout():
    name = ns()
    q = CTX.Queue()
    cr = CTX.Process(target=_creator, args=(name, q, "hang"))
    cr.start()
    assert q.get(timeout=60) == ("role", True)
    fo = CTX.Process(target=_follower, args=(name, q, 1.0))
    fo.start()
    got = [q.get(timeout=60), q.get(timeout=60)]
    cr.kill()
    fo.join(30)
    cr.join(30)
    C.cleanup_namespace(name)
    assert got == [("role", False), ("error", "TimeoutError")]


class Tiny(nn.Module):
    def __init__(self):
        super().__init__()
        self.a = nn.Linear(8, 8)
        self.b = nn.Linear(8, 8)
        self.b.weight = self.a.weight  # alias
        self.register_buffer("stats", torch.arange(5, dtype=torch.float32))
        self.register_buffer("scratch", torch.zeros(3), persistent=False)


def test_tensor_store_roundtrip():
    n = ns()
    torch.manual_seed(0)
    src = Tiny()
    st = SharedTensorStore.create_from_model(n, src, ["a.weight", "a.bias"])
    hdr = bytes(st.seg.buf[:4])
    assert hdr == b"FTTS"
    with torch.device("meta"):
        dst = Tiny()
    at = SharedTensorStore.attach(n)
    at.materialize_into(dst, "cpu")
    assert torch.equal(dst.a.weight, src.a.weight) and dst.b.weight is dst.a.weight
    assert torch.equal(dst.stats, src.stats) and "scratch" not in dst.state_dict()
    at.close(), st.close()
    C.cleanup_namespace(n)


def _session_worker(base, q, profile_dir, seed_model, barrier):
    import torch as T

    import flextensor_b200 as ft
    from flextensor_b200.planner import NthLayerStrategy

    class MLP(T.nn.Module):
        def __init__(self):
            super().__init__()
            self.fc1 = T.nn.Linear(64, 128)
            self.fc2 = T.nn.Linear(128, 64)

        def forward(self, x):
            return self.fc2(T.relu(self.fc1(x)))

    def creator():
        T.manual_seed(seed_model)
        return MLP()

    def follower():
        with T.device("meta"):
            return MLP()

    cfg = ft.OffloadConfig(pinned_memory=False, include_patterns=["fc1", "fc2"], num_blocks=2, min_blocks=2,
                           load_strategy=NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2, cyclic=True))
    s = ft.SharedOffloadSession(base, wait_timeout=60)
    m = s.offload_from_profile(profile_dir, config=cfg, creator_model_factory=creator,
                               follower_model_factory=follower)
    x = T.ones(4, 64)
    with T.no_grad():
        y = m(x)
    q.put(y.sum().item())
    barrier.wait(120)  # every worker stays attached until all have run
    s.close()


def test_shared_session_creator_and_follower(tmp_path):
    import flextensor_b200 as ft
    from flextensor_b200.planner import NthLayerStrategy

    class MLP(nn.Module):
        def __init__(self):
            super().__init__()
            self.fc1 = nn.Linear(64, 128)
            self.fc2 = nn.Linear(128, 64)

        def forward(self, x):
            return self.fc2(torch.relu(self.fc1(x)))

    torch.manual_seed(3)
    m = MLP()
    want = m(torch.ones(4, 64)).sum().item()
    cfg = ft.OffloadConfig(pinned_memory=False, include_patterns=["fc1", "fc2"], num_blocks=2, min_blocks=2,
                           profiling_iters=1, load_strategy=NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2,
                                                                             cyclic=True))
    mm = ft.offload(m, cfg)
    for _ in range(ft.get_offload_manager().iters_before_inference):
        mm(torch.ones(4, 64))
    ft.save_profile(str(tmp_path))
    ft.release()
    base = ns()
    q = CTX.Queue()
    bar = CTX.Barrier(2)
    ps = [CTX.Process(target=_session_worker, args=(base, q, str(tmp_path), 3, bar)) for _ in range(2)]
    for p in ps:
        p.start()
    got = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(60)
    assert all(abs(g - want) < 1e-4 for g in got), (got, want)
