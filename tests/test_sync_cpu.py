"""Cross-process primitives: counting semaphore permits (and their release when a holder
dies), the append-only string journal and the one-shot ready condition."""

import os
import time
import uuid

import pytest

from flextensor_b200.shm.sync import MultiprocessCondition, SemaphoreLock, SharedMultiString


def _holder(name, slots, log, hold, start):
    s = SemaphoreLock(name, slots)
    start.wait(timeout=60)  # all holders compete at once, however slowly the processes spawned
    s.acquire(timeout=30)
    with open(log, "a") as f:
        f.write(f"in {time.time()}\n")
    time.sleep(hold)
    with open(log, "a") as f:
        f.write(f"out {time.time()}\n")
    s.release()
    s.close()


def _die_holding(name):
    s = SemaphoreLock(name, 1)
    s.acquire(timeout=10)
    os._exit(9)


def _writer(name, i):
    j = SharedMultiString(name)
    for k in range(5):
        j.append(f"w{i}-{k}")


def _waiter(name, q):
    c = MultiprocessCondition(name)
    q.put(c.wait_for_ready(timeout=20))


def _mp():
    import multiprocessing as mp

    return mp.get_context("spawn")


def test_semaphore_bounds_concurrency(tmp_path):
    name = f"ftsem{uuid.uuid4().hex[:8]}"
    log = str(tmp_path / "log")
    ctx = _mp()
    start = ctx.Barrier(4)
    ps = [ctx.Process(target=_holder, args=(name, 2, log, 1.0, start)) for _ in range(4)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(60)
    events = sorted((float(t), kind) for kind, t in (line.split() for line in open(log)))
    inside = peak = 0
    for _, kind in events:
        inside += 1 if kind == "in" else -1
        peak = max(peak, inside)
    assert peak == 2 and all(p.exitcode == 0 for p in ps)
    SemaphoreLock(name, 2).unlink()


def test_permit_of_dead_holder_is_released():
    name = f"ftsem{uuid.uuid4().hex[:8]}"
    p = _mp().Process(target=_die_holding, args=(name,))
    p.start()
    p.join(30)
    assert p.exitcode == 9
    s = SemaphoreLock(name, 1)
    s.acquire(timeout=5)  # would time out if the permit had leaked
    s.release()
    with pytest.raises(RuntimeError):
        s.release()
    s.unlink()


def test_journal_and_condition():
    name = f"ftjr{uuid.uuid4().hex[:8]}"
    ctx = _mp()
    ws = [ctx.Process(target=_writer, args=(name, i)) for i in range(3)]
    for w in ws:
        w.start()
    for w in ws:
        w.join(30)
    got = SharedMultiString(name).get_list()
    assert sorted(got) == sorted(f"w{i}-{k}" for i in range(3) for k in range(5))
    SharedMultiString(name).unlink()

    q = ctx.Queue()
    cname = f"ftcv{uuid.uuid4().hex[:8]}"
    waiter = ctx.Process(target=_waiter, args=(cname, q))
    waiter.start()
    time.sleep(0.5)
    cond = MultiprocessCondition(cname)
    cond.notify_ready("creator-ready")
    assert q.get(timeout=30) == ["creator-ready"]
    waiter.join(10)
    with pytest.raises(TimeoutError):
        MultiprocessCondition(f"ftcv{uuid.uuid4().hex[:8]}").wait_for_ready(timeout=0.2)
    cond.unlink()


def test_two_handles_in_one_process_contend():
    name = f"ftsem{uuid.uuid4().hex[:8]}"
    a, b = SemaphoreLock(name, 1), SemaphoreLock(name, 1)
    a.acquire(timeout=5)
    with pytest.raises(BlockingIOError):
        b.acquire(non_blocking=True)
    a.release()
    b.acquire(non_blocking=True)
    b.release()
    a.unlink()


def test_closing_one_handle_keeps_the_others_permit():
    name = f"ftsem{uuid.uuid4().hex[:8]}"
    holder, other, probe = SemaphoreLock(name, 1), SemaphoreLock(name, 1), SemaphoreLock(name, 1)
    holder.acquire(timeout=5)
    other.close()  # closing a handle that holds nothing must not free holder's permit
    with pytest.raises(BlockingIOError):
        probe.acquire(non_blocking=True)
    holder.close()  # frees it
    probe.acquire(non_blocking=True)
    probe.unlink()


def test_threads_sharing_a_handle_are_bounded():
    import threading

    name = f"ftsem{uuid.uuid4().hex[:8]}"
    s = SemaphoreLock(name, 2)
    lock = threading.Lock()
    state = {"inside": 0, "peak": 0}
    go = threading.Barrier(6)

    def worker():
        go.wait(timeout=10)
        s.acquire(timeout=30)
        with lock:
            state["inside"] += 1
            state["peak"] = max(state["peak"], state["inside"])
        time.sleep(0.05)
        with lock:
            state["inside"] -= 1
        s.release()

    ts = [threading.Thread(target=worker) for _ in range(6)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(60)
    assert state["peak"] == 2 and s.held == 0
    s.unlink()
