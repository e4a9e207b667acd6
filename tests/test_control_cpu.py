"""Failure handling of the bounded control plane with real Gloo ranks on the CPU (no GPU):
a follower that never joins a broadcast trips the leader's watchdog; a rank that dies before
the outcome exchange poisons the survivors; a failed request poisons every member."""

import os
import socket
import time

import pytest


def _exit(q, code=0):
    q.close()
    q.join_thread()  # flush queued results before the hard exit
    os._exit(code)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout=4.0):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout))
    from flextensor_b200.parallel.control import ControlPlane

    return ControlPlane(timeout_seconds=timeout)


def _healthy(rank, world, port, q):
    cp = _init(rank, world, port)
    cmd = cp.broadcast_object({"prompt": "cat", "steps": 3} if rank == 0 else None)
    ok = cp.request_ok({"ok": True, "rank": rank})
    q.put((rank, cmd, ok, cp.poisoned))
    cp.close()


def _stalled_follower(rank, world, port, q):
    cp = _init(rank, world, port, timeout=60.0)   # collective timeout far above the watchdog
    if rank == 0:
        q.put(("leader-start", time.time()))
        time.sleep(0.5)                           # let the queue feeder flush before the watchdog exit
        cp.broadcast_object({"cmd": 1}, timeout_seconds=2.0)   # watchdog ends this process (code 3)
        q.put(("leader-returned", None))
    else:
        time.sleep(30)                            # never joins the broadcast
    _exit(q)


def _dead_rank(rank, world, port, q):
    cp = _init(rank, world, port, timeout=3.0)
    if rank == world - 1:
        os._exit(7)                               # dies before the outcome exchange
    try:
        cp.exchange_status({"ok": True})
        q.put((rank, "exchange returned"))
    except Exception as e:                         # noqa: BLE001
        q.put((rank, type(e).__name__, cp.poisoned))
        try:
            cp.broadcast_object(1)
        except Exception as e2:                    # noqa: BLE001
            q.put((rank, "after-poison", type(e2).__name__))
    _exit(q)


def _failed_request(rank, world, port, q):
    cp = _init(rank, world, port)
    ok = cp.request_ok({"ok": rank != 1, "rank": rank})
    q.put((rank, ok, cp.poisoned))
    _exit(q)


def _spawn(fn, world, timeout=60):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    deadline = time.time() + timeout
    for p in ps:
        p.join(max(1.0, deadline - time.time()))
    for p in ps:
        if p.is_alive():
            p.kill()
            p.join(5)
    out = []
    while not q.empty():
        out.append(q.get())
    return ps, out


def test_healthy_replica():
    ps, out = _spawn(_healthy, 3)
    assert sorted(o[0] for o in out) == [0, 1, 2]
    for rank, cmd, ok, poisoned in out:
        assert cmd == {"prompt": "cat", "steps": 3} and ok and not poisoned


def test_broadcast_watchdog_ends_stalled_leader():
    ps, out = _spawn(_stalled_follower, 2, timeout=40)
    assert ps[0].exitcode == 3, f"leader exit code {ps[0].exitcode}"
    assert ("leader-returned", None) not in out


@pytest.mark.parametrize("world", [2, 3])
def test_dead_rank_poisons_survivors(world):
    ps, out = _spawn(_dead_rank, world, timeout=60)
    assert ps[-1].exitcode == 7
    survivors = [o for o in out if len(o) == 3 and o[1] == "ReplicaFatalError"]
    assert len(survivors) == world - 1 and all(o[2] for o in survivors), out
    refused = [o for o in out if o[1] == "after-poison"]
    assert len(refused) == world - 1 and all(o[2] == "ReplicaFatalError" for o in refused)


def test_failed_request_poisons_every_member():
    ps, out = _spawn(_failed_request, 3)
    assert len(out) == 3 and all(not ok and poisoned for _, ok, poisoned in out)
