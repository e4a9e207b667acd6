"""Pipeline parallelism on the CPU: the stage split, the micro-batch schedule (receives posted
ahead of compute, sends overlapping the next micro-batch, outputs returned to the first stage)
over an in-memory transport with one thread per stage, and the Wan DiT split over 2 and 3 gloo
ranks against the unsplit model, resident and with each stage's blocks streamed by its own
offload manager."""

import itertools
import os
import queue
import random
import socket
import threading

import pytest
import torch

from flextensor_b200.parallel.pp import PipelineStage, split_stages


def _brute(costs, k):
    n = len(costs)
    best = None
    for cuts in itertools.combinations(range(1, n), k - 1):
        b = (0,) + cuts + (n,)
        v = max(sum(costs[b[i]:b[i + 1]]) for i in range(k))
        best = v if best is None else min(best, v)
    return best


@pytest.mark.parametrize("seed", range(30))
def test_split_stages_is_optimal_and_contiguous(seed):
    rnd = random.Random(seed)
    n = rnd.randint(1, 9)
    k = rnd.randint(1, n)
    costs = [rnd.choice([0, 1, 2, 5, 7.5, 10]) for _ in range(n)]
    bounds = split_stages(costs, k)
    assert len(bounds) == k and bounds[0][0] == 0 and bounds[-1][1] == n
    assert all(a < b for a, b in bounds) and all(bounds[i][1] == bounds[i + 1][0] for i in range(k - 1))
    assert max(sum(costs[a:b]) for a, b in bounds) == _brute(costs, k)


def test_split_stages_rejects_impossible_splits():
    with pytest.raises(ValueError):
        split_stages([1.0, 2.0], 3)
    with pytest.raises(ValueError):
        split_stages([1.0, -1.0], 1)
    assert split_stages([4, 1, 1, 1, 1], 2) == [(0, 1), (1, 5)]


class _Mailbox:
    """In-memory transport: one FIFO per (src, dst, channel); the log records every post, wait
    and compute in the order the stage threads issue them."""

    def __init__(self, log):
        self.q = {}
        self.lock = threading.Lock()
        self.log = log

    def _chan(self, key):
        with self.lock:
            return self.q.setdefault(key, queue.Queue())

    def send(self, t, src, dst, channel):
        self.log.append(("send", src, dst, channel))
        self._chan((src, dst, channel)).put(t.clone())

        class H:
            def wait(self_inner):
                return None

        return H()

    def recv(self, t, src, dst, channel):
        self.log.append(("post_recv", src, dst, channel))
        ch = self._chan((src, dst, channel))

        class H:
            def wait(self_inner):
                t.copy_(ch.get(timeout=30))

        return H()


def _run_threads(n_stages, n_micro, depth, back):
    log = []
    box = _Mailbox(log)
    results = {}
    weights = [float(s + 2) for s in range(n_stages)]
    inputs = [torch.full((2, 3), float(m + 1)) for m in range(n_micro)]

    def make_fn(s):
        def fn(x, m):
            log.append(("compute", s, m))
            return x * weights[s] + s

        return fn

    def body(s):
        st = PipelineStage(make_fn(s), s, n_stages, box, depth)
        results[s] = st.run(n_micro, inputs=inputs if s == 0 else None,
                            recv_spec=lambda m: ((2, 3), torch.float32),
                            out_spec=(lambda m: ((2, 3), torch.float32)) if back else None)

    ts = [threading.Thread(target=body, args=(s,)) for s in range(n_stages)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(60)
        assert not t.is_alive(), "pipeline deadlocked"
    want = []
    for x in inputs:
        for s in range(n_stages):
            x = x * weights[s] + s
        want.append(x)
    return log, results, want


@pytest.mark.parametrize("n_stages,n_micro,depth", [(1, 3, 2), (2, 1, 2), (2, 5, 1), (3, 6, 2), (4, 7, 3)])
@pytest.mark.parametrize("back", [True, False])
def test_schedule_results_and_overlap(n_stages, n_micro, depth, back):
    log, results, want = _run_threads(n_stages, n_micro, depth, back)
    last = n_stages - 1
    for w, got in zip(want, results[last]):
        assert torch.equal(w, got)
    if n_stages > 1:
        assert all(results[s] is None for s in range(1, last))
        if back:
            for w, got in zip(want, results[0]):
                assert torch.equal(w, got)
        else:
            assert results[0] is None
    for s in range(1, n_stages):  # the receive of m + depth is posted before m is computed
        posts = [i for i, e in enumerate(log) if e == ("post_recv", s - 1, s, "fwd")]
        computes = [i for i, e in enumerate(log) if e[0] == "compute" and e[1] == s]
        assert len(posts) == n_micro and len(computes) == n_micro
        for m in range(n_micro - depth):
            assert posts[m + depth] < computes[m]
        assert posts[min(depth, n_micro) - 1] < computes[0]  # the first `depth` before any compute
    if back and n_stages > 1:  # outputs head back to stage 0 as they are computed
        sends = [i for i, e in enumerate(log) if e == ("send", last, 0, "back")]
        computes = [i for i, e in enumerate(log) if e[0] == "compute" and e[1] == last]
        posts = [i for i, e in enumerate(log) if e == ("post_recv", last, 0, "back")]
        assert len(sends) == len(posts) == n_micro
        first_compute = min(i for i, e in enumerate(log) if e == ("compute", 0, 0))
        assert max(posts) < first_compute
        for m in range(n_micro - 1):
            assert computes[m] < sends[m] < computes[m + 1]
    for s in range(n_stages - 1):  # each output leaves before the next micro-batch is computed
        sends = [i for i, e in enumerate(log) if e == ("send", s, s + 1, "fwd")]
        computes = [i for i, e in enumerate(log) if e[0] == "compute" and e[1] == s]
        for m in range(n_micro - 1):
            assert computes[m] < sends[m] < computes[m + 1]


def test_stage_argument_checks():
    with pytest.raises(ValueError):
        PipelineStage(lambda x, m: x, 2, 2)
    with pytest.raises(ValueError):
        PipelineStage(lambda x, m: x, 0, 2)  # several stages, no transport
    st = PipelineStage(lambda x, m: x, 0, 1)
    with pytest.raises(ValueError):
        st.run(2, inputs=[torch.zeros(1)])
    with pytest.raises(ValueError):
        PipelineStage(lambda x, m: x, 1, 2, _Mailbox([])).run(1)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(cfg, n_micro):
    g = torch.Generator().manual_seed(5)
    lat = [torch.randn(1 + (i % 2), cfg.in_channels, 2, 8, 8, generator=g) for i in range(n_micro)]
    ts = [torch.full((lat[i].shape[0],), 100.0 * (i + 1)) for i in range(n_micro)]
    ctx = [torch.randn(lat[i].shape[0], 5, cfg.text_dim, generator=g) for i in range(n_micro)]
    return lat, ts, ctx


def _wan_pp_worker(rank, world, port, q, offload=False):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from flextensor_b200.models.wan import WanDiT, init_wan_params_, tiny_config
        from flextensor_b200.models.wan_pp import WanPipelineParallel

        cfg = tiny_config(num_layers=5)
        m = WanDiT(cfg, impl="torch")
        init_wan_params_(m, seed=3)
        pp = WanPipelineParallel(m, depth=2)
        lat, ts, ctx = _inputs(cfg, 4)
        if rank not in (0, world - 1):
            lat = [torch.empty(x.shape, device="meta") for x in lat]
        runs = 1
        if offload:
            import flextensor_b200 as ft
            from flextensor_b200.planner import NthLayerStrategy

            pp.offload(ft.OffloadConfig(pinned_memory=False, include_patterns=["blocks.*"], profiling_iters=1,
                                        num_blocks=2, min_blocks=2,
                                        load_strategy=NthLayerStrategy(1, threshold_mb=0.0, n_blocks=2, cyclic=True)))
            runs = 3  # 4 micro-batches a run: discovery, profiling and inference all pass
        for _ in range(runs):
            outs = pp(lat, ts, ctx)
            if outs is not None:
                outs = [o.numpy().copy() for o in outs]
        extra = None
        if offload:
            om = ft.get_offload_manager(f"wan_pp{rank}")
            extra = (om.phase.value, len(om.get_tensor_manager().loader.plan.host_blocks))
            ft.release(f"wan_pp{rank}")
        q.put((rank, pp.bounds, len(m.blocks), outs, extra))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,offload", [(2, False), (3, False), (2, True)])
def test_wan_pipeline_matches_unsplit_model(world, offload):
    """With ``offload``, each stage streams its blocks under its own manager (``wan_pp<r>``)
    through discovery, profiling and inference; the outputs stay bit-identical."""
    import torch.multiprocessing as mp

    from flextensor_b200.models.wan import WanDiT, init_wan_params_, tiny_config

    cfg = tiny_config(num_layers=5)
    ref = WanDiT(cfg, impl="torch")
    init_wan_params_(ref, seed=3)
    lat, ts, ctx = _inputs(cfg, 4)
    with torch.no_grad():
        want = [ref(lat[i], ts[i], ctx[i]) for i in range(4)]
    ctx_mp = mp.get_context("spawn")
    q = ctx_mp.Queue()
    port = _free_port()
    ps = [ctx_mp.Process(target=_wan_pp_worker, args=(r, world, port, q, offload)) for r in range(world)]
    for p in ps:
        p.start()
    res = sorted((q.get(timeout=180) for _ in ps), key=lambda t: t[0])
    for p in ps:
        p.join(30)
    bounds = res[0][1]
    assert [b - a for a, b in bounds] == [r[2] for r in res] and sum(r[2] for r in res) == 5
    for rank, _, _, outs, extra in res:
        if offload:
            assert extra[0] == "inference" and extra[1] > 0, (rank, extra)
        if rank in (0, world - 1):
            assert len(outs) == 4
            for w, o in zip(want, outs):
                torch.testing.assert_close(torch.from_numpy(o), w, rtol=0, atol=0)
        else:
            assert outs is None
