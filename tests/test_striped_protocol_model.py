"""CPU model of striped host streaming between ranks (``TransferEngine::submit_striped`` in
``ops/csrc/runtime.cpp``, the publish / gather / wait-acks kernels of ``ops/csrc/p2p.cu``), run
under random interleavings. Every rank runs the same plan: use i of the weight ring goes to slot
``i % K``. Per rank there are two streams:

* copy stream, per use i (slot s, that slot's epoch e): wait until this rank's compute released
  the slot's previous use; if e > 1 wait until every peer acked epoch e - 1 of the slot; copy
  this rank's stripe host->device in pieces; publish e to every rank; gather: for each peer (any
  order) wait for its flag >= e and pull its stripe in pieces; the last CTA out acks every peer;
  record ready(i);
* compute stream, per use i: wait ready(i), read the whole slot, release the slot.

The model asserts that every pulled piece and every piece compute reads belong to use i, and
that nothing deadlocks. With a ring of two or more slots the flag chain alone already orders
reuse (a rank copies into slot s again only after gathering a later use, which needs every
peer's publish of it, which each peer's copy stream issues after its gather of s); the acks are
what a one-slot ring and the heap teardown rely on. The model fails a one-slot ring without the
ack wait, a publish before the stripe has landed, and an ack sent before the pull ends.
"""

import random

import pytest

PIECES = 2


def run(world, uses, n_slots, seed, wait_acks=True, publish_after_copy=True, ack_after_pull=True):
    rnd = random.Random(seed)
    # mem[r][s][q]: pieces of rank q's stripe held in rank r's slot s (value = the use they belong to)
    mem = [[[[None] * PIECES for _ in range(world)] for _ in range(n_slots)] for _ in range(world)]
    flags = [[[0] * n_slots for _ in range(world)] for _ in range(world)]  # flags[r][q][s]
    acks = [[[0] * n_slots for _ in range(world)] for _ in range(world)]   # acks[r][q][s]
    ready = [[False] * uses for _ in range(world)]
    released = [[False] * uses for _ in range(world)]

    def copy_stream(r):
        epochs = [0] * n_slots
        for i in range(uses):
            s = i % n_slots
            epochs[s] += 1
            e = epochs[s]
            if i >= n_slots:
                while not released[r][i - n_slots]:
                    yield
            if e > 1 and wait_acks:
                while not all(acks[r][q][s] >= e - 1 for q in range(world) if q != r):
                    yield
            for k in range(PIECES):
                mem[r][s][r][k] = i
                if not publish_after_copy and k == 0:
                    for p in range(world):
                        flags[p][r][s] = e
                yield
            for p in range(world):
                flags[p][r][s] = e
                yield
            peers = [p for p in range(world) if p != r]
            rnd.shuffle(peers)
            for p in peers:
                while flags[r][p][s] < e:
                    yield
                for k in range(PIECES):
                    v = mem[p][s][p][k]
                    assert v == i, f"rank {r} use {i}: piece {k} of rank {p}'s stripe holds use {v}"
                    mem[r][s][p][k] = v
                    if not ack_after_pull:
                        acks[p][r][s] = e
                    yield
            for p in peers:
                acks[p][r][s] = e
            ready[r][i] = True
            yield

    def compute_stream(r):
        for i in range(uses):
            s = i % n_slots
            while not ready[r][i]:
                yield
            for q in range(world):
                for k in range(PIECES):
                    assert mem[r][s][q][k] == i, f"rank {r} use {i}: compute reads use {mem[r][s][q][k]} of {q}"
                    yield
            released[r][i] = True

    gens = [copy_stream(r) for r in range(world)] + [compute_stream(r) for r in range(world)]
    alive = set(range(len(gens)))
    for _ in range(600000):
        if not alive:
            return
        g = rnd.choice(sorted(alive))
        try:
            next(gens[g])
        except StopIteration:
            alive.discard(g)
    raise AssertionError("deadlock")


@pytest.mark.parametrize("world", [2, 3, 4, 8])
@pytest.mark.parametrize("n_slots", [1, 2, 3])
@pytest.mark.parametrize("seed", range(6))
def test_striped_protocol(world, n_slots, seed):
    run(world, 8, n_slots, seed)


@pytest.mark.parametrize("n_slots", [2, 3])
@pytest.mark.parametrize("seed", range(6))
def test_ring_reuse_is_ordered_by_the_flag_chain(n_slots, seed):
    run(4, 9, n_slots, seed, wait_acks=False)


@pytest.mark.parametrize("mutant", [dict(n_slots=1, wait_acks=False), dict(n_slots=1, ack_after_pull=False),
                                    dict(n_slots=2, publish_after_copy=False)])
def test_model_catches_broken_protocols(mutant):
    failures = 0
    for seed in range(40):
        try:
            run(3, 7, seed=seed, **mutant)
        except AssertionError:
            failures += 1
    assert failures > 0
