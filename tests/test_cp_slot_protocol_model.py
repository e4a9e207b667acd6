"""CPU model of the context-parallel K/V slot protocol between ranks (``parallel/cp.py`` host
side, ``ops/csrc/p2p.cu`` publish / wait-acks kernels, the gather inside the CP attention
kernel), run under random interleavings of the ranks.

Per attention call c every rank uses slot ``c % n_slots`` (two in the package) at that slot's epoch e:
* begin: if e > 1, wait until every peer's ack for this slot is >= e - 1, then write its own
  rows into its local slot;
* publish: store e into ``flags[p][rank][slot]`` of every rank p;
* attention: for each peer p (in any order), wait ``flags[rank][p][slot] >= e``, copy p's rows
  from p's slot in pieces, then store e into ``acks[p][rank][slot]``; finally read the whole slot.

The model asserts that every copied piece and every row the attention reads belong to call c
(no overwrite of rows a peer is still gathering, no stale rows) and that nothing deadlocks.

What it shows about the design: with the two-slot ring, the flags alone already order slot
reuse (a rank reaches call c+2 only after every peer published call c+1, which each peer does
after its call-c gather ends). The acks are what keep a ring of one slot safe, and what the
teardown waits on before the heap is freed; the model fails a one-slot ring without the ack
wait, or with an ack sent before the copy ends.
"""

import random

import pytest

PIECES = 3


def run(world, calls, seed, n_slots=2, wait_acks=True, ack_after_copy=True):
    rnd = random.Random(seed)
    # slot memory: mem[r][s][q] = list of PIECES values, rows of rank q held in r's slot s
    mem = [[[[None] * PIECES for _ in range(world)] for _ in range(n_slots)] for _ in range(world)]
    flags = [[[0] * n_slots for _ in range(world)] for _ in range(world)]  # flags[r][q][s]
    acks = [[[0] * n_slots for _ in range(world)] for _ in range(world)]   # acks[r][q][s]

    def rank(r):
        epochs = [0] * n_slots
        for c in range(calls):
            s = c % n_slots
            epochs[s] += 1
            e = epochs[s]
            if e > 1 and wait_acks:
                while not all(acks[r][q][s] >= e - 1 for q in range(world) if q != r):
                    yield
            for i in range(PIECES):  # the K/V projections write this rank's rows, piece by piece
                mem[r][s][r][i] = c
                yield
            for p in range(world):
                flags[p][r][s] = e
                yield
            peers = [p for p in range(world) if p != r]
            rnd.shuffle(peers)
            for p in peers:
                while flags[r][p][s] < e:
                    yield
                for i in range(PIECES):
                    v = mem[p][s][p][i]
                    assert v == c, f"rank {r} call {c}: piece {i} of rank {p}'s rows holds call {v}"
                    mem[r][s][p][i] = v
                    if not ack_after_copy and i == 0:
                        acks[p][r][s] = e
                    yield
                acks[p][r][s] = e
            for q in range(world):
                assert mem[r][s][q] == [c] * PIECES, f"rank {r} call {c}: attention reads {mem[r][s][q]} of {q}"
            yield

    gens = [rank(r) for r in range(world)]
    alive = set(range(world))
    for _ in range(200000):
        if not alive:
            return
        r = rnd.choice(sorted(alive))
        try:
            next(gens[r])
        except StopIteration:
            alive.discard(r)
    raise AssertionError("deadlock")


@pytest.mark.parametrize("world", [2, 3, 4, 8])
@pytest.mark.parametrize("n_slots", [1, 2])
@pytest.mark.parametrize("seed", range(8))
def test_cp_slot_protocol(world, n_slots, seed):
    run(world, 7, seed, n_slots=n_slots)


@pytest.mark.parametrize("seed", range(8))
def test_two_slot_reuse_is_ordered_by_the_flags_alone(seed):
    run(4, 9, seed, n_slots=2, wait_acks=False, ack_after_copy=False)


@pytest.mark.parametrize("mutant", [{"wait_acks": False}, {"ack_after_copy": False}])
def test_model_catches_broken_one_slot_protocols(mutant):
    failures = 0
    for seed in range(40):
        try:
            run(3, 7, seed, n_slots=1, **mutant)
        except AssertionError:
            failures += 1
    assert failures > 0
