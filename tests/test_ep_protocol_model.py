"""CPU model of the expert-parallel MoE protocol between ranks (``parallel/ep.py`` host side,
``ops/csrc/p2p.cu`` publish / wait-acks, the pulls and flags inside ``moe_sm100.cu``), run under
random interleavings of the ranks. Every rank is both a token source and an expert. Per MoE
layer call at epoch e, in each rank's stream order:

1. source: if e > 1, wait until every expert acked epoch e - 1; pack the send buffer; store e
   into every rank's send flag for this source;
2. dispatch GEMM: for each source (any order) wait for its send flag >= e, pull its rows in
   pieces, ack the source;
3. combine GEMM: store the output rows into each source's combine buffer in pieces, then store e
   into that source's combine flag for this expert;
4. reduce: wait for every expert's combine flag >= e, read the combine buffer.

The model asserts that every pulled piece and every combined row read belongs to epoch e, and
that nothing deadlocks. As for the context-parallel slots, the flag chain alone already orders
reuse of the single send and combine buffers: a source packs e + 1 only after its reduce of e,
which waits for every expert's combine of e, which follows that expert's pull of e. The model
shows that (it passes without the ack wait) and fails a flag stored before its data.
"""

import random

import pytest

PIECES = 3


def run(world, calls, seed, wait_acks=True, flag_after_pack=True, comb_flag_after_store=True):
    rnd = random.Random(seed)
    send = [[0] * PIECES for _ in range(world)]                           # send[p]: p's packed rows
    comb = [[[0] * PIECES for _ in range(world)] for _ in range(world)]   # comb[p][q]: rows q computed for p
    send_flags = [[0] * world for _ in range(world)]                      # send_flags[r][p]
    send_acks = [[0] * world for _ in range(world)]                       # send_acks[p][q]
    comb_flags = [[0] * world for _ in range(world)]                      # comb_flags[p][q]

    def rank(r):
        for e in range(1, calls + 1):
            if e > 1 and wait_acks:
                while not all(send_acks[r][q] >= e - 1 for q in range(world) if q != r):
                    yield
            for i in range(PIECES):
                send[r][i] = e
                if not flag_after_pack and i == 0:
                    for p in range(world):
                        send_flags[p][r] = e
                yield
            for p in range(world):
                send_flags[p][r] = e
                yield
            order = list(range(world))
            rnd.shuffle(order)
            pulled = {}
            for p in order:  # dispatch GEMM: pull every source's rows for this expert
                while send_flags[r][p] < e:
                    yield
                got = []
                for i in range(PIECES):
                    got.append(send[p][i])
                    yield
                assert got == [e] * PIECES, f"expert {r} epoch {e}: pulled {got} from source {p}"
                pulled[p] = got
                if p != r:
                    send_acks[p][r] = e
            rnd.shuffle(order)
            for p in order:  # combine GEMM: store into each source's combine buffer, then flag
                for i in range(PIECES):
                    comb[p][r][i] = pulled[p][i]
                    if not comb_flag_after_store and i == 0:
                        comb_flags[p][r] = e
                    yield
                comb_flags[p][r] = e
            for q in range(world):  # reduce
                while comb_flags[r][q] < e:
                    yield
                assert comb[r][q] == [e] * PIECES, f"source {r} epoch {e}: combine rows of {q} are {comb[r][q]}"
            yield

    gens = [rank(r) for r in range(world)]
    alive = set(range(world))
    for _ in range(400000):
        if not alive:
            return
        r = rnd.choice(sorted(alive))
        try:
            next(gens[r])
        except StopIteration:
            alive.discard(r)
    raise AssertionError("deadlock")


@pytest.mark.parametrize("world", [2, 3, 4, 8])
@pytest.mark.parametrize("seed", range(8))
def test_ep_protocol(world, seed):
    run(world, 6, seed)


@pytest.mark.parametrize("seed", range(8))
def test_buffer_reuse_is_ordered_by_the_flag_chain(seed):
    run(4, 6, seed, wait_acks=False)


@pytest.mark.parametrize("mutant", [{"flag_after_pack": False}, {"comb_flag_after_store": False}])
def test_model_catches_flags_before_data(mutant):
    failures = 0
    for seed in range(40):
        try:
            run(3, 5, seed, **mutant)
        except AssertionError:
            failures += 1
    assert failures > 0
