"""Barrier-protocol model of the CTA-pair tensor-parallel GEMM (``tp_gemm_pair_kernel``), checked
on the CPU before the kernel runs on a GPU.

Two CTAs each run a TMA producer and an epilogue; the leader also runs the MMA thread. The
mbarrier semantics are real, including the transaction bytes that both CTAs' loads count on the
leader's full barrier. Under randomised schedules the model asserts:
* every parity wait sees exactly the intended phase or the next one, never an ambiguous state;
* the MMA never reads a stage that a load is still filling;
* no CTA reloads a stage the MMA still reads;
* the MMA never writes an accumulator that an epilogue of either CTA is still reading;
* every tile is stored exactly once by each CTA, and nothing deadlocks.
"""

import random

import pytest

STAGES = 6


class Bar:
    def __init__(self, name, count):
        self.name, self.count, self.arr, self.tx, self.done = name, count, count, 0, 0

    def _maybe_complete(self):
        if self.arr == 0 and self.tx == 0:
            self.done += 1
            self.arr = self.count

    def arrive(self, n=1):
        self.arr -= n
        assert self.arr >= 0, f"{self.name}: over-arrival"
        self._maybe_complete()

    def expect_tx(self, nbytes):  # arrive.expect_tx: one arrival plus the bytes to wait for
        self.tx += nbytes
        self.arrive()

    def complete_tx(self, nbytes):
        self.tx -= nbytes
        self._maybe_complete()

    def ready(self, phase):
        assert self.done in (phase, phase + 1), f"{self.name}: wait for phase {phase}, {self.done} completed"
        return self.done == phase + 1


def run(tiles, kblocks, seed, tempty_count=8, expect_ctas=2):
    rnd = random.Random(seed)
    full = [Bar(f"full{s}", 1) for s in range(STAGES)]                  # leader's copy is used
    empty = [[Bar(f"empty{c}.{s}", 1) for s in range(STAGES)] for c in range(2)]
    tfull = [[Bar(f"tfull{c}.{a}", 1) for a in range(2)] for c in range(2)]
    tempty = [Bar(f"tempty{a}", tempty_count) for a in range(2)]        # leader's copy
    st = {"filling": [set() for _ in range(STAGES)], "reading": [False] * STAGES,
          "acc_read": [0, 0], "acc_write": [False, False], "stored": [[], []]}
    inflight = []  # (stage, cta, bytes) loads not yet landed

    def producer(c):
        for i in range(tiles * kblocks):
            s, use = i % STAGES, i // STAGES
            while use > 0 and not empty[c][s].ready(use - 1):
                yield
            assert not st["reading"][s], "reload of a stage the MMA still reads"
            if c == 0:
                full[s].expect_tx(expect_ctas * 32768)
            st["filling"][s].add(c)
            inflight.append((s, c, 32768))
            yield

    def memory():
        while True:
            if inflight and rnd.random() < 0.5:
                s, c, n = inflight.pop(rnd.randrange(len(inflight)))
                st["filling"][s].discard(c)
                full[s].complete_tx(n)
            yield

    def mma():
        i = 0
        for t in range(tiles):
            acc, use = t & 1, t >> 1
            while use > 0 and not tempty[acc].ready(use - 1):
                yield
            assert st["acc_read"][acc] == 0, "MMA writes an accumulator an epilogue still reads"
            st["acc_write"][acc] = True
            for _ in range(kblocks):
                s = i % STAGES
                while not full[s].ready(i // STAGES):
                    yield
                assert not st["filling"][s], "MMA reads a stage that is still being filled"
                st["reading"][s] = True
                yield
                st["reading"][s] = False
                for c in range(2):  # tcgen05.commit multicast to both CTAs
                    empty[c][s].arrive()
                i += 1
            st["acc_write"][acc] = False
            for c in range(2):
                tfull[c][acc].arrive()

    def epilogue(c):
        for t in range(tiles):
            acc, use = t & 1, t >> 1
            while not tfull[c][acc].ready(use):
                yield
            assert not st["acc_write"][acc]
            st["acc_read"][acc] += 1
            for _ in range(rnd.randint(1, 5)):
                yield
            st["acc_read"][acc] -= 1
            st["stored"][c].append(t)
            tempty[acc].arrive(4)  # 4 epilogue warps, remote arrive for the non-leader

    actors = [producer(0), producer(1), memory(), mma(), epilogue(0), epilogue(1)]
    finite = {0, 1, 3, 4, 5}
    alive = [True] * len(actors)
    for _ in range(400000):
        i = rnd.randrange(len(actors))
        if not alive[i]:
            continue
        try:
            next(actors[i])
        except StopIteration:
            alive[i] = False
        if not any(alive[k] for k in finite):
            assert st["stored"] == [list(range(tiles)), list(range(tiles))]
            return
    raise AssertionError("deadlock")


@pytest.mark.parametrize("tiles,kblocks", [(1, 1), (3, 2), (5, 7), (8, 3)])
@pytest.mark.parametrize("seed", range(10))
def test_tp_pair_protocol(tiles, kblocks, seed):
    run(tiles, kblocks, seed)


@pytest.mark.parametrize("mutant", [{"tempty_count": 4}, {"expect_ctas": 1}])
def test_model_catches_broken_protocols(mutant):
    """The model is strong enough to see the two pair-specific mistakes: an accumulator-empty
    barrier that counts one CTA's epilogue only, and a full barrier that expects one CTA's bytes."""
    failures = 0
    for seed in range(20):
        try:
            run(5, 3, seed, **mutant)
        except AssertionError:
            failures += 1
    assert failures > 0
