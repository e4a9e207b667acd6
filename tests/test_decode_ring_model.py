"""CPU model of the decode kernel's TMA ring (``ops/csrc/decode_sm100.cu``) under random schedules.

mbarrier semantics as the kernel uses them: a phase completes when its arrival count is reached
and its transaction bytes have landed; ``wait(parity)`` returns as soon as the barrier's current
(incomplete) phase parity differs from ``parity``. One producer issues tiles in order; several
consumer warps each take every NCW-th tile; TMA completions land in random order.

Checked invariants: a consumer only reads a stage that holds exactly the tile it waits for, and
no barrier phase receives more arrivals than its count (the ``arrive.expect_tx`` of a refill must
not land in a phase that is still pending).

The shared-stage layout (tile i -> stage i % DSTAGES, any warp) violates them under some
schedules: a warp's wait for the second use of a stage passes while the first use is still in
flight, because a fresh barrier's "previous" phase counts as complete. The per-warp layout the
kernel uses (each warp owns SPW stages, used in order) never does.
"""

import random

import pytest


class Bar:
    def __init__(self, count):
        self.count, self.arrived, self.pending_tx, self.completed = count, 0, 0, 0
        self.overflow = False

    @property
    def parity(self):  # parity of the current (incomplete) phase
        return self.completed & 1

    def try_wait(self, parity):
        return self.parity != parity

    def arrive(self, tx=0):
        self.arrived += 1
        self.pending_tx += tx
        if self.arrived > self.count:
            self.overflow = True
        self._maybe_complete()

    def land(self, tx):
        self.pending_tx -= tx
        self._maybe_complete()

    def _maybe_complete(self):
        if self.arrived >= self.count and self.pending_tx == 0:
            self.completed += 1
            self.arrived, self.pending_tx = 0, 0


def simulate(n_tiles, ncw, stages, per_warp, spw, seed, steps=20000):
    rng = random.Random(seed)
    full = [Bar(1) for _ in range(stages)]
    empty = [Bar(1) for _ in range(stages)]
    content = [None] * stages           # tile whose bytes are in the stage (after landing)
    in_flight = []                       # (stage, tile)

    def stage_of(i):
        if per_warp:
            w, j = i % ncw, i // ncw
            return w * spw + (j % spw), (j // spw) & 1
        return i % stages, (i // stages) & 1

    nxt = 0                              # producer's next tile
    cons = {w: w for w in range(ncw)}    # each warp's next tile
    violations = []
    for _ in range(steps):
        actors = ["prod", "land"] + [f"w{w}" for w in range(ncw)]
        a = rng.choice(actors)
        if a == "prod" and nxt < n_tiles:
            s, ph = stage_of(nxt)
            if empty[s].try_wait(ph ^ 1):
                full[s].arrive(tx=1)
                if full[s].overflow:
                    violations.append(("double arrival", nxt, s))
                in_flight.append((s, nxt))
                nxt += 1
        elif a == "land" and in_flight:
            s, t = in_flight.pop(rng.randrange(len(in_flight)))
            content[s] = t
            full[s].land(1)
        elif a.startswith("w"):
            w = int(a[1:])
            i = cons[w]
            if i >= n_tiles:
                continue
            s, ph = stage_of(i)
            if full[s].try_wait(ph):
                if content[s] != i:
                    violations.append(("stale read", i, s, content[s]))
                empty[s].arrive()
                cons[w] = i + ncw
        if nxt >= n_tiles and all(c >= n_tiles for c in cons.values()) and not in_flight:
            break
    return violations


@pytest.mark.parametrize("seed", range(200))
def test_per_warp_stages_never_alias(seed):
    assert simulate(n_tiles=24, ncw=4, stages=8, per_warp=True, spw=2, seed=seed) == []


def test_shared_stages_can_alias():
    """The layout the kernel used before: some schedule reads a stage early."""
    found = [v for seed in range(400) for v in simulate(n_tiles=12, ncw=4, stages=6, per_warp=False, spw=0,
                                                           seed=seed)]
    assert found, "the model should expose the shared-stage parity race"
