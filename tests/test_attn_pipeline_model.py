"""Barrier-protocol model of the one-tile attention kernel (``attn1_fwd_kernel``), checked on the
CPU before the kernel runs on a GPU.

Each actor is a generator: the TMA producer, the MMA issuer, the tensor core and the softmax
warp group. They run under a randomised scheduler against mbarriers with real phase semantics.
A parity wait on phase k is only unambiguous while the barrier has completed exactly k or k+1
phases. The model asserts that every wait in the kernel's protocol sees one of those two
states, that nothing deadlocks, and that each S / P / O access happens in a legal order:
* a softmax never reads an S buffer the tensor core is still writing;
* QK^T never overwrites a P that the PV has not consumed;
* O is never rescaled while a PV into it is in flight.
"""

import random

import pytest

KV = 3  # K/V ring depth of the kernel


class Bar:
    def __init__(self, name, count):
        self.name, self.count, self.pending, self.done = name, count, count, 0

    def arrive(self, n=1):
        self.pending -= n
        assert self.pending >= 0, f"{self.name}: over-arrival"
        if self.pending == 0:
            self.done += 1
            self.pending = self.count

    def ready(self, phase):
        c = self.done
        assert c in (phase, phase + 1), f"{self.name}: wait for phase {phase} while {c} phases completed"
        return c == phase + 1


def run(n_kv, seed, rescale_every=0):
    rnd = random.Random(seed)
    B = {}

    def bar(name, count=1):
        B[name] = Bar(name, count)
        return B[name]

    k_full = [bar(f"k_full{s}") for s in range(KV)]
    k_empty = [bar(f"k_empty{s}") for s in range(KV)]
    v_full = [bar(f"v_full{s}") for s in range(KV)]
    v_empty = [bar(f"v_empty{s}") for s in range(KV)]
    s_full = [bar(f"s_full{u}") for u in range(2)]
    p_half = [bar(f"p_half{u}", 4) for u in range(2)]
    p_full = [bar(f"p_full{u}", 4) for u in range(2)]
    o_done, o_final = bar("o_done"), bar("o_final")
    state = {"S_writer": [None, None], "P_owner": [None, None], "pv_in_flight": 0, "pv_done": 0}
    tc = []  # tensor-core queue: ops run in issue order

    # waits name the phase INDEX they mean; the kernel passes its parity to the hardware
    def producer():
        for j in range(n_kv):
            s, use = j % KV, j // KV
            while use > 0 and not k_empty[s].ready(use - 1):  # previous use of the stage released
                yield
            yield
            k_full[s].arrive()
            while use > 0 and not v_empty[s].ready(use - 1):
                yield
            yield
            v_full[s].arrive()

    def issue_S(j):
        tc.append(("S", j))

    def mma():
        for j in range(min(2, n_kv)):
            while not k_full[j % KV].ready(j // KV):
                yield
            issue_S(j)
        for j in range(n_kv):
            s, pph = j % KV, j >> 1
            while not v_full[s].ready(j // KV):
                yield
            while not p_half[j & 1].ready(pph):
                yield
            tc.append(("PV1", j))
            while not p_full[j & 1].ready(pph):
                yield
            tc.append(("PV2", j))
            if j == n_kv - 1:
                tc.append(("final", j))
            if j + 2 < n_kv:
                while not k_full[(j + 2) % KV].ready((j + 2) // KV):
                    yield
                issue_S(j + 2)
            yield

    def tensor_core():
        while True:
            if not tc:
                yield
                continue
            op, j = tc.pop(0)
            for _ in range(rnd.randint(1, 4)):  # the op runs for a while
                if op == "S":
                    state["S_writer"][j & 1] = j
                if op.startswith("PV"):
                    state["pv_in_flight"] = 1
                yield
            if op == "S":
                # S(j) overwrites buffer j % 2: the P of block j - 2 there must have been consumed
                assert state["P_owner"][j & 1] in (None, "consumed"), f"S({j}) over live P"
                state["S_writer"][j & 1] = None
                state["P_owner"][j & 1] = None
                s_full[j & 1].arrive()
                k_empty[j % KV].arrive()
            elif op == "PV1":
                pass
            elif op == "PV2":
                state["pv_in_flight"] = 0
                state["pv_done"] += 1
                state["P_owner"][j & 1] = "consumed"
                o_done.arrive()
                v_empty[j % KV].arrive()
            elif op == "final":
                o_final.arrive()

    def softmax():
        for j in range(n_kv):
            while not s_full[j & 1].ready(j >> 1):
                yield
            assert state["S_writer"][j & 1] is None, f"softmax({j}) reads an S being written"
            state["P_owner"][j & 1] = j
            for _ in range(rnd.randint(1, 6)):
                yield
            if rescale_every and j > 0 and j % rescale_every == 0:
                while not o_done.ready(j - 1):
                    yield
                assert state["pv_in_flight"] == 0 and state["pv_done"] == j, f"O rescaled with PV in flight ({j})"
            p_half[j & 1].arrive(4)
            for _ in range(rnd.randint(1, 6)):
                yield
            p_full[j & 1].arrive(4)
        while not o_final.ready(0):
            yield
        assert state["pv_done"] == n_kv

    actors = [producer(), mma(), tensor_core(), softmax()]
    alive = [True] * 4
    for _ in range(200000):
        i = rnd.randrange(4)
        if not alive[i]:
            continue
        try:
            next(actors[i])
        except StopIteration:
            alive[i] = False
        if not alive[0] and not alive[1] and not alive[3]:
            return
    raise AssertionError("deadlock: the protocol did not finish")


@pytest.mark.parametrize("n_kv", [1, 2, 3, 4, 7, 16])
@pytest.mark.parametrize("seed", range(12))
def test_one_tile_attention_protocol(n_kv, seed):
    run(n_kv, seed)


@pytest.mark.parametrize("seed", range(12))
def test_one_tile_attention_protocol_with_rescales(seed):
    run(11, seed, rescale_every=2)
