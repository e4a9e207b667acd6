"""Byte accounting of the fused all-gather GEMM's row gather (``gather_rows`` and the TMA
producer's per-block waits in ``ops/csrc/tp_sm100.cu``; scratch sizing ``tp_ag_counter_words``
in ``ops/csrc/ft_tp.h``), restated in Python with the same integer arithmetic and checked over
random shapes:

* the gather splits each peer's ``rows x row_bytes`` into ``TP_PIECE``-byte pieces; a landed
  piece adds its overlap with every 128-row block it touches to ``done_blk[peer][block]``;
* a tile's producer waits until ``done_blk[q][b]`` reaches the block's full byte count for every
  block b of every peer q whose rows the tile reads (1-SM tiles of 128 rows, and each CTA's 128
  rows of a 256-row CTA-pair tile).

Checked: the counters stay inside the scratch the host zeroes; each block's count reaches
exactly its target once all its pieces landed, and never before (every piece that touches a
block adds a positive count); every row a tile reads lies in a block it waited for.
"""

import random

import pytest

TP_PIECE = 12288
BM = 128


def counter_words(M, world):
    return world * (2 + (M // world + 127) // 128) if world > 1 else 2 * world


def pieces_of(rows, row_bytes):
    rank_bytes = rows * row_bytes
    n = (rank_bytes + TP_PIECE - 1) // TP_PIECE
    return [(i * TP_PIECE, min(TP_PIECE, rank_bytes - i * TP_PIECE)) for i in range(n)]


def contributions(off, n, row_bytes):
    blk = BM * row_bytes
    b0, b1 = off // blk, (off + n - 1) // blk
    out = []
    for b in range(b0, b1 + 1):
        lo, hi = max(off, b * blk), min(off + n, (b + 1) * blk)
        out.append((b, hi - lo))
    return out


def waited_blocks(r0, r1, rows, rank):
    """The producer loop: (peer, block, bytes) for rows [r0, r1)."""
    out = []
    for q in range(r0 // rows, (r1 - 1) // rows + 1):
        if q == rank:
            continue
        qb = q * rows
        lo, hi = max(r0, qb) - qb, min(r1, qb + rows) - qb
        for b in range(lo // BM, (hi - 1) // BM + 1):
            out.append((q, b, (min((b + 1) * BM, rows) - b * BM)))
    return out


def _shapes(seed):
    rnd = random.Random(seed)
    world = rnd.choice([2, 3, 4, 8])
    rows = rnd.choice([1, 7, 64, 127, 128, 129, 300, 1000, 2048]) * rnd.choice([1, 1, 2])
    K = 8 * rnd.randint(1, 1200)  # row_bytes = 2K: a multiple of 16, as the host requires
    return world, rows, K


@pytest.mark.parametrize("seed", range(60))
def test_block_counts_reach_exactly_their_targets(seed):
    world, rows, K = _shapes(seed)
    M, row_bytes = rows * world, 2 * K
    nblk = (rows + BM - 1) // BM
    words = counter_words(M, world)
    done_blk_base = 2 * world
    for p in range(world):
        counts = [0] * nblk
        touching = [0] * nblk
        for off, n in pieces_of(rows, row_bytes):
            assert n > 0
            for b, c in contributions(off, n, row_bytes):
                assert c > 0 and 0 <= b < nblk
                assert done_blk_base + p * nblk + b < words  # inside the zeroed scratch
                counts[b] += c
                touching[b] += 1
        for b in range(nblk):
            target = (min((b + 1) * BM, rows) - b * BM) * row_bytes
            assert counts[b] == target, (p, b, counts[b], target)
            assert target < 2 ** 32  # u32 counters (the host rejects row_bytes * 128 >= 2^32)
            assert touching[b] >= 1


@pytest.mark.parametrize("seed", range(60))
@pytest.mark.parametrize("pair", [False, True])
def test_tiles_wait_for_every_block_they_read(seed, pair):
    world, rows, _ = _shapes(seed)
    M = rows * world
    for rank in range(world):
        tiles = []
        if pair:  # each CTA of a 256-row pair tile reads its own 128 rows
            for mt2 in range((M + 255) // 256):
                for crank in (0, 1):
                    r0 = mt2 * 256 + crank * BM
                    if r0 < M:
                        tiles.append((r0, min(r0 + BM, M)))
        else:
            tiles = [(mt * BM, min(mt * BM + BM, M)) for mt in range((M + BM - 1) // BM)]
        for r0, r1 in tiles:
            waited = {(q, b) for q, b, _ in waited_blocks(r0, r1, rows, rank)}
            for r in range(r0, r1):
                q = r // rows
                if q == rank:
                    continue
                assert (q, (r - q * rows) // BM) in waited, (rank, r0, r1, r)
