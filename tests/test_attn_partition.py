"""CPU: the balanced partition of the tensor-core flash-decode, restated step for step from
attn_mma.cu (sk_tiles, sk_per, sk_find_start, ItemIter::next and the merge's split count),
checked for the properties the kernel and the merge rely on: every tile of every computed
(sequence, kv head) pair is taken by exactly one CTA; a pair's pieces are numbered 0, 1, ...
in token order; the merge's split count equals the pieces' nsplit_b; no pair has more than
kMaxSplits pieces (the partial workspace holds that many); skipped sequences take no tiles.
The GPU tests run the kernel itself on ragged batches against the oracle."""
import numpy as np
import pytest

from conftest import attn_mma_plan

KT, KMAX, KMIN = 64, 64, 4


def sk_tiles(pos, max_pos, cap):
    return pos // KT + 1 if 0 <= pos <= max_pos and pos < cap else 0


def sk_per(total, nmax, grid):
    return max(-(-total // grid), (nmax + KMAX - 2) // (KMAX - 1), KMIN)


def partition(pos, hkv, grid, max_pos, cap):
    """{(b, kvh, tile): (cta, split, nsplit_b)} and the merge's split count per pair."""
    B = len(pos)
    n = [sk_tiles(int(p), max_pos, cap) for p in pos]
    total = sum(n) * hkv
    per = sk_per(total, max(n), grid)
    owner = {}
    for c in range(grid):
        lo, hi = c * per, min(c * per + per, total)
        # sk_find_start: the first sequence whose pairs hold tile lo
        bs, run = B, 0
        if lo < total:
            for b in range(B):
                if n[b] > 0 and run + n[b] * hkv > lo:
                    bs = b
                    break
                run += n[b] * hkv
        if bs < B:
            kvh = (lo - run) // n[bs]
            b, P = bs, run + kvh * n[bs]
        else:
            b, kvh, P = B, 0, total
        # ItemIter::next
        while b < B and P < hi:
            nn, P0, bb, kv = n[b], P, b, kvh
            P += nn
            kvh += 1
            if kvh == hkv:
                kvh, b = 0, b + 1
            if nn == 0 or P0 + nn <= lo:
                continue
            s0, s1 = max(lo, P0) - P0, min(hi, P0 + nn) - P0
            split, nsb = c - P0 // per, (P0 + nn - 1) // per - P0 // per + 1
            for t in range(s0, s1):
                assert (bb, kv, t) not in owner
                owner[(bb, kv, t)] = (c, split, nsb)
    merge = {}
    for b in range(B):
        for kv in range(hkv):
            if n[b]:
                P = sum(n[:b]) * hkv + kv * n[b]
                merge[(b, kv)] = (P + n[b] - 1) // per - P // per + 1
    return n, owner, merge


def check(pos, hkv, grid, max_pos, cap):
    n, owner, merge = partition(pos, hkv, grid, max_pos, cap)
    assert len(owner) == sum(n) * hkv
    for b in range(len(pos)):
        for kv in range(hkv):
            if not n[b]:
                assert (b, kv) not in merge
                continue
            pieces = [owner[(b, kv, t)] for t in range(n[b])]
            splits = [p[1] for p in pieces]
            assert splits == sorted(splits)                      # token order
            assert sorted(set(splits)) == list(range(merge[(b, kv)]))
            assert all(p[2] == merge[(b, kv)] for p in pieces)   # kernel and merge agree
            assert merge[(b, kv)] <= KMAX


@pytest.mark.parametrize("B,ctx", [(64, 8205), (16, 8192), (40, 6000), (64, 32768)])
def test_uniform_and_headline_batches(B, ctx):
    check([ctx - 1 - (b % 3) for b in range(B)], 2, 148, ctx - 1, ctx + 8)


def test_one_long_sequence_among_short_ones():
    """Most tiles in one pair: the share per CTA is raised so that pair spans at most 64 CTAs."""
    pos = [200_000] + [10] * 30
    check(pos, 2, 148, 200_000, 200_008)
    n, owner, merge = partition(pos, 2, 148, 200_000, 200_008)
    assert max(merge.values()) <= KMAX


def test_seeded_ragged_batches_with_skipped_sequences():
    rng = np.random.default_rng(7)
    for _ in range(200):
        B = int(rng.integers(1, 90))
        hkv = int(rng.choice([1, 2, 4]))
        cap = int(rng.integers(1, 40_000))
        max_pos = int(rng.integers(0, cap))
        pos = [int(rng.choice([rng.integers(0, cap), 0, max_pos, max_pos + 1, -1])) for _ in range(B)]
        check(pos, hkv, int(rng.choice([148, 132, 7])), max_pos, cap)


def test_headline_step_takes_the_balanced_partition():
    """The bench's step (B=64, ctx ~8.2K, 2 kv heads) is where the balanced plan pays: 112
    tiles on every CTA against 9 items of 13 tiles on the busiest one."""
    assert attn_mma_plan(64, 2, 8205, 148) == "balanced"
    assert attn_mma_plan(1, 2, 32768, 148) == "chunk"
    assert sk_per(64 * 2 * 129, 129, 148) == 112
