"""CPU model of the tcgen05 decode kernel's work split (stream-K over the
128-token tiles of every (sequence, KV head) segment), mirroring the index
math of range_start / cta_of_tile / piece_at / piece_slot in
inference_c_b200/csrc/pkv_decode.cu.  Checks that every tile is processed
exactly once, that no two partial pieces of a CTA share a slot, and that the
merge of every split segment finds exactly the slots that were written."""
from __future__ import annotations

import numpy as np
import pytest

TILE = 128


def split(lengths, kv_heads, grid):
    nt = [(int(L) + TILE - 1) // TILE for L in lengths]
    prefix = np.concatenate([[0], np.cumsum([n * kv_heads for n in nt])]).astype(np.int64)
    total = int(prefix[-1])
    if total == 0:
        return {}, {}, nt, prefix, 0, 0
    ncta = min(grid, total)                      # CTAs past the tile count idle

    def range_start(c):
        return total * c // ncta

    covered = np.zeros(total, np.int64)
    written, direct = {}, set()
    for c in range(ncta):
        s, e = range_start(c), range_start(c + 1)
        assert e > s                             # every working CTA owns a tile
        t = s
        while t < e:
            lo, hi = 0, len(lengths) - 1         # last sequence starting at or before t
            while lo < hi:
                mid = (lo + hi + 1) // 2
                if prefix[mid] <= t:
                    lo = mid
                else:
                    hi = mid - 1
            b = lo
            n = int(prefix[b + 1] - prefix[b]) // kv_heads
            w = t - prefix[b]
            g, k0 = int(w // n), int(w % n)
            seg = int(prefix[b]) + g * n
            k1 = min(n, k0 + (e - t))
            covered[seg + k0:seg + k1] += 1
            first_piece = t == s
            t += k1 - k0
            if k0 == 0 and k1 == n:
                direct.add((b, g))
                continue
            key = (c, 0 if first_piece else 1)
            assert key not in written
            written[key] = (b, g, k0, k1)
    assert (covered == 1).all()
    return written, direct, nt, prefix, total, ncta


def check(lengths, kv_heads, grid):
    written, direct, nt, prefix, total, ncta = split(lengths, kv_heads, grid)
    if total == 0:
        return 0
    cta_of = lambda t: ((t + 1) * ncta - 1) // total  # noqa: E731
    slot_of = lambda c, seg: 1 if total * c // ncta < seg else 0  # noqa: E731
    merged = 0
    for b, n in enumerate(nt):
        for g in range(kv_heads if n else 0):
            seg = int(prefix[b]) + g * n
            first, last = cta_of(seg), cta_of(seg + n - 1)
            if first == last:
                assert (b, g) in direct
                continue
            pieces = [written[(c, slot_of(c, seg))] for c in range(first, last + 1)]
            assert all(p[:2] == (b, g) for p in pieces)
            spans = sorted(p[2:] for p in pieces)
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(x[1] == y[0] for x, y in zip(spans, spans[1:]))
            merged += 1
    return merged


@pytest.mark.parametrize("seed", range(200))
def test_random_shapes(seed):
    rng = np.random.default_rng(seed)
    B = int(rng.integers(1, 80))
    lengths = rng.integers(0, 3000, B)
    lengths[rng.random(B) < 0.1] = 0
    check(lengths, int(rng.choice([1, 2, 4, 8])), int(rng.integers(1, 257)))


def test_config_shapes():
    from inference_c_b200 import workloads as W
    assert check(W.context_lengths(3, 0), 8, 148) > 0          # config 3, one GPU
    check(W.context_lengths(2, 0), 8, 148)                      # config 2
    assert check([131072], 1, 148) == 1                         # config 4 per GPU
    lengths = np.arange(1100) % 300                              # sliced launches
    check(lengths[:1024], 1, 148)
    check(lengths[1024:], 1, 148)                                # fewer tiles than CTAs
