"""CPU model of the tcgen05 decode kernel's work split (stream-K over the
128-token tiles of every (sequence, KV head) segment, cut into static units
and, with the dynamic tail, rounds of smaller claimed units), mirroring the
index math of make_sched / unit_start / unit_of_tile / unit_slot / piece_at in
inference_c_b200/csrc/pkv_decode.cu and the host's choice of min_unit.
Checks that every tile is processed exactly once whatever order the units are
claimed in, that no two partial pieces of a unit share a slot, that the merge
of every split segment finds exactly the slots that were written, that no two
split segments share a ticket (their first unit), and that no segment meets
more units than the in-kernel merge holds."""
from __future__ import annotations

import numpy as np
import pytest

TILE = 128
MAX_ROUNDS = 5
IN_KERNEL_MERGE_MAX = 32


def make_sched(T, grid, min_unit):
    n = min(grid, max(T, 1))
    sizes, dyn = [], 0
    sz = T // (n * 8)
    if min_unit > 0 and sz >= min_unit:
        while len(sizes) < MAX_ROUNDS:
            cur = max(sz, min_unit)
            sizes.append(cur)
            dyn += cur * n
            if cur == min_unit:
                break
            sz >>= 1
    return {"T": T, "S": T - dyn, "n": n, "sizes": sizes}


def units(sc):
    return sc["n"] * (1 + len(sc["sizes"]))


def unit_start(sc, u):
    n, S = sc["n"], sc["S"]
    if u < n:
        return S * u // n
    off, k = S, u - n
    for size in sc["sizes"]:
        if k < n:
            return off + k * size
        off += n * size
        k -= n
    return sc["T"]


def unit_of_tile(sc, t):
    n, S = sc["n"], sc["S"]
    if t < S:
        return ((t + 1) * n - 1) // S
    off, u = t - S, n
    for size in sc["sizes"]:
        if off < n * size:
            return u + off // size
        off -= n * size
        u += n
    return u


MIN_UNIT_TILES = 8


def host_min_unit(max_seq_len, merge_in_kernel=True, floor=MIN_UNIT_TILES):
    tiles = (max_seq_len + TILE - 1) // TILE
    if not merge_in_kernel:
        return 0
    return max(floor, (tiles + 23) // 24)


def split(lengths, kv_heads, grid, min_unit, rng=None):
    nt = [(int(L) + TILE - 1) // TILE for L in lengths]
    prefix = np.concatenate([[0], np.cumsum([n * kv_heads for n in nt])]).astype(np.int64)
    total = int(prefix[-1])
    if total == 0:
        return {}, {}, nt, prefix, None
    sc = make_sched(total, grid, min_unit)
    assert sc["S"] >= sc["n"] and (total - sc["S"]) * 4 <= total
    order = list(range(units(sc)))
    if rng is not None:  # dynamic units are claimed in any order the SMs finish in
        dyn = order[sc["n"]:]
        rng.shuffle(dyn)
        order = order[:sc["n"]] + dyn
    covered = np.zeros(total, np.int64)
    written, direct = {}, set()
    for u in order:
        s, e = unit_start(sc, u), unit_start(sc, u + 1)
        assert e > s                             # every unit owns a tile
        assert unit_of_tile(sc, s) == u and unit_of_tile(sc, e - 1) == u
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
            key = (u, 0 if first_piece else 1)
            assert key not in written
            written[key] = (b, g, k0, k1)
    assert (covered == 1).all()
    assert unit_start(sc, units(sc)) == total
    return written, direct, nt, prefix, sc


def check(lengths, kv_heads, grid, min_unit=0, rng=None):
    written, direct, nt, prefix, sc = split(lengths, kv_heads, grid, min_unit, rng)
    if sc is None:
        return 0
    slot_of = lambda u, seg: 1 if unit_start(sc, u) < seg else 0  # noqa: E731
    merged, tickets = 0, set()
    for b, n in enumerate(nt):
        for g in range(kv_heads if n else 0):
            seg = int(prefix[b]) + g * n
            first, last = unit_of_tile(sc, seg), unit_of_tile(sc, seg + n - 1)
            if first == last:
                assert (b, g) in direct
                continue
            if min_unit > 0:
                assert last - first + 1 <= IN_KERNEL_MERGE_MAX
            assert first not in tickets          # one split segment per ticket
            tickets.add(first)
            pieces = [written[(u, slot_of(u, seg))] for u in range(first, last + 1)]
            assert all(p[:2] == (b, g) for p in pieces)
            spans = sorted(p[2:] for p in pieces)
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(x[1] == y[0] for x, y in zip(spans, spans[1:]))
            merged += 1
    return merged


@pytest.mark.parametrize("seed", range(200))
def test_random_shapes_static(seed):
    rng = np.random.default_rng(seed)
    B = int(rng.integers(1, 80))
    lengths = rng.integers(0, 3000, B)
    lengths[rng.random(B) < 0.1] = 0
    check(lengths, int(rng.choice([1, 2, 4, 8])), int(rng.integers(1, 257)))


@pytest.mark.parametrize("seed", range(200))
def test_random_shapes_dynamic(seed):
    rng = np.random.default_rng(1000 + seed)
    B = int(rng.integers(1, 400))
    max_len = int(rng.choice([300, 3000, 20000, 70000]))
    lengths = rng.integers(0, max_len, B)
    lengths[rng.random(B) < 0.1] = 0
    # floor 1 as well as the kernel's floor: the index math holds for any unit size
    check(lengths, int(rng.choice([1, 2, 4, 8])), int(rng.integers(1, 257)),
          host_min_unit(max_len, floor=int(rng.choice([1, MIN_UNIT_TILES]))), rng)


def test_config_shapes():
    from inference_c_b200 import workloads as W
    assert check(W.context_lengths(3, 0), 8, 148) > 0          # config 3, one GPU
    check(W.context_lengths(2, 0), 8, 148)                      # config 2
    assert check([131072], 1, 148) == 1                         # config 4 per GPU
    lengths = np.arange(1100) % 300                              # sliced launches
    check(lengths[:1024], 1, 148)
    check(lengths[1024:], 1, 148)                                # fewer tiles than CTAs


def test_config_shapes_dynamic():
    """The dynamic tail on the bench's shapes: its rounds and unit sizes."""
    from inference_c_b200 import workloads as W
    rng = np.random.default_rng(5)
    l3 = W.context_lengths(3, 0)
    assert check(l3, 8, 148, host_min_unit(int(l3.max()) + 100), rng) > 0
    sc = make_sched(int(sum((l3 + 127) // 128)) * 8, 148, host_min_unit(int(l3.max()) + 100))
    assert len(sc["sizes"]) >= 3 and sc["sizes"][-1] == host_min_unit(int(l3.max()) + 100)
    l2 = W.context_lengths(2, 0)                                # short launch: static split
    assert check(l2, 8, 148, host_min_unit(int(l2.max()) + 100), rng) > 0
    sc = make_sched(int(sum((l2 + 127) // 128)) * 8, 148, host_min_unit(int(l2.max()) + 100))
    assert not sc["sizes"]
    for shard in W.shard_by_length(l3, 8):                      # config 3 on 8 GPUs
        check(l3[shard], 8, 148, host_min_unit(int(l3.max()) + 100), rng)
