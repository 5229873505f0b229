"""CPU model of the prefill kernel's item order (item_order in
inference_c_b200/csrc/pkv_prefill.cu): each CTA walks rounds of gridDim.x
consecutive items, in the dense layout with the CTA order reversed every
other round, and stops at the first item past the end.  Checks that every
item is taken exactly once, for any grid and item count, and that the
serpentine order balances config 7 (one causal 4096-row sequence per KV head,
items longest first) the way the kernel's comment states."""
from __future__ import annotations

import numpy as np
import pytest


def item_order(k: int, cta: int, grid: int, serpentine: bool) -> int:
    c = grid - 1 - cta if serpentine and (k & 1) else cta
    return k * grid + c


def items_of(cta: int, grid: int, total: int, serpentine: bool) -> list[int]:
    out, k = [], 0
    while True:
        u = item_order(k, cta, grid, serpentine)
        if u >= total:
            return out
        out.append(u)
        k += 1


@pytest.mark.parametrize("seed", range(50))
def test_every_item_once(seed):
    rng = np.random.default_rng(seed)
    grid = int(rng.integers(1, 300))
    total = int(rng.integers(0, 5000))
    for serpentine in (False, True):
        seen = np.zeros(total, np.int64)
        for cta in range(grid):
            for u in items_of(cta, grid, total, serpentine):
                seen[u] += 1
        assert (seen == 1).all()


def test_serpentine_balances_config7():
    # 32 query tiles x 16 head pairs, longest first: item u has 32 - u // 16 key tiles
    grid, total = 148, 512
    size = lambda u: 32 - u // 16  # noqa: E731
    loads = {s: [sum(size(u) for u in items_of(c, grid, total, s)) for c in range(grid)]
             for s in (False, True)}
    mean = sum(size(u) for u in range(total)) / grid
    assert max(loads[False]) == 74 and round(mean) == 57
    assert max(loads[True]) <= 60
