"""The C11 host layer on the GPU: a device pool attached to a cache through
the SDK's backend hook, the batch step transaction (begin_decode, length
check, reserve, device table upload, commit or rollback, end_decode), prefix
import through a step, and decode steps checked against the oracle."""
from __future__ import annotations

import numpy as np
import pytest

import inference_c_b200 as P
from inference_c_b200 import workloads as W
from tests.gpu_cases import check_close, to_device_bits, to_host_bits

pytestmark = pytest.mark.gpu


def _setup(n_seq=3, pages=64, max_pages=32, layers=2, kvh=2, d=128):
    cache = P.PagedKVCache(16, pages, 8)
    pool = P.PagedPool(cache, 0, P.PKV_DTYPE_F16, layers, kvh, d, 8, max_pages)
    seqs = [cache.sequence_create() for _ in range(n_seq)]
    return cache, pool, seqs


def dump_pool(layer: P.PkvPagedLayer, cuda):
    """Whole K and V pools in physical order, read with an identity table."""
    import torch
    pages = layer.block_count
    rows = pages * layer.block_size
    kv = layer.kv_heads * layer.head_dim
    ident = torch.arange(pages, dtype=torch.int32, device=cuda).view(1, -1)
    lens = torch.tensor([rows], dtype=torch.int32, device=cuda)
    offs = torch.tensor([0, rows], dtype=torch.int32, device=cuda)
    k = torch.empty(rows, kv, dtype=torch.float16, device=cuda)
    v = torch.empty_like(k)
    P.kv_gather(layer, P.make_batch(ident, lens), k, v, offs)
    torch.cuda.synchronize()
    return to_host_bits(k), to_host_bits(v)


def _tables(cache, seqs, width):
    tab = np.zeros((len(seqs), width), np.uint32)
    for b, s in enumerate(seqs):
        t = cache.block_table(s)
        tab[b, :len(t)] = t
    return tab


def test_pool_attaches_once_and_frees_with_cache(lib, cuda):
    cache, pool, _ = _setup()
    assert lib.pkv_pool_from_cache(cache.handle) == pool.handle
    with pytest.raises(P.PkvError, match="already has a CUDA pool"):
        P.PagedPool(cache, 0, P.PKV_DTYPE_F16, 1, 2, 128, 8, 32)
    layer = pool.layer(1)
    assert layer.block_count == 64 and layer.kv_heads == 2 and layer.head_dim == 128
    k, v = dump_pool(layer, cuda)
    assert not k.any() and not v.any()  # pools start zeroed
    cache.free()  # runs the pool's destroy callback


def test_prefix_import_then_decode_steps(lib, oracle_mod, cuda):
    import torch
    kvh, d, qh, layers = 2, 128, 8, 2
    cache, pool, seqs = _setup(kvh=kvh, d=d, layers=layers)
    past = [37, 16, 90]
    for r in range(1, 7):  # interleaved reservations: fragmented tables
        for s, L in zip(seqs, past):
            cache.reserve(s, min(L, 16 * r))
    kv = kvh * d
    host_k = [W.normal_bits(40 + l, (sum(past), kv), "f16", stream=1) for l in range(layers)]
    host_v = [W.normal_bits(40 + l, (sum(past), kv), "f16", stream=2) for l in range(layers)]
    # prefix import: every token of the prefix is new in this step
    pool.step_begin(seqs, past)
    for l in range(layers):
        P.kv_import(pool.layer(l), pool.step_batch(), to_device_bits(host_k[l], "f16", cuda),
                    to_device_bits(host_v[l], "f16", cuda), pool.step_row_offsets())
    pool.step_end(True)
    assert [cache.length(s) for s in seqs] == past
    rows = 64 * 16
    mk = [np.zeros((rows, kv), np.uint16) for _ in range(layers)]
    mv = [np.zeros((rows, kv), np.uint16) for _ in range(layers)]
    tab = _tables(cache, seqs, 32)
    assert len({int(x) for x in tab[tab > 0]}) == int((tab > 0).sum())
    offs = np.concatenate([[0], np.cumsum(past)]).astype(np.int32)
    for l in range(layers):
        oracle_mod.kv_rows(mk[l], mv[l], 16, tab, np.array(past), offs, host_k[l].copy(),
                           host_v[l].copy(), to_pool=True, tail=False)
    lengths = list(past)
    ws = P.decode_workspace(3, qh, d, 200, device=cuda)
    out = torch.empty(3, qh, d, dtype=torch.float32, device=cuda)
    for step in range(20):  # crosses a page boundary for every sequence
        pool.step_begin(seqs, [1, 1, 1])
        batch = pool.step_batch()
        lengths = [L + 1 for L in lengths]
        tab = _tables(cache, seqs, 32)
        for l in range(layers):
            nk = W.normal_bits(1000 + step * 7 + l, (3, kv), "f16", stream=3)
            nv = W.normal_bits(1000 + step * 7 + l, (3, kv), "f16", stream=4)
            q = W.normal_bits(1000 + step * 7 + l, (3, qh, d), "f16", stream=5)
            layer = pool.layer(l)
            P.kv_append(layer, batch, to_device_bits(nk, "f16", cuda),
                        to_device_bits(nv, "f16", cuda))
            P.paged_decode(layer, batch, to_device_bits(q, "f16", cuda), out,
                           float(1 / np.sqrt(d)), 200, ws)
            oracle_mod.kv_rows(mk[l], mv[l], 16, tab, np.array(lengths), None, nk.copy(),
                               nv.copy(), to_pool=True, tail=True)
            torch.cuda.synchronize()
            want = oracle_mod.paged_decode(q, "f16", mk[l], mv[l], kvh, d, 16, tab,
                                           np.array(lengths), float(1 / np.sqrt(d)))
            check_close(out.cpu().numpy(), want, f"step {step} layer {l}")
        pool.step_end(True)
    assert [cache.length(s) for s in seqs] == lengths
    for l in range(layers):
        k, v = dump_pool(pool.layer(l), cuda)
        assert np.array_equal(k, mk[l]) and np.array_equal(v, mv[l])
    assert P.device_fault(0) == 0
    cache.free()


def test_step_rollback_and_atomic_failure(lib, cuda):
    cache, pool, seqs = _setup(pages=8, max_pages=8)
    for s in seqs:
        cache.reserve(s, 16)
        cache.set_length(s, 16)
    free0 = cache.free_blocks()
    # explicit rollback: lengths and pages come back, locks are released
    pool.step_begin(seqs, [20, 1, 17])
    assert cache.free_blocks() == free0 - 5  # 36, 17, 33 tokens: 2 + 1 + 2 pages
    pool.step_end(False)
    assert cache.free_blocks() == free0 and [cache.length(s) for s in seqs] == [16, 16, 16]
    assert all(cache.begin_decode(s) for s in seqs)
    for s in seqs:
        cache.end_decode(s)
    # out of pages on the third sequence: nothing changes anywhere
    with pytest.raises(P.PkvError, match="out of pages"):
        pool.step_begin(seqs, [16, 16, 64])
    assert cache.free_blocks() == free0 and [cache.length(s) for s in seqs] == [16, 16, 16]
    # a sequence already decoding fails the whole step; the others stay unlocked
    assert cache.begin_decode(seqs[1])
    with pytest.raises(P.PkvError, match="already decoding"):
        pool.step_begin(seqs, [1, 1, 1])
    cache.end_decode(seqs[1])
    assert cache.begin_decode(seqs[0])
    cache.end_decode(seqs[0])
    # the SDK's rule: the current length must be 0 or equal to past
    with pytest.raises(P.PkvError, match="length mismatch"):
        pool.step_begin(seqs, [1, 1, 1], past_lengths=[16, 15, 16])
    assert cache.free_blocks() == free0
    # one open step at a time; release is refused while the step holds the lock
    pool.step_begin(seqs, [1, 1, 1])
    with pytest.raises(P.PkvError, match="already open"):
        pool.step_begin(seqs, [1, 1, 1])
    assert cache.release(seqs[0]) == 0
    pool.step_end(True)
    assert [cache.length(s) for s in seqs] == [17, 17, 17]
    cache.free()


def test_truncation_resends_table_rows(lib, oracle_mod, cuda):
    """After set_length drops pages and another sequence takes them, the
    next step's pages at the same logical indices differ; the device table
    must follow or appends would land in the other sequence's pages."""
    import torch
    cache, pool, seqs = _setup(n_seq=2, pages=16, max_pages=8, layers=1, kvh=1, d=64)
    a, b = seqs
    pool.step_begin([a, b], [40, 40])
    pool.step_end(True)
    cache.set_length(a, 10)           # a drops pages 1, 2
    cache.reserve(b, 80)              # b takes them
    pool.step_begin([a, b], [30, 1])  # a gets fresh pages at indices 1, 2
    batch = pool.step_batch()
    tab = _tables(cache, [a, b], 8)
    lens = np.array([40, 41])
    kv = 64
    krow = W.normal_bits(5, (31, kv), "f16", stream=1)
    vrow = W.normal_bits(5, (31, kv), "f16", stream=2)
    offs = np.array([0, 30, 31], np.int32)
    P.kv_append(pool.layer(0), batch, to_device_bits(krow, "f16", cuda),
                to_device_bits(vrow, "f16", cuda), pool.step_row_offsets())
    torch.cuda.synchronize()
    mk = np.zeros((16 * 16, kv), np.uint16)
    mv = np.zeros((16 * 16, kv), np.uint16)
    oracle_mod.kv_rows(mk, mv, 16, tab, lens, offs, krow.copy(), vrow.copy(), to_pool=True,
                       tail=True)
    k, v = dump_pool(pool.layer(0), cuda)
    assert np.array_equal(k, mk) and np.array_equal(v, mv)
    pool.step_end(True)
    assert P.device_fault(0) == 0
    cache.free()


def test_large_staging_spreads_over_ctas(lib, cuda):
    """A step that brings 5,600 new page-table entries (a prefix import of
    many pages) is applied by several staging CTAs: the rows imported through
    it must read back bit for bit through the table, and so must the rows of
    the two small steps after it (one staging CTA, both slots reused)."""
    import torch
    n, per = 8, 700  # 8 sequences x 700 pages of 16 tokens
    cache = P.PagedKVCache(16, n * (per + 2), n)
    pool = P.PagedPool(cache, 0, P.PKV_DTYPE_F16, 1, 1, 128, n, per + 2)
    layer = pool.layer(0)
    seqs = [cache.sequence_create() for _ in range(n)]
    lengths = np.array([16 * per - 3 * b for b in range(n)], np.int64)
    g = torch.Generator(device=cuda).manual_seed(11)
    rows_k = [torch.randn(int(L), 128, generator=g, device=cuda).half() for L in lengths]
    rows_v = [torch.randn(int(L), 128, generator=g, device=cuda).half() for L in lengths]

    def offsets(counts):
        return torch.from_numpy(np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)).to(cuda)

    pool.step_begin(seqs, lengths.tolist())
    P.kv_import(layer, pool.step_batch(), torch.cat(rows_k), torch.cat(rows_v), offsets(lengths))
    pool.step_end(True)
    for _ in range(2):  # one appended row per sequence per step
        nk = torch.randn(n, 128, generator=g, device=cuda).half()
        nv = torch.randn(n, 128, generator=g, device=cuda).half()
        pool.step_begin(seqs, [1] * n)
        P.kv_append(layer, pool.step_batch(), nk, nv)
        pool.step_end(True)
        for b in range(n):
            rows_k[b] = torch.cat([rows_k[b], nk[b:b + 1]])
            rows_v[b] = torch.cat([rows_v[b], nv[b:b + 1]])
    lengths = lengths + 2
    assert [cache.length(s_) for s_ in seqs] == lengths.tolist()
    pool.step_begin(seqs, [0] * n)  # read everything back through the table
    k = torch.empty(int(lengths.sum()), 128, dtype=torch.float16, device=cuda)
    v = torch.empty_like(k)
    P.kv_gather(layer, pool.step_batch(), k, v, offsets(lengths))
    torch.cuda.synchronize()
    pool.step_end(True)
    assert np.array_equal(to_host_bits(k), to_host_bits(torch.cat(rows_k)))
    assert np.array_equal(to_host_bits(v), to_host_bits(torch.cat(rows_v)))
    assert P.device_fault(0) == 0
    cache.free()


@pytest.mark.parametrize("fused", [True, False])
def test_decode_stepper_back_to_back(lib, oracle_mod, cuda, fused):
    """DecodeStepper steps queued back to back with no host synchronisation:
    the decode kernel releases its dependents early, so each step's staging
    (and, unfused, its append) launches while the previous decode still
    streams.  Every step's output (its own buffer) must match the oracle on
    the pages as they were at that step, and the pages must end bit-exact.
    A step whose decode call is refused rolls back."""
    import torch
    n, kvh, qh, d, steps = 8, 2, 8, 128, 24
    cache = P.PagedKVCache(16, 1024, n)
    pool = P.PagedPool(cache, 0, P.PKV_DTYPE_F16, 1, kvh, d, n, 160)
    layer = pool.layer(0)
    seqs = [cache.sequence_create() for _ in range(n)]
    past = [300 + 217 * b for b in range(n)]
    for r in range(1, 160):  # interleaved reservations: fragmented tables
        for s, L in zip(seqs, past):
            if 16 * (r - 1) < L:
                cache.reserve(s, min(L, 16 * r))
    kv = kvh * d
    host_k = W.normal_bits(71, (sum(past), kv), "f16", stream=1)
    host_v = W.normal_bits(71, (sum(past), kv), "f16", stream=2)
    pool.step_begin(seqs, past)
    P.kv_import(layer, pool.step_batch(), to_device_bits(host_k, "f16", cuda),
                to_device_bits(host_v, "f16", cuda), pool.step_row_offsets())
    pool.step_end(True)
    mk = np.zeros((1024 * 16, kv), np.uint16)
    mv = np.zeros_like(mk)
    offs = np.concatenate([[0], np.cumsum(past)]).astype(np.int32)
    oracle_mod.kv_rows(mk, mv, 16, _tables(cache, seqs, 160), np.array(past), offs, host_k.copy(),
                       host_v.copy(), to_pool=True, tail=False)
    nks = [W.normal_bits(500 + i, (n, kv), "f16", stream=3) for i in range(steps)]
    nvs = [W.normal_bits(500 + i, (n, kv), "f16", stream=4) for i in range(steps)]
    qs = [W.normal_bits(500 + i, (n, qh, d), "f16", stream=5) for i in range(steps)]
    dk = [to_device_bits(x, "f16", cuda) for x in nks]
    dv = [to_device_bits(x, "f16", cuda) for x in nvs]
    dq = [to_device_bits(x, "f16", cuda) for x in qs]
    outs = [torch.empty(n, qh, d, dtype=torch.float32, device=cuda) for _ in range(steps)]
    max_len = max(past) + steps + 1
    ws = P.decode_workspace(n, qh, d, max_len, device=cuda)
    scale = float(1 / np.sqrt(d))
    stepper = P.DecodeStepper(pool, layer, seqs, dq[0], dk[0], dv[0], outs[0], scale, max_len,
                              ws, fused=fused)
    for i in range(steps):
        stepper.bind(dq[i], dk[i], dv[i], outs[i])
        stepper.step()
    torch.cuda.synchronize()
    lengths = np.array(past)
    for i in range(steps):
        lengths = lengths + 1
        tab = _tables(cache, seqs, 160)
        oracle_mod.kv_rows(mk, mv, 16, tab, lengths, None, nks[i].copy(), nvs[i].copy(),
                           to_pool=True, tail=True)
        want = oracle_mod.paged_decode(qs[i], "f16", mk, mv, kvh, d, 16, tab, lengths, scale)
        check_close(outs[i].cpu().numpy(), want, f"step {i}")
    assert [cache.length(s) for s in seqs] == lengths.tolist()
    k, v = dump_pool(layer, cuda)
    assert np.array_equal(k, mk) and np.array_equal(v, mv)
    # a refused decode (workspace too small) rolls the step back
    small = torch.zeros(64, dtype=torch.uint8, device=cuda)
    bad = P.DecodeStepper(pool, layer, seqs, dq[0], dk[0], dv[0], outs[0], scale, max_len, small,
                          fused=fused)
    with pytest.raises(P.PkvError, match="workspace"):
        bad.step()
    assert [cache.length(s) for s in seqs] == lengths.tolist()
    assert all(cache.begin_decode(s) for s in seqs)
    for s in seqs:
        cache.end_decode(s)
    assert P.device_fault(0) == 0
    cache.free()
