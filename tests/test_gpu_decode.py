"""GPU parity of pkv_paged_decode against the oracle (the SDK's
tensor_sdpa_f32 semantics on the gathered pages), within max-abs 2e-3 /
max-rel 1e-2, across GQA groups, head sizes, storage and output dtypes,
ragged and edge lengths, split-K chunking, and at full config sizes through
size-independent properties."""
from __future__ import annotations

import base64
import json
import pathlib

import numpy as np
import pytest

import inference_c_b200 as P
from inference_c_b200 import workloads as W
from tests.gpu_cases import (PagedCase, check_close, report, sdk_paged_attention, to_device_bits,
                             to_host_bits)

pytestmark = pytest.mark.gpu
GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


def _run_decode(case: PagedCase, out_dtype=None, chunk: int = 0, max_len: int | None = None):
    import torch
    out_dtype = out_dtype or torch.float32
    max_len = max_len or int(case.lengths.max(initial=0))
    ws = P.decode_workspace(len(case.lengths), case.q_heads, case.head_dim, max_len, chunk,
                            device=case.device)
    out = torch.full((len(case.lengths), case.q_heads, case.head_dim), float("nan"),
                     dtype=out_dtype, device=case.device)
    P.paged_decode(case.layer(), case.batch(), case.d_q, out, case.scale, max_len, ws, chunk)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), ws


def _round_like(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    return W.bf16_bits_to_f32(W.f32_to_bf16_bits(x))


def _oracle(case: PagedCase, oracle_mod):
    return oracle_mod.paged_decode(case.q, case.dtype, case.kpool, case.vpool, case.kv_heads,
                                   case.head_dim, case.block_size, case.tables, case.lengths,
                                   case.scale)


def test_golden_decode_small(lib, oracle_mod, cuda):
    fx = json.loads((GOLDEN / "decode_small.json").read_text())
    case = PagedCase(fx["lengths"], fx["q_heads"], fx["kv_heads"], fx["head_dim"],
                     fx["block_size"], "f16", seed=fx["seed"], device=cuda,
                     pool_pages=fx["pool_pages"])
    # PagedCase draws its pools with streams 1/2/3; the fixture used 51/52/53
    kv = fx["kv_heads"] * fx["head_dim"]
    rows = fx["pool_pages"] * fx["block_size"]
    case.kpool = W.normal_bits(fx["seed"], (rows, kv), "f16", stream=51)
    case.vpool = W.normal_bits(fx["seed"], (rows, kv), "f16", stream=52)
    case.q = W.normal_bits(fx["seed"], (len(fx["lengths"]), fx["q_heads"], fx["head_dim"]), "f16",
                           stream=53)
    case.d_kpool = to_device_bits(case.kpool, "f16", cuda)
    case.d_vpool = to_device_bits(case.vpool, "f16", cuda)
    case.d_q = to_device_bits(case.q, "f16", cuda)
    want = np.frombuffer(base64.b64decode(fx["out_f32_b64"]), np.float32).reshape(fx["shape"])
    got, _ = _run_decode(case)
    check_close(got, want, "golden decode_small")


@pytest.mark.parametrize("group,head_dim,dtype", [
    (1, 64, "f16"), (2, 64, "bf16"), (4, 128, "f16"), (8, 128, "f16"), (4, 64, "bf16"),
    (8, 64, "f16"), (1, 128, "bf16"), (2, 128, "f16")])
def test_decode_matches_oracle(lib, oracle_mod, cuda, group, head_dim, dtype):
    import torch
    kvh = 2
    lengths = [0, 1, 2, 15, 16, 17, 63, 64, 65, 200, 777]
    case = PagedCase(lengths, kvh * group, kvh, head_dim, 16, dtype, seed=group * 100 + head_dim,
                     device=cuda)
    want = _oracle(case, oracle_mod)
    for chunk in (0, 64, 128):
        got, _ = _run_decode(case, torch.float32, chunk)
        check_close(got, want, f"group {group} d {head_dim} {dtype} chunk {chunk}")
        # a storage-dtype output is the same FP32 result rounded to nearest even
        half, _ = _run_decode(case, case.d_q.dtype, chunk)
        assert np.array_equal(half, _round_like(got, dtype)), f"{dtype} output rounding"
    assert P.device_fault(0) == 0


@pytest.mark.parametrize("group,block_size,dtype", [
    (16, 16, "f16"), (4, 32, "bf16"), (8, 64, "f16"), (2, 128, "f16")])
def test_tcgen05_shapes(lib, oracle_mod, cuda, group, block_size, dtype):
    """GQA 16 and page sizes 32..128 (tcgen05 path only, head_dim 128)."""
    import torch
    lengths = [1, 127, 128, 129, 300, 1000]
    case = PagedCase(lengths, 2 * group, 2, 128, block_size, dtype, seed=group + block_size,
                     device=cuda)
    want = _oracle(case, oracle_mod)
    for chunk in (0, 128, 256):
        got, _ = _run_decode(case, torch.float32, chunk)
        check_close(got, want, f"group {group} block {block_size} chunk {chunk}")
    assert P.device_fault(0) == 0


@pytest.mark.parametrize("group,kv_heads,block_size,dtype", [
    (1, 8, 16, "f16"),     # config 1's shape: MHA 8 heads, head_dim 64
    (2, 2, 16, "bf16"), (4, 4, 32, "f16"), (8, 2, 16, "bf16"), (2, 6, 64, "f16")])
def test_tcgen05_head_dim_64_paired(lib, oracle_mod, cuda, group, kv_heads, block_size, dtype):
    """head_dim 64 on the tensor cores: KV heads 2g and 2g+1 run as one
    128-column segment (block-diagonal query tile).  Ragged lengths, a
    split over many CTAs, pages of 16-64 tokens, storage-dtype output."""
    import torch
    lengths = [0, 1, 15, 16, 17, 127, 128, 129, 700, 5000]
    case = PagedCase(lengths, kv_heads * group, kv_heads, 64, block_size, dtype,
                     seed=300 + 7 * group + kv_heads, device=cuda)
    want = _oracle(case, oracle_mod)
    got, _ = _run_decode(case, torch.float32)
    check_close(got, want, f"d=64 paired group {group} kv {kv_heads} block {block_size}")
    half, _ = _run_decode(case, case.d_q.dtype)
    assert np.array_equal(half, _round_like(got, dtype)), "storage-dtype output rounding"
    assert P.device_fault(0) == 0


def test_tcgen05_head_dim_64_one_long_sequence(lib, oracle_mod, cuda):
    """One long sequence at head_dim 64 with two KV heads: one segment cut
    into a piece per CTA, merged by the separate merge kernel (paired
    outputs of 64 dims)."""
    import torch
    case = PagedCase([40000, 3], 8, 2, 64, 16, "f16", seed=31, device=cuda)
    want = _oracle(case, oracle_mod)
    got, _ = _run_decode(case, torch.float32)
    check_close(got, want, "d=64 wide split")
    assert P.device_fault(0) == 0


def test_wide_split_uses_merge_kernel(lib, oracle_mod, cuda):
    """One KV head and one long sequence: every CTA takes a piece of the same
    (sequence, head) segment, so the separate merge kernel combines ~148
    partials (config 4's per-GPU shape after the head split)."""
    import torch
    case = PagedCase([40000, 3], 8, 1, 128, 16, "f16", seed=21, device=cuda)
    want = _oracle(case, oracle_mod)
    got, _ = _run_decode(case, torch.float32)
    check_close(got, want, "wide split")
    assert P.device_fault(0) == 0


def test_batch_above_one_launch(lib, oracle_mod, cuda):
    """More sequences than one tcgen05 launch holds (1024): sliced launches."""
    import torch
    lengths = (W.uniform(5, 1100) * 300).astype(np.int64)
    case = PagedCase(lengths, 4, 1, 128, 16, "f16", seed=22, device=cuda)
    want = _oracle(case, oracle_mod)
    got, _ = _run_decode(case, torch.float32)
    check_close(got, want, "1100 sequences")


@pytest.mark.parametrize("group,head_dim", [(1, 128), (4, 128), (8, 128), (2, 64), (4, 64)])
def test_simt_kernel_forced(lib, oracle_mod, cuda, monkeypatch, group, head_dim):
    """The CUDA-core kernel (forced) on shapes the tcgen05 kernel serves."""
    import torch
    monkeypatch.setenv("PKV_DECODE_KERNEL", "simt")
    lengths = [0, 1, 16, 17, 200, 777]
    case = PagedCase(lengths, 2 * group, 2, head_dim, 16, "f16", seed=50 + group,
                     device=cuda)
    want = _oracle(case, oracle_mod)
    for chunk in (0, 128):
        got, _ = _run_decode(case, torch.float32, chunk)
        check_close(got, want, f"simt group {group} chunk {chunk}")


def test_decode_ignores_poison_past_length(lib, oracle_mod, cuda):
    """Slots past a sequence's length (the tail of its last page) hold NaN
    here; they must not reach the output."""
    import torch
    lengths = [1, 17, 100, 333]
    case = PagedCase(lengths, 8, 2, 128, 16, "f16", seed=5, device=cuda)
    want = _oracle(case, oracle_mod)
    nan16 = np.uint16(0x7E00)
    for b, L in enumerate(lengths):
        for pos in range(L, ((L + 15) // 16) * 16):
            row = int(case.tables[b, pos // 16]) * 16 + pos % 16
            case.kpool[row] = nan16
            case.vpool[row] = nan16
    unused = sorted(set(range(case.pool_pages)) - set(case.tables[case.tables > 0].tolist()))
    case.d_kpool.copy_(to_device_bits(case.kpool, "f16", cuda))
    case.d_vpool.copy_(to_device_bits(case.vpool, "f16", cuda))
    for chunk in (0, 64):
        got, _ = _run_decode(case, torch.float32, chunk)
        check_close(got, want, f"poisoned tail chunk {chunk}")
    assert unused is not None


def test_nan_inside_length_propagates_like_sdk(lib, oracle_mod, cuda):
    import torch
    case = PagedCase([40], 4, 1, 64, 16, "f16", seed=8, device=cuda)
    row = int(case.tables[0, 1]) * 16 + 3  # position 19
    case.vpool[row, 5] = np.uint16(0x7E00)
    case.d_vpool.copy_(to_device_bits(case.vpool, "f16", cuda))
    want = _oracle(case, oracle_mod)
    got, _ = _run_decode(case, torch.float32)
    assert np.isnan(want[0, :, 5]).all() and not np.isnan(np.delete(want[0], 5, axis=1)).any()
    check_close(got, want, "NaN in V")


def test_workspace_stays_reusable(lib, oracle_mod, cuda):
    """Split-K tickets reset themselves: the same scratch serves many calls."""
    import torch
    case = PagedCase([300, 5, 1000], 8, 2, 128, 16, "f16", seed=9, device=cuda)
    want = _oracle(case, oracle_mod)
    ws = P.decode_workspace(3, 8, 128, 1000, 64, device=cuda)
    out = torch.empty(3, 8, 128, dtype=torch.float32, device=cuda)
    for _ in range(5):
        out.fill_(float("nan"))
        P.paged_decode(case.layer(), case.batch(), case.d_q, out, case.scale, 1000, ws, 64)
        torch.cuda.synchronize()
        check_close(out.cpu().numpy(), want, "repeat")
    counters = ws[: 256 + 6144].cpu().numpy()  # claim words and tickets
    assert not counters.any()


def test_workspace_serves_growing_batches(lib, oracle_mod, cuda):
    """One scratch, made once for the largest batch, serves calls whose batch
    grows and shrinks: the tickets and the dynamic tail's claim words sit at
    fixed offsets, never where an earlier call left partials.  Every call has
    enough segments for in-kernel merges; the long ones (16 sequences of up to
    30k tokens, ~100 tiles a CTA) also run the dynamic tail."""
    import torch
    ws = P.decode_workspace(16, 32, 128, 30000, device=cuda)
    for b, top, seed in [(10, 3000, 61), (16, 30000, 62), (10, 3000, 63), (16, 30000, 64)]:
        rng = np.random.default_rng(seed)
        case = PagedCase(rng.integers(1, top, b), 32, 8, 128, 16, "f16", seed=seed, device=cuda)
        out = torch.full((b, 32, 128), float("nan"), dtype=torch.float32, device=cuda)
        P.paged_decode(case.layer(), case.batch(), case.d_q, out, case.scale, 30000, ws)
        torch.cuda.synchronize()
        check_close(out.cpu().numpy(), _oracle(case, oracle_mod), f"batch {b}")
        assert not ws[: 256 + 6144].cpu().numpy().any()
    assert P.device_fault(0) == 0


def test_cfg2_full_size(lib, oracle_mod, cuda):
    """Config 2 at its full size (B=32, GQA 32/8, d=128, L~U[1024,4096])."""
    c = W.CONFIGS[2]
    lengths = W.context_lengths(2, seed=1)
    case = PagedCase(lengths, c.q_heads, c.kv_heads, c.head_dim, c.block_size, "f16", seed=1,
                     device=cuda)
    want = _oracle(case, oracle_mod)
    got, _ = _run_decode(case)
    check_close(got, want, "cfg2")


def test_cfg4_single_long_sequence(lib, oracle_mod, cuda):
    """Config 4 shape on one GPU: one 131072-token sequence, GQA 64/8."""
    c = W.CONFIGS[4]
    case = PagedCase([W.CFG4_TOKENS], c.q_heads, c.kv_heads, c.head_dim, 16, "f16", seed=4,
                     device=cuda)
    want = _oracle(case, oracle_mod)
    got, _ = _run_decode(case)
    check_close(got, want, "cfg4")


def test_cfg3_full_size_properties(lib, oracle_mod, cuda):
    """Config 3 at full size (B=256, ~9.7 GB of pages).  Parity of every
    sequence of the launch against the SDK's tensor_sdpa_f32 (all host
    threads, 32 sequences at a time), and two size-independent properties
    on all of them: doubling V doubles the output exactly, and moving every
    page to another physical slot (same logical content) changes nothing."""
    import torch
    c = W.CONFIGS[3]
    lengths = W.context_lengths(3, seed=3)
    pages = (lengths + 15) // 16
    pool_pages = int(pages.sum() * 1.1) + 16
    tables, stride = W.shuffled_tables(lengths, 16, pool_pages, seed=3)
    g = torch.Generator(device=cuda).manual_seed(3)
    rows = pool_pages * 16
    kpool = torch.randn(rows, c.kv_width, generator=g, device=cuda).half()
    vpool = torch.randn(rows, c.kv_width, generator=g, device=cuda).half()
    q = torch.randn(len(lengths), c.q_heads, c.head_dim, generator=g, device=cuda).half()
    d_tables = torch.from_numpy(tables.view(np.int32)).to(cuda)
    d_lens = torch.from_numpy(lengths.astype(np.int32)).to(cuda)
    max_len = int(lengths.max())
    ws = P.decode_workspace(len(lengths), c.q_heads, c.head_dim, max_len, device=cuda)
    out = torch.empty(len(lengths), c.q_heads, c.head_dim, dtype=torch.float32, device=cuda)
    layer = P.make_layer(kpool, vpool, 16, c.kv_heads, c.head_dim)
    P.paged_decode(layer, P.make_batch(d_tables, d_lens), q, out, c.scale, max_len, ws)
    torch.cuda.synchronize()
    base = out.cpu().numpy()
    assert np.isfinite(base).all()
    # parity of all 256 sequences: each group's pages are gathered on the
    # device into a compact pool (identity tables) and copied to the host
    want = np.zeros_like(base)
    hq = to_host_bits(q)
    for g0 in range(0, len(lengths), 32):
        grp = np.arange(g0, min(g0 + 32, len(lengths)))
        npg = pages[grp]
        first = np.concatenate([[0], np.cumsum(npg)])
        ids = np.concatenate([tables[b, :int(pages[b])] for b in grp]).astype(np.int64)
        idx = torch.from_numpy(ids).to(cuda)
        sel = (idx[:, None] * 16 + torch.arange(16, device=cuda)[None, :]).reshape(-1)
        hk, hv = to_host_bits(kpool[sel]), to_host_bits(vpool[sel])
        ctab = np.zeros((len(grp), int(npg.max())), np.uint32)
        for i in range(len(grp)):
            ctab[i, :int(npg[i])] = np.arange(first[i], first[i + 1], dtype=np.uint32)
        outs = sdk_paged_attention(oracle_mod, "f16", np.ascontiguousarray(hq[grp]), None, hk, hv,
                                   c.kv_heads, c.head_dim, 16, ctab, lengths[grp], c.q_heads,
                                   c.scale, False)
        for i, b in enumerate(grp):
            want[b] = outs[i][0]
    report("cfg3 all 256 sequences vs SDK tensor_sdpa_f32", *check_close(base, want, "cfg3"))
    # property 1: V -> 2V doubles the output bit for bit
    vpool.mul_(2)
    P.paged_decode(layer, P.make_batch(d_tables, d_lens), q, out, c.scale, max_len, ws)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), 2 * base)
    vpool.div_(2)
    # property 2: relocate every page (new ids, same content)
    perm = W.permutation(77, pool_pages, stream=5)
    inv = torch.from_numpy(np.argsort(perm)).to(cuda)
    kv_rows = torch.arange(rows, device=cuda).view(pool_pages, 16)
    new_order = kv_rows[inv].reshape(-1)
    k2, v2 = kpool[new_order], vpool[new_order]
    t2 = torch.from_numpy(perm.astype(np.int64)).to(cuda)[d_tables.long()].int()
    t2 = torch.where(torch.arange(stride, device=cuda)[None, :] < torch.from_numpy(
        pages).to(cuda)[:, None], t2, torch.zeros_like(t2))
    del kpool, vpool
    layer2 = P.make_layer(k2, v2, 16, c.kv_heads, c.head_dim)
    P.paged_decode(layer2, P.make_batch(t2.contiguous(), d_lens), q, out, c.scale, max_len, ws)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), base)
    assert P.device_fault(0) == 0
