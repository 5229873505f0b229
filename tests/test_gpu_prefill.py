"""GPU parity of pkv_paged_prefill (tcgen05 chunked prefill over the paged
cache) against the oracle -- the SDK's tensor_sdpa_f32 semantics with the
causal offset kv_len - q_len -- within max-abs 2e-3 / max-rel 1e-2; at config
5's full size through one whole sequence against the SDK's own
tensor_sdpa_f32, sampled rows of the others and an exact V-scaling
property."""
from __future__ import annotations

import base64
import json
import pathlib

import numpy as np
import pytest

import inference_c_b200 as P
from inference_c_b200 import workloads as W
from tests.gpu_cases import check_close, report, sdk_paged_attention, to_device_bits, to_host_bits

pytestmark = pytest.mark.gpu
GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


class PrefillCase:
    """Pools holding `past` context tokens plus each sequence's new chunk."""

    def __init__(self, past, chunk, q_heads, kv_heads, dtype, seed, device, block_size=16,
                 streams=(1, 2, 3), pool_pages=None, head_dim=128):
        import torch
        self.past = np.asarray(past, np.int64)
        self.chunk = np.asarray(chunk, np.int64)
        self.lengths = self.past + self.chunk
        self.q_heads, self.kv_heads, self.dtype, self.bs = q_heads, kv_heads, dtype, block_size
        self.hd = head_dim
        need = int(sum((int(L) + block_size - 1) // block_size for L in self.lengths))
        self.pool_pages = pool_pages or need + 4
        self.tables, _ = W.shuffled_tables(self.lengths, block_size, self.pool_pages, seed)
        kv = kv_heads * head_dim
        rows = self.pool_pages * block_size
        self.kpool = W.normal_bits(seed, (rows, kv), dtype, stream=streams[0])
        self.vpool = W.normal_bits(seed, (rows, kv), dtype, stream=streams[1])
        self.offs = np.concatenate([[0], np.cumsum(self.chunk)]).astype(np.int32)
        self.q = W.normal_bits(seed, (int(self.offs[-1]), q_heads, head_dim), dtype,
                               stream=streams[2])
        self.device = device
        self.d_k = to_device_bits(self.kpool, dtype, device)
        self.d_v = to_device_bits(self.vpool, dtype, device)
        self.d_q = to_device_bits(self.q, dtype, device)
        self.d_tab = torch.from_numpy(self.tables.view(np.int32)).to(device)
        self.d_len = torch.from_numpy(self.lengths.astype(np.int32)).to(device)
        self.d_offs = torch.from_numpy(self.offs).to(device)

    def run(self, causal=True, out_dtype=None, scale=1 / np.sqrt(128)):
        import torch
        out = torch.full((int(self.offs[-1]), self.q_heads, self.hd), float("nan"),
                         dtype=out_dtype or torch.float32, device=self.device)
        layer = P.make_layer(self.d_k, self.d_v, self.bs, self.kv_heads, self.hd)
        P.paged_prefill(layer, P.make_batch(self.d_tab, self.d_len), self.d_q, self.d_offs, out,
                        scale, int(self.chunk.max()), causal)
        torch.cuda.synchronize()
        return out.float().cpu().numpy()

    def oracle(self, oracle_mod, causal=True, rows=None, scale=1 / np.sqrt(128)):
        want = np.zeros((int(self.offs[-1]), self.q_heads, self.hd), np.float32)
        for b in range(len(self.lengths)):
            sel = np.arange(self.offs[b], self.offs[b + 1]) if rows is None else \
                np.array([r for r in rows if self.offs[b] <= r < self.offs[b + 1]], np.int64)
            if len(sel) == 0:
                continue
            pos = self.past[b] + (sel - self.offs[b])
            want[sel] = oracle_mod.paged_attention_rows(
                self.q[sel], pos, causal, self.dtype, self.kpool, self.vpool, self.kv_heads, self.hd,
                self.bs, self.tables[b], int(self.lengths[b]), float(scale))
        return want


def test_golden_prefill_small(lib, oracle_mod, cuda):
    fx = json.loads((GOLDEN / "prefill_small.json").read_text())
    case = PrefillCase(fx["past"], fx["chunk"], fx["q_heads"], fx["kv_heads"], "bf16",
                       fx["seed"], cuda, fx["block_size"], streams=(61, 62, 63),
                       pool_pages=fx["pool_pages"])
    want = np.frombuffer(base64.b64decode(fx["out_f32_b64"]), np.float32).reshape(fx["shape"])
    check_close(case.run(True), want, "golden prefill_small (SDK tensor_sdpa_f32)")
    assert P.device_fault(0) == 0


@pytest.mark.parametrize("dtype,causal,group", [("bf16", True, 4), ("f16", True, 2),
                                                ("bf16", False, 4), ("bf16", True, 1)])
def test_prefill_matches_oracle(lib, oracle_mod, cuda, dtype, causal, group):
    """Ragged chunks across 128-row tiles, pages cut mid-tile, short and
    2k+ contexts (both P paths)."""
    case = PrefillCase([0, 300, 2100, 37], [200, 129, 130, 1], 2 * group, 2, dtype,
                       seed=10 + group, device=cuda)
    got = case.run(causal)
    check_close(got, case.oracle(oracle_mod, causal), f"{dtype} causal={causal} group={group}")
    assert P.device_fault(0) == 0


@pytest.mark.parametrize("dtype,causal,group,block", [("bf16", True, 4, 16), ("f16", True, 2, 32),
                                                      ("bf16", False, 3, 16), ("f16", True, 1, 64)])
def test_prefill_head_dim_64(lib, oracle_mod, cuda, dtype, causal, group, block):
    """head_dim 64 (one 64-column half per Q/K/V row, N=64 PV product)."""
    case = PrefillCase([0, 300, 2100, 37], [200, 129, 130, 1], 2 * group, 2, dtype,
                       seed=40 + group, device=cuda, block_size=block, head_dim=64)
    got = case.run(causal, scale=0.125)
    check_close(got, case.oracle(oracle_mod, causal, scale=0.125),
                f"d=64 {dtype} causal={causal} group={group} block={block}")
    assert P.device_fault(0) == 0


@pytest.mark.parametrize("scale", [-0.12, 0.0])
def test_prefill_nonpositive_scale(lib, oracle_mod, cuda, scale):
    """A scale <= 0 (allowed by the SDK: any finite scale) takes the general
    instantiation, which scales before the row max."""
    case = PrefillCase([0, 300], [200, 129], 8, 2, "bf16", seed=21, device=cuda)
    got = case.run(True, scale=scale)
    check_close(got, case.oracle(oracle_mod, True, scale=scale), f"scale {scale}")
    assert P.device_fault(0) == 0


def test_prefill_storage_dtype_output(lib, oracle_mod, cuda):
    import torch
    case = PrefillCase([100], [150], 8, 2, "bf16", seed=3, device=cuda)
    f32 = case.run(True)
    half = case.run(True, torch.bfloat16)
    assert np.array_equal(half, W.bf16_bits_to_f32(W.f32_to_bf16_bits(f32)))


def test_cfg5_full_size(lib, oracle_mod, cuda):
    """Config 5 at full size: 8 sequences of 8192 past + 2048 new BF16 tokens,
    GQA 32/8, causal within the chunk.  One whole sequence (all 2048 chunk
    rows x 32 heads) against the SDK's tensor_sdpa_f32 on all host threads,
    sampled rows (chunk start, tile edges, end) of the other seven against
    the oracle; doubling V doubles every output exactly."""
    import torch
    c = W.CONFIGS[5]
    case = PrefillCase([W.CFG5_PAST] * 8, [W.CFG5_CHUNK] * 8, c.q_heads, c.kv_heads, "bf16",
                       seed=5, device=cuda)
    got = case.run(True)
    assert np.isfinite(got).all()
    # sequence 3 in full: its chunk cut into 16 blocks of 128 rows, block j a
    # "sequence" of length past + 128(j + 1) with the same pages (the causal
    # offset kv_len - q_len then places its rows exactly), so the host
    # threads share the work
    b, blk = 3, 128
    nb = W.CFG5_CHUNK // blk
    r0 = int(case.offs[b])
    q_rows = np.ascontiguousarray(case.q[r0:r0 + W.CFG5_CHUNK])
    lens = W.CFG5_PAST + blk * np.arange(1, nb + 1)
    tabs = np.repeat(case.tables[b:b + 1], nb, axis=0)
    outs = sdk_paged_attention(oracle_mod, "bf16", q_rows, blk * np.arange(nb + 1), case.kpool,
                               case.vpool, c.kv_heads, 128, 16, tabs, lens, c.q_heads,
                               float(1 / np.sqrt(128)), True)
    whole = np.concatenate(outs)
    report("cfg5 sequence 3, all 2048 rows x 32 heads, vs SDK tensor_sdpa_f32",
           *check_close(got[r0:r0 + W.CFG5_CHUNK], whole, "cfg5 whole sequence"))
    rows = []
    for s in range(8):
        if s != b:
            base = int(case.offs[s])
            rows += [base + r for r in (0, 1, 127, 128, 1023, 1919, 2046, 2047)]
    want = case.oracle(oracle_mod, True, rows)
    report("cfg5 sampled rows of the other 7 sequences",
           *check_close(got[rows], want[rows], "cfg5 sampled rows"))
    case.d_v.mul_(2)
    twice = case.run(True)
    assert np.array_equal(twice, 2 * got)
    assert P.device_fault(0) == 0
