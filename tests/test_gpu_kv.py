"""GPU parity of the KV append / import / gather kernels: bit-exact against the
oracle's page addressing, including config 1 end to end (512 one-token
appends, then the pool hashed and compared with the SDK-generated fixture)."""
from __future__ import annotations

import base64
import hashlib
import json
import pathlib

import numpy as np
import pytest

import inference_c_b200 as P
from inference_c_b200 import workloads as W
from tests.gpu_cases import PagedCase, check_close, to_device_bits, to_host_bits

pytestmark = pytest.mark.gpu
GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


def test_cfg1_append_then_decode(lib, oracle_mod, cuda):
    import torch
    fx = json.loads((GOLDEN / "cfg1.json").read_text())
    c = W.CONFIGS[1]
    seed = fx["seed"]
    table = W.cfg1_table(seed)
    rows = W.CFG1_POOL_PAGES * c.block_size
    kpool = torch.zeros(rows, c.kv_width, dtype=torch.float16, device=cuda)
    vpool = torch.zeros_like(kpool)
    krows = to_device_bits(W.normal_bits(seed, (W.CFG1_TOKENS, c.kv_width), "f16", stream=41),
                           "f16", cuda)
    vrows = to_device_bits(W.normal_bits(seed, (W.CFG1_TOKENS, c.kv_width), "f16", stream=42),
                           "f16", cuda)
    q = to_device_bits(W.normal_bits(seed, (1, c.q_heads, c.head_dim), "f16", stream=43), "f16",
                       cuda)
    tables = torch.from_numpy(table.view(np.int32).reshape(1, -1)).to(cuda)
    layer = P.make_layer(kpool, vpool, c.block_size, c.kv_heads, c.head_dim)
    lens = torch.zeros(1, dtype=torch.int32, device=cuda)
    for t in range(W.CFG1_TOKENS):
        lens.fill_(t + 1)
        P.kv_append(layer, P.make_batch(tables, lens), krows[t:t + 1], vrows[t:t + 1])
    torch.cuda.synchronize()
    assert P.device_fault(0) == 0
    assert hashlib.sha256(to_host_bits(kpool).tobytes()).hexdigest() == fx["k_pool_sha256"]
    assert hashlib.sha256(to_host_bits(vpool).tobytes()).hexdigest() == fx["v_pool_sha256"]
    want = np.frombuffer(base64.b64decode(fx["decode_out_f32_b64"]), np.float32).reshape(
        fx["shape"])
    ws = P.decode_workspace(1, c.q_heads, c.head_dim, W.CFG1_TOKENS, device=cuda)
    for out_dtype in (torch.float32, torch.float16):
        out = torch.empty(1, c.q_heads, c.head_dim, dtype=out_dtype, device=cuda)
        P.paged_decode(layer, P.make_batch(tables, lens), q, out, c.scale, W.CFG1_TOKENS, ws)
        torch.cuda.synchronize()
        check_close(out[0].float().cpu().numpy(), want, f"cfg1 decode {out_dtype}")


@pytest.mark.parametrize("dtype,block_size,kv_heads,head_dim", [
    ("f16", 16, 8, 128), ("bf16", 16, 2, 128), ("f16", 12, 4, 64), ("bf16", 1, 1, 64)])
def test_append_import_gather_bitexact(lib, oracle_mod, cuda, dtype, block_size, kv_heads,
                                       head_dim):
    import torch
    lengths = np.array([0, 1, 5, block_size, block_size + 1, 3 * block_size + 7])
    case = PagedCase(lengths, kv_heads, kv_heads, head_dim, block_size, dtype, seed=17,
                     device=cuda)
    kv = kv_heads * head_dim
    # import every prefix, then gather it back: identity
    offs = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    total = int(offs[-1])
    krows = W.normal_bits(23, (total, kv), dtype, stream=4)
    vrows = W.normal_bits(23, (total, kv), dtype, stream=5)
    d_offs = torch.from_numpy(offs).to(cuda)
    layer, batch = case.layer(), case.batch()
    P.kv_import(layer, batch, to_device_bits(krows, dtype, cuda), to_device_bits(vrows, dtype, cuda),
                d_offs)
    kg = torch.empty(total, kv, dtype=case.d_kpool.dtype, device=cuda)
    vg = torch.empty_like(kg)
    P.kv_gather(layer, batch, kg, vg, d_offs)
    torch.cuda.synchronize()
    assert np.array_equal(to_host_bits(kg), krows) and np.array_equal(to_host_bits(vg), vrows)
    hk, hv = case.kpool.copy(), case.vpool.copy()
    oracle_mod.kv_rows(hk, hv, block_size, case.tables, lengths, offs, krows.copy(), vrows.copy(),
                       to_pool=True, tail=False)
    assert np.array_equal(to_host_bits(case.d_kpool), hk)
    assert np.array_equal(to_host_bits(case.d_vpool), hv)
    # ragged multi-row append at the tail (2 rows, 0 rows, ...)
    n_new = np.minimum(lengths, np.array([0, 1, 2, 3, 1, 9]))
    aoffs = np.concatenate([[0], np.cumsum(n_new)]).astype(np.int32)
    ak = W.normal_bits(29, (int(aoffs[-1]), kv), dtype, stream=6)
    av = W.normal_bits(29, (int(aoffs[-1]), kv), dtype, stream=7)
    P.kv_append(layer, batch, to_device_bits(ak, dtype, cuda), to_device_bits(av, dtype, cuda),
                torch.from_numpy(aoffs).to(cuda))
    torch.cuda.synchronize()
    oracle_mod.kv_rows(hk, hv, block_size, case.tables, lengths, aoffs, ak.copy(), av.copy(),
                       to_pool=True, tail=True)
    assert np.array_equal(to_host_bits(case.d_kpool), hk)
    assert np.array_equal(to_host_bits(case.d_vpool), hv)
    assert P.device_fault(0) == 0


def test_out_of_range_page_is_reported_not_written(lib, cuda):
    """A block-table entry past the pool is skipped by the kernel's bounds
    check and reported through pkv_device_fault; nothing is written."""
    import torch
    case = PagedCase([20], 2, 2, 64, 16, "f16", seed=3, device=cuda)
    before = to_host_bits(case.d_kpool).copy()
    bad = case.d_tables.clone()
    bad[0, 1] = case.pool_pages + 5  # position 19 lives on logical page 1
    rows = torch.zeros(1, 128, dtype=torch.float16, device=cuda)
    P.kv_append(case.layer(), P.make_batch(bad, case.d_lens), rows, rows)
    torch.cuda.synchronize()
    assert P.device_fault(0) == 1
    assert P.device_fault(0) == 0  # cleared by the read
    assert np.array_equal(to_host_bits(case.d_kpool), before)
