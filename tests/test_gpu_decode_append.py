"""pkv_paged_decode_append: a decode step's append and paged decode in one
call.  On the tensor-core path the decode kernel's producer warps store each
sequence's new K/V row into its page just before the TMA that reads it; the
pages must come out bit-identical to pkv_kv_append's, and the outputs equal
to those of the two separate calls and within tolerance of the oracle run on
the appended pages.  Shapes cover the tensor-core kernel (static split, the
dynamic tail, the separate merge kernel, paired head_dim 64, BF16, pages of
16-64 tokens), the CUDA-core kernel (two launches behind the same call), and
new rows that open a page or a 128-token tile."""
from __future__ import annotations

import numpy as np
import pytest

import inference_c_b200 as P
from inference_c_b200 import workloads as W
from tests.gpu_cases import PagedCase, check_close, to_device_bits, to_host_bits

pytestmark = pytest.mark.gpu

# lengths after the append: 1 (the new row is the whole context), page and
# tile edges on both sides, a few long ones
EDGES = [1, 2, 15, 16, 17, 127, 128, 129, 300, 1000, 4097]


def _host_append(case: PagedCase, nk: np.ndarray, nv: np.ndarray):
    """The pools after storing row b at position lengths[b] - 1."""
    k, v = case.kpool.copy(), case.vpool.copy()
    for b, L in enumerate(case.lengths):
        if L == 0:
            continue
        pos = int(L) - 1
        row = int(case.tables[b][pos // case.block_size]) * case.block_size + pos % case.block_size
        k[row], v[row] = nk[b], nv[b]
    return k, v


def _both_paths(case: PagedCase, oracle_mod, cuda, out_dtype, max_len, seed, ws_len=None):
    import torch
    n, kv = len(case.lengths), case.kv_heads * case.head_dim
    nk = W.normal_bits(seed, (n, kv), case.dtype, stream=6)
    nv = W.normal_bits(seed, (n, kv), case.dtype, stream=7)
    d_nk, d_nv = to_device_bits(nk, case.dtype, cuda), to_device_bits(nv, case.dtype, cuda)
    ws = P.decode_workspace(n, case.q_heads, case.head_dim, ws_len or max_len, device=cuda)
    outs, pools = [], []
    for fused in (False, True):
        kp, vp = case.d_kpool.clone(), case.d_vpool.clone()
        layer = P.make_layer(kp, vp, case.block_size, case.kv_heads, case.head_dim)
        out = torch.full((n, case.q_heads, case.head_dim), float("nan"), dtype=out_dtype,
                         device=cuda)
        if fused:
            P.paged_decode_append(layer, case.batch(), d_nk, d_nv, case.d_q, out, case.scale,
                                  max_len, ws)
        else:
            P.kv_append(layer, case.batch(), d_nk, d_nv)
            P.paged_decode(layer, case.batch(), case.d_q, out, case.scale, max_len, ws)
        torch.cuda.synchronize()
        outs.append(out.float().cpu().numpy())
        pools.append((to_host_bits(kp), to_host_bits(vp)))
    hk, hv = _host_append(case, nk, nv)
    for kp, vp in pools:  # both paths store the same bits where the oracle does
        assert np.array_equal(kp, hk) and np.array_equal(vp, hv)
    # same kernel, same schedule: the outputs agree bit for bit
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    want = oracle_mod.paged_decode(case.q, case.dtype, hk, hv, case.kv_heads, case.head_dim,
                                   case.block_size, case.tables, case.lengths, case.scale)
    if out_dtype != torch.float32:
        want = torch.from_numpy(want).to(out_dtype).float().numpy()
    check_close(outs[1], want, "fused append + decode")
    assert P.device_fault(0) == 0


@pytest.mark.parametrize("q_heads,kv_heads,head_dim,block_size,dtype,out", [
    (32, 8, 128, 16, "f16", "f32"),    # config 2/3 shape
    (16, 4, 128, 32, "bf16", "bf16"),  # BF16, 32-token pages
    (16, 2, 128, 64, "f16", "f16"),    # 64-token pages
    (8, 8, 64, 16, "f16", "f32"),      # config 1 shape: paired head_dim 64
    (16, 4, 64, 16, "bf16", "f32"),    # paired, group 4
    (6, 3, 64, 16, "f16", "f32"),      # odd KV-head count: CUDA-core kernel
])
def test_fused_matches_separate_calls(lib, oracle_mod, cuda, q_heads, kv_heads, head_dim,
                                      block_size, dtype, out):
    import torch
    rng = np.random.default_rng(head_dim * 100 + block_size + kv_heads)
    lengths = np.array(EDGES + list(rng.integers(1, 3000, 9)))
    case = PagedCase(lengths, q_heads, kv_heads, head_dim, block_size, dtype, seed=81,
                     device=cuda)
    od = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[out]
    _both_paths(case, oracle_mod, cuda, od, int(lengths.max()), seed=82)


def test_fused_dynamic_tail(lib, oracle_mod, cuda):
    """Long launch (CTA shares above 64 tiles): units of the dynamic tail
    store the rows of the segments they end."""
    import torch
    rng = np.random.default_rng(83)
    lengths = rng.integers(8000, 30000, 16)
    lengths[:3] = [1, 128, 129]
    case = PagedCase(lengths, 32, 8, 128, 16, "f16", seed=84, device=cuda)
    _both_paths(case, oracle_mod, cuda, torch.float32, 30000, seed=85)


def test_fused_merge_kernel_path(lib, oracle_mod, cuda):
    """One long sequence over few KV heads: segments cut into many pieces,
    merged by the separate kernel; the row sits in the last piece."""
    import torch
    case = PagedCase([50001], 64, 8, 128, 16, "f16", seed=86, device=cuda)
    _both_paths(case, oracle_mod, cuda, torch.float32, 50001, seed=87)


def test_fused_batch_above_one_launch(lib, oracle_mod, cuda):
    """More sequences than one tensor-core launch holds (1024): each sliced
    launch reads the new rows of its own sequences."""
    import torch
    lengths = (W.uniform(5, 1100) * 300).astype(np.int64) + 1
    case = PagedCase(lengths, 4, 1, 128, 16, "f16", seed=91, device=cuda)
    _both_paths(case, oracle_mod, cuda, torch.float32, int(lengths.max()), seed=92)


def test_fused_empty_sequence_records_fault(lib, oracle_mod, cuda):
    """A sequence of length 0 has no position for its row: nothing is
    stored, its output is zero and fault code 3 is recorded (pkv_kv_append's
    rule); the other sequences are served."""
    import torch
    lengths = np.array([40, 0, 300])
    case = PagedCase(lengths, 8, 2, 128, 16, "f16", seed=88, device=cuda)
    kv = 2 * 128
    nk = W.normal_bits(89, (3, kv), "f16", stream=6)
    nv = W.normal_bits(89, (3, kv), "f16", stream=7)
    ws = P.decode_workspace(3, 8, 128, 300, device=cuda)
    out = torch.full((3, 8, 128), float("nan"), dtype=torch.float32, device=cuda)
    P.paged_decode_append(case.layer(), case.batch(), to_device_bits(nk, "f16", cuda),
                          to_device_bits(nv, "f16", cuda), case.d_q, out, case.scale, 300, ws)
    torch.cuda.synchronize()
    assert P.device_fault(0) == 3
    hk, hv = _host_append(case, nk, nv)
    assert np.array_equal(to_host_bits(case.d_kpool), hk)
    assert np.array_equal(to_host_bits(case.d_vpool), hv)
    got = out.cpu().numpy()
    assert not got[1].any()
    want = oracle_mod.paged_decode(case.q, "f16", hk, hv, 2, 128, 16, case.tables, lengths,
                                   case.scale)
    check_close(got, want, "with an empty sequence")
    assert P.device_fault(0) == 0


def test_fused_refuses_bad_rows(lib, cuda):
    import torch
    case = PagedCase([40], 8, 2, 128, 16, "f16", seed=90, device=cuda)
    ws = P.decode_workspace(1, 8, 128, 40, device=cuda)
    out = torch.empty(1, 8, 128, dtype=torch.float32, device=cuda)
    rows = torch.zeros(1, 256 + 8, dtype=torch.float16, device=cuda)
    with pytest.raises(P.PkvError, match="16-byte aligned"):
        P.paged_decode_append(case.layer(), case.batch(), rows[:, 1:], rows[:, 1:], case.d_q, out,
                              case.scale, 40, ws)
