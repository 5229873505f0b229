"""pkv_paged_decode_static_scratch: the decode entry point for callers that
cannot allocate device memory when they call it (its split-K scratch is a
static 8 MiB device array inside the library).  Called through the C ABI on
two calls in a row and compared with pkv_paged_decode (caller workspace) and
with the CPU oracle, with the tolerance the other decode tests use; a refused
call must leave the array untouched.  This file sorts last so that a run
stopping at the first failure has run every other test before it."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import inference_c_b200 as P
from tests.gpu_cases import PagedCase, check_close

pytestmark = pytest.mark.gpu


def _existing(case, out_dtype):
    import torch
    max_len = int(case.lengths.max())
    ws = P.decode_workspace(len(case.lengths), case.q_heads, case.head_dim, max_len,
                            device=case.device)
    out = torch.empty(len(case.lengths), case.q_heads, case.head_dim, dtype=out_dtype,
                      device=case.device)
    P.paged_decode(case.layer(), case.batch(), case.d_q, out, case.scale, max_len, ws)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


@pytest.mark.parametrize("q_heads,kv_heads,head_dim,dtype", [
    (32, 8, 128, "f16"),   # tcgen05 kernel (config-2 shape, shorter contexts)
    (8, 2, 64, "bf16"),    # CUDA-core kernel
])
def test_matches_workspace_entry_two_calls(lib, oracle_mod, cuda, q_heads, kv_heads, head_dim,
                                           dtype):
    import torch
    lengths = [0, 1, 17, 300, 1024, 2500]
    case = PagedCase(lengths, q_heads, kv_heads, head_dim, 16, dtype, seed=77, device=cuda)
    want = _existing(case, torch.float32)
    oracle = oracle_mod.paged_decode(case.q, case.dtype, case.kpool, case.vpool, case.kv_heads,
                                     case.head_dim, case.block_size, case.tables, case.lengths,
                                     case.scale)
    max_len = int(case.lengths.max())
    for call in range(2):  # the array keeps the last call's contents
        out = torch.full((len(lengths), q_heads, head_dim), float("nan"), dtype=torch.float32,
                         device=cuda)
        P.paged_decode_static_scratch(case.layer(), case.batch(), case.d_q, out, case.scale,
                                      max_len)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        check_close(got, want, f"static-scratch call {call} vs workspace entry")
        check_close(got, oracle, f"static-scratch call {call} vs oracle")
    assert P.device_fault(0) == 0


def test_refuses_shapes_above_the_static_maximum(lib, cuda):
    import torch
    case = PagedCase([40], 8, 1, 64, 16, "f16", seed=5, device=cuda)
    out = torch.empty(1, 8, 64, dtype=torch.float32, device=cuda)
    err = ctypes.create_string_buffer(256)
    # a CUDA-core shape (head_dim 64 with one KV head, which the tensor-core
    # kernel does not pair) declaring up to 16M positions: its per-chunk
    # partials would need ~35 MB, above the 8 MiB array
    ok = lib.pkv_paged_decode_static_scratch(ctypes.byref(case.layer()),
                                             ctypes.byref(case.batch()), 8, case.d_q.data_ptr(),
                                             ctypes.c_float(case.scale), out.data_ptr(),
                                             P.PKV_DTYPE_F32, 1 << 24, None, err, len(err))
    assert ok == 0 and b"static maximum" in err.value


def test_refused_call_leaves_the_array_alone(lib, oracle_mod, cuda):
    """A call refused for its arguments (batch 0 here) returns 0 before it
    clears any ticket; a valid call after it still matches the oracle."""
    import torch
    case = PagedCase([5, 700], 8, 2, 128, 16, "f16", seed=78, device=cuda)
    out = torch.empty(2, 8, 128, dtype=torch.float32, device=cuda)
    err = ctypes.create_string_buffer(256)
    empty = P.PkvBatch(case.batch().block_tables, case.batch().table_stride,
                       case.batch().seq_lens, 0)
    ok = lib.pkv_paged_decode_static_scratch(ctypes.byref(case.layer()), ctypes.byref(empty), 8,
                                             case.d_q.data_ptr(), ctypes.c_float(case.scale),
                                             out.data_ptr(), P.PKV_DTYPE_F32, 700, None, err,
                                             len(err))
    assert ok == 0 and b"invalid batch" in err.value
    P.paged_decode_static_scratch(case.layer(), case.batch(), case.d_q, out, case.scale, 700)
    torch.cuda.synchronize()
    want = oracle_mod.paged_decode(case.q, case.dtype, case.kpool, case.vpool, case.kv_heads,
                                   case.head_dim, case.block_size, case.tables, case.lengths,
                                   case.scale)
    check_close(out.cpu().numpy(), want, "static-scratch after a refused call")
