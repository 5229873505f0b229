"""GPU parity of the dense FP16 SDPA entry points (pkv_sdpa_f16 with device
tensors, pkv_sdpa_f16_host in the SDK backend hook's host form) against the
CPU restatement of the SDK's tensor_sdpa_f32 and, where it was built, the
SDK's own tensor_sdpa_f32 (within max-abs 2e-3 / max-rel 1e-2 over
|ref| >= 1e-2).  Covers GQA, causal with q_len < kv_len (offset kv_len -
q_len), kv_len a multiple of 16 (the tensors are the page pool) or not (the
rows are copied to whole pages), several batches, and the refused shapes."""
from __future__ import annotations

import numpy as np
import pytest

import inference_c_b200 as P
from oracle import oracle as O
from tests.gpu_cases import check_close

pytestmark = pytest.mark.gpu


def case(B, Hq, Hkv, Lq, Lk, seed):
    rng = np.random.default_rng(seed)
    f = lambda *shape: rng.standard_normal(shape).astype(np.float16)
    return f(B, Hq, Lq, 128), f(B, Hkv, Lk, 128), f(B, Hkv, Lk, 128)


def expected(q, k, v, scale, causal, oracle_mod):
    return oracle_mod.sdpa_f32(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32),
                               scale, causal)


@pytest.mark.parametrize("B,Hq,Hkv,Lq,Lk,causal", [
    (1, 4, 1, 1, 1, True),        # one key
    (2, 8, 2, 100, 300, True),    # kv_len not a multiple of 16: copied into pages
    (2, 8, 2, 256, 256, True),    # the tensors themselves are the page pool
    (1, 8, 8, 130, 400, False),   # MHA, no causal mask
    (3, 6, 2, 129, 129, True),    # odd group (3 query heads per KV head)
])
def test_device_entry_matches_oracle(lib, oracle_mod, cuda, B, Hq, Hkv, Lq, Lk, causal):
    import torch
    q, k, v = case(B, Hq, Hkv, Lq, Lk, seed=B * 1000 + Lq)
    scale = 1 / np.sqrt(128)
    dq, dk, dv = (torch.from_numpy(a).to(cuda) for a in (q, k, v))
    out = torch.empty_like(dq)
    P.sdpa_f16(dq, dk, dv, out, scale, causal)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    want = expected(q, k, v, scale, causal, oracle_mod)
    check_close(got, want, f"dense B={B} Hq={Hq} Hkv={Hkv} Lq={Lq} Lk={Lk} causal={causal}")
    assert P.device_fault(0) == 0


def test_host_hook_and_sdk_cpu(lib, oracle_mod, cuda):
    q, k, v = case(2, 8, 4, 64, 200, seed=7)
    scale = 0.1
    got = P.sdpa_f16_host(q.view(np.uint16), k.view(np.uint16), v.view(np.uint16), scale, True)
    assert got is not None
    got = got.view(np.float16).astype(np.float32)
    check_close(got, expected(q, k, v, scale, True, oracle_mod), "host hook vs oracle")
    if O.ref_cuda_available():  # the SDK's own CUDA backend (run_f16) on the same GPU
        ref = O.ref_cuda_sdpa_f16(q.view(np.uint16), k.view(np.uint16), v.view(np.uint16), scale,
                                  True)
        assert ref is not None
        check_close(got, ref.view(np.float16).astype(np.float32), "host hook vs SDK CUDA sdpa")
    if O.ref_available():  # the SDK's own tensor_sdpa_f32
        want = O.ref_sdpa_f32(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32),
                              scale, True)
        check_close(got, want, "host hook vs SDK tensor_sdpa_f32")


def test_refused_shapes(lib, cuda):
    q, k, v = case(1, 4, 2, 32, 16, seed=1)  # q_len > kv_len
    assert P.sdpa_f16_host(q.view(np.uint16), k.view(np.uint16), v.view(np.uint16), 0.1,
                           True) is None
    q, k, v = case(1, 4, 2, 8, 16, seed=2)
    mask = np.zeros((8, 16), np.float16).view(np.uint16)
    assert P.sdpa_f16_host(q.view(np.uint16), k.view(np.uint16), v.view(np.uint16), 0.1, True,
                           mask=mask) is None
