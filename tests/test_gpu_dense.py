"""GPU parity of the dense FP16 SDPA entry points (pkv_sdpa_f16 with device
tensors, pkv_sdpa_f16_host in the SDK backend hook's host form) against the
CPU restatement of the SDK's tensor_sdpa_f32 and, where it was built, the
SDK's own tensor_sdpa_f32 and CUDA run_f16 (within max-abs 2e-3 / max-rel
1e-2 over |ref| >= 1e-2).  Covers GQA, causal with q_len < kv_len (offset
kv_len - q_len) and q_len > kv_len (offset 0), kv_len a multiple of 16 (the
tensors are the page pool) or not (the rows are copied to whole pages),
several batches, additive masks (finite, -inf entries, fully masked rows,
row strides that do or do not allow 16-byte loads), a +inf mask entry (the
CUDA backend's zero row), scales <= 0, and the refused shapes."""
from __future__ import annotations

import numpy as np
import pytest

import inference_c_b200 as P
from oracle import oracle as O
from tests.gpu_cases import check_close

pytestmark = pytest.mark.gpu


def case(B, Hq, Hkv, Lq, Lk, seed, d=128):
    rng = np.random.default_rng(seed)
    f = lambda *shape: rng.standard_normal(shape).astype(np.float16)
    return f(B, Hq, Lq, d), f(B, Hkv, Lk, d), f(B, Hkv, Lk, d)


def expected(q, k, v, scale, causal, oracle_mod):
    return oracle_mod.sdpa_f32(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32),
                               scale, causal)


@pytest.mark.parametrize("B,Hq,Hkv,Lq,Lk,causal", [
    (1, 4, 1, 1, 1, True),        # one key
    (2, 8, 2, 100, 300, True),    # kv_len not a multiple of 16: copied into pages
    (2, 8, 2, 256, 256, True),    # the tensors themselves are the page pool
    (1, 8, 8, 130, 400, False),   # MHA, no causal mask
    (3, 6, 2, 129, 129, True),    # odd group (3 query heads per KV head)
    (65, 16, 8, 16, 32, True),    # 520 (batch, KV head) sequences: two kernel launches
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


def test_host_hook_reports_a_recorded_fault(lib, oracle_mod, cuda):
    """A fault code left in the prefill kernel's fault word makes the run_f16
    hook return 0 (its output would be partial).  The code is planted from
    the host -- no kernel faults -- and the hook clears it: the next call
    succeeds and matches the oracle."""
    import ctypes
    q, k, v = case(1, 4, 2, 32, 64, seed=3)
    plant = lib.pkv_internal_plant_prefill_fault
    plant.argtypes, plant.restype = [ctypes.c_uint32], ctypes.c_int
    assert plant(4) == 1
    bits = (q.view(np.uint16), k.view(np.uint16), v.view(np.uint16))
    assert P.sdpa_f16_host(*bits, 0.1, True) is None
    got = P.sdpa_f16_host(*bits, 0.1, True)
    assert got is not None
    check_close(got.view(np.float16).astype(np.float32), expected(q, k, v, 0.1, True, oracle_mod),
                "host hook after a reported fault")
    assert P.device_fault(0) == 0


def make_mask(Lq, Lk, seed, dead_rows=()):
    """N(0, 2) additive mask with ~10 % -inf entries and fully masked rows."""
    rng = np.random.default_rng(seed)
    m = (rng.standard_normal((Lq, Lk)) * 2).astype(np.float16)
    m[rng.random((Lq, Lk)) < 0.1] = -np.inf
    for r in dead_rows:
        m[r] = -np.inf
    return m


@pytest.mark.parametrize("B,Hq,Hkv,Lq,Lk,causal", [
    (2, 8, 2, 100, 300, True),    # kv_len % 8 != 0: scalar mask loads
    (1, 8, 8, 130, 256, False),   # 16-byte mask loads, no causal mask
    (1, 4, 1, 200, 136, True),    # q_len > kv_len (causal offset 0)
    (2, 6, 2, 129, 129, False),   # odd group
])
def test_device_entry_with_mask(lib, oracle_mod, cuda, B, Hq, Hkv, Lq, Lk, causal):
    import torch
    q, k, v = case(B, Hq, Hkv, Lq, Lk, seed=B * 7000 + Lq)
    mask = make_mask(Lq, Lk, seed=Lq + Lk, dead_rows=(3, Lq - 1))
    scale = 1 / np.sqrt(128)
    dq, dk, dv = (torch.from_numpy(a).to(cuda) for a in (q, k, v))
    dm = torch.from_numpy(mask).to(cuda)
    out = torch.empty_like(dq)
    P.sdpa_f16(dq, dk, dv, out, scale, causal, mask=dm)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    want = oracle_mod.sdpa_f32(q.astype(np.float32), k.astype(np.float32),
                               v.astype(np.float32), scale, causal, mask=mask.astype(np.float32))
    check_close(got, want, f"masked B={B} Hq={Hq} Hkv={Hkv} Lq={Lq} Lk={Lk} causal={causal}")
    assert not got[:, :, 3].any() and not got[:, :, Lq - 1].any()  # fully masked rows
    assert P.device_fault(0) == 0


@pytest.mark.parametrize("Lq,Lk,causal", [(300, 100, True), (300, 100, False)])
def test_device_entry_q_longer_than_kv(lib, oracle_mod, cuda, Lq, Lk, causal):
    import torch
    q, k, v = case(1, 8, 2, Lq, Lk, seed=Lq * 3 + Lk)
    scale = 1 / np.sqrt(128)
    dq, dk, dv = (torch.from_numpy(a).to(cuda) for a in (q, k, v))
    out = torch.empty_like(dq)
    P.sdpa_f16(dq, dk, dv, out, scale, causal)
    torch.cuda.synchronize()
    check_close(out.float().cpu().numpy(), expected(q, k, v, scale, causal, oracle_mod),
                f"Lq={Lq} > Lk={Lk} causal={causal}")


@pytest.mark.parametrize("scale", [-0.09, 0.0])
def test_device_entry_nonpositive_scale(lib, oracle_mod, cuda, scale):
    import torch
    q, k, v = case(1, 8, 2, 64, 200, seed=5)
    dq, dk, dv = (torch.from_numpy(a).to(cuda) for a in (q, k, v))
    out = torch.empty_like(dq)
    P.sdpa_f16(dq, dk, dv, out, scale, True)
    torch.cuda.synchronize()
    check_close(out.float().cpu().numpy(), expected(q, k, v, scale, True, oracle_mod),
                f"scale {scale}")


def test_host_hook_with_mask(lib, oracle_mod, cuda):
    q, k, v = case(2, 8, 4, 64, 200, seed=8)
    mask = make_mask(64, 200, seed=9, dead_rows=(10,))
    got = P.sdpa_f16_host(q.view(np.uint16), k.view(np.uint16), v.view(np.uint16), 0.1, True,
                          mask=mask.view(np.uint16))
    assert got is not None
    got = got.view(np.float16).astype(np.float32)
    want = oracle_mod.sdpa_f32(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32),
                               0.1, True, mask=mask.astype(np.float32))
    check_close(got, want, "host hook with mask vs oracle")
    if O.ref_cuda_available():
        ref = O.ref_cuda_sdpa_f16(q.view(np.uint16), k.view(np.uint16), v.view(np.uint16), 0.1,
                                  True, mask=mask.view(np.uint16))
        assert ref is not None
        check_close(got, ref.view(np.float16).astype(np.float32), "host hook vs SDK CUDA sdpa")
    if O.ref_available():
        want = O.ref_sdpa_f32(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32),
                              0.1, True, mask=mask.astype(np.float32))
        check_close(got, want, "host hook vs SDK tensor_sdpa_f32 (mask)")


def test_positive_infinite_mask_row(lib, oracle_mod, cuda):
    """A +inf mask entry makes that row's maximum non-finite: zeros, as the
    SDK CUDA backend's softmax_rows_kernel gives (its CPU path would instead
    spread the row uniformly over the +inf keys)."""
    q, k, v = case(1, 4, 2, 16, 64, seed=12)
    mask = np.zeros((16, 64), np.float16)
    mask[5, 7] = np.inf
    got = P.sdpa_f16_host(q.view(np.uint16), k.view(np.uint16), v.view(np.uint16), 0.1, False,
                          mask=mask.view(np.uint16))
    assert got is not None
    got = got.view(np.float16).astype(np.float32)
    assert not got[:, :, 5].any()
    rows = [r for r in range(16) if r != 5]
    want = expected(q, k, v, 0.1, False, oracle_mod)
    check_close(got[:, :, rows], want[:, :, rows], "rows without +inf")
    if O.ref_cuda_available():
        ref = O.ref_cuda_sdpa_f16(q.view(np.uint16), k.view(np.uint16), v.view(np.uint16), 0.1,
                                  False, mask=mask.view(np.uint16))
        assert ref is not None and not ref.view(np.float16)[:, :, 5].astype(np.float32).any()


def test_refused_shapes(lib, cuda):
    q, k, v = case(1, 4, 2, 32, 16, seed=1, d=96)
    assert P.sdpa_f16_host(q.view(np.uint16), k.view(np.uint16), v.view(np.uint16), 0.1,
                           True) is None  # head_dim 96
    q, k, v = case(1, 4, 2, 32, 16, seed=1)
    v64 = np.ascontiguousarray(v[..., :64])
    assert P.sdpa_f16_host(q.view(np.uint16), k.view(np.uint16), v64.view(np.uint16), 0.1,
                           True) is None  # value_dim 64 != head_dim 128


# ---- head_dim 64 (SmolVLM-class text models: the SDK's callers read head_dim
# from the model config, tests/smolvlm/src/app/text_model.c:603-604) ----

@pytest.mark.parametrize("B,Hq,Hkv,Lq,Lk,causal", [
    (1, 4, 1, 1, 1, True),
    (2, 9, 3, 100, 300, True),    # kv_len not a multiple of 16, odd group (3)
    (2, 8, 2, 256, 256, True),    # the tensors are the page pool
    (1, 8, 8, 130, 400, False),   # MHA, no causal mask
    (1, 4, 1, 300, 100, True),    # q_len > kv_len
])
def test_head_dim_64_device_entry(lib, oracle_mod, cuda, B, Hq, Hkv, Lq, Lk, causal):
    import torch
    q, k, v = case(B, Hq, Hkv, Lq, Lk, seed=B * 31 + Lq, d=64)
    scale = 0.125
    dq, dk, dv = (torch.from_numpy(a).to(cuda) for a in (q, k, v))
    out = torch.empty_like(dq)
    P.sdpa_f16(dq, dk, dv, out, scale, causal)
    torch.cuda.synchronize()
    check_close(out.float().cpu().numpy(), expected(q, k, v, scale, causal, oracle_mod),
                f"d=64 B={B} Hq={Hq} Hkv={Hkv} Lq={Lq} Lk={Lk} causal={causal}")
    assert P.device_fault(0) == 0


def test_head_dim_64_host_hook_with_mask_against_sdk(lib, oracle_mod, cuda):
    """The run_f16 hook at head_dim 64 with an additive mask: against the
    restatement, the SDK's own tensor_sdpa_f32 and its CUDA run_f16."""
    q, k, v = case(2, 8, 2, 96, 250, seed=64, d=64)
    mask = make_mask(96, 250, seed=65, dead_rows=(7,))
    bits = (q.view(np.uint16), k.view(np.uint16), v.view(np.uint16))
    got = P.sdpa_f16_host(*bits, 0.125, True, mask=mask.view(np.uint16))
    assert got is not None
    got = got.view(np.float16).astype(np.float32)
    f32 = (q.astype(np.float32), k.astype(np.float32), v.astype(np.float32))
    check_close(got, oracle_mod.sdpa_f32(*f32, 0.125, True, mask=mask.astype(np.float32)),
                "d=64 host hook vs oracle")
    assert not got[:, :, 7].any()
    if O.ref_available():
        check_close(got, O.ref_sdpa_f32(*f32, 0.125, True, mask=mask.astype(np.float32)),
                    "d=64 host hook vs SDK tensor_sdpa_f32")
    if O.ref_cuda_available():
        ref = O.ref_cuda_sdpa_f16(*bits, 0.125, True, mask=mask.view(np.uint16))
        assert ref is not None
        check_close(got, ref.view(np.float16).astype(np.float32), "d=64 host hook vs SDK CUDA")
