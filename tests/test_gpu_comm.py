"""The NCCL all-gather with a deadline against the real NCCL on one GPU:
a communicator of two ranks whose second rank never joins.  pkv_comm_init
must give up at its deadline (no GPU work is issued before every rank has
joined, so nothing waits on the device), and the decode step that needed
the collective is ended without commit: the sequence keeps its length and
pages, and its decode lock is free again.  NVLS stays off in NCCL here."""
from __future__ import annotations

import ctypes
import os
import time

import numpy as np
import pytest

import inference_c_b200 as P

pytestmark = pytest.mark.gpu


@pytest.mark.timeout(120)
def test_missing_peer_times_out_and_the_step_rolls_back(lib, cuda):
    import torch
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    cache = P.PagedKVCache(16, 64, 2)
    pool = P.PagedPool(cache, 0, P.PKV_DTYPE_F16, 1, 2, 128, 2, 16)
    seq = cache.sequence_create()
    pool.step_begin([seq], [40])
    pool.step_end(True)
    free0 = cache.free_blocks()
    layer = pool.layer(0)
    k = torch.randn(1, 256, device=cuda).half()
    q = torch.randn(1, 8, 128, device=cuda).half()
    out = torch.empty(1, 8, 128, device=cuda, dtype=torch.float32)
    ws = P.decode_workspace(1, 8, 128, 64, device=cuda)
    pool.step_begin([seq], [1])
    b = pool.step_batch()
    P.kv_append(layer, b, k, k)
    P.paged_decode(layer, b, q, out, 0.1, 64, ws)
    t0 = time.monotonic()
    with pytest.raises(P.PkvError, match="to join"):
        P.Comm(P.comm_unique_id(), 2, 0, 0, timeout_s=2.0)
    took = time.monotonic() - t0
    pool.step_end(False)  # the collective failed: roll the step back
    torch.cuda.synchronize()
    assert 1.9 <= took < 60
    assert cache.length(seq) == 40 and cache.free_blocks() == free0
    assert cache.begin_decode(seq)  # the lock was released
    cache.end_decode(seq)
    assert np.isfinite(out.cpu().numpy()).all()
    assert P.device_fault(0) == 0
