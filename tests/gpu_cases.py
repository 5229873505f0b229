"""Helpers shared by the GPU tests: seeded paged cases on the device and the
tolerance check the parity tests use.

Tolerance (stated by the task for attention outputs against the FP32 CPU
result): max-abs <= 2e-3 and max-rel <= 1e-2, the relative error taken over
elements with |reference| >= 1e-2 (REL_FLOOR) because near-zero references
make relative error meaningless.  Page contents, block tables and gathered
K/V are compared bit for bit.
"""
from __future__ import annotations

import numpy as np

from inference_c_b200 import workloads as W

ABS_TOL = 2e-3
REL_TOL = 1e-2
REL_FLOOR = 1e-2


def check_close(got: np.ndarray, want: np.ndarray, what: str = "") -> tuple[float, float]:
    got = np.asarray(got, dtype=np.float32)
    want = np.asarray(want, dtype=np.float32)
    assert got.shape == want.shape, (got.shape, want.shape)
    assert np.array_equal(np.isnan(got), np.isnan(want)), f"{what}: NaN pattern differs"
    ok = ~np.isnan(want)
    diff = np.abs(got[ok] - want[ok])
    max_abs = float(diff.max()) if diff.size else 0.0
    big = np.abs(want[ok]) >= REL_FLOOR
    max_rel = float((diff[big] / np.abs(want[ok][big])).max()) if big.any() else 0.0
    assert max_abs <= ABS_TOL, f"{what}: max-abs {max_abs:.3e} > {ABS_TOL}"
    assert max_rel <= REL_TOL, f"{what}: max-rel {max_rel:.3e} > {REL_TOL}"
    return max_abs, max_rel


def torch_dtype(name: str):
    import torch
    return {"f16": torch.float16, "bf16": torch.bfloat16}[name]


def to_device_bits(bits: np.ndarray, dtype: str, device):
    """uint16 storage bits (numpy) -> a CUDA tensor of that dtype, same bits."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).copy())
    return t.to(device).view(torch_dtype(dtype))


def to_host_bits(t) -> np.ndarray:
    import torch
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


class PagedCase:
    """A seeded paged batch: host bit arrays (for the oracle) and their
    device copies (for the kernels)."""

    def __init__(self, lengths, q_heads: int, kv_heads: int, head_dim: int, block_size: int,
                 dtype: str, seed: int, device, pool_pages: int | None = None,
                 extra_pages: int = 8):
        import torch
        self.lengths = np.asarray(lengths, dtype=np.int64)
        self.q_heads, self.kv_heads, self.head_dim = q_heads, kv_heads, head_dim
        self.block_size, self.dtype, self.seed = block_size, dtype, seed
        need = int(sum((int(L) + block_size - 1) // block_size for L in self.lengths))
        self.pool_pages = pool_pages or need + extra_pages
        self.tables, self.stride = W.shuffled_tables(self.lengths, block_size, self.pool_pages, seed)
        kv = kv_heads * head_dim
        rows = self.pool_pages * block_size
        self.kpool = W.normal_bits(seed, (rows, kv), dtype, stream=1)
        self.vpool = W.normal_bits(seed, (rows, kv), dtype, stream=2)
        self.q = W.normal_bits(seed, (len(self.lengths), q_heads, head_dim), dtype, stream=3)
        self.device = device
        self.d_kpool = to_device_bits(self.kpool, dtype, device)
        self.d_vpool = to_device_bits(self.vpool, dtype, device)
        self.d_q = to_device_bits(self.q, dtype, device)
        self.d_tables = torch.from_numpy(self.tables.view(np.int32)).to(device)
        self.d_lens = torch.from_numpy(self.lengths.astype(np.int32)).to(device)

    @property
    def scale(self) -> float:
        return float(1.0 / np.sqrt(self.head_dim))

    def layer(self):
        from inference_c_b200 import make_layer
        return make_layer(self.d_kpool, self.d_vpool, self.block_size, self.kv_heads,
                          self.head_dim)

    def batch(self):
        from inference_c_b200 import make_batch
        return make_batch(self.d_tables, self.d_lens)
