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


def host_threads() -> int:
    import os
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:  # pragma: no cover
        return max(1, os.cpu_count() or 1)


def sdk_paged_attention(oracle_mod, dtype: str, q: np.ndarray, q_offsets, kpool: np.ndarray,
                        vpool: np.ndarray, kv_heads: int, head_dim: int, block_size: int,
                        tables: np.ndarray, seq_lens: np.ndarray, q_heads: int, scale: float,
                        causal: bool) -> list[np.ndarray]:
    """Attention of every sequence of a paged batch, on all host threads:
    the SDK's own tensor_sdpa_f32 (oracle/_ref, through RefJob) where it was
    built, else the CPU restatement (which matches it bit for bit).  q holds
    storage bits, [rows][q_heads][head_dim]; q_offsets (None: one row per
    sequence) gives each sequence's rows, its last positions.  Returns one
    float32 [rows_b][q_heads][head_dim] array per sequence."""
    from concurrent.futures import ThreadPoolExecutor
    n = len(seq_lens)
    offs = np.arange(n + 1) if q_offsets is None else np.asarray(q_offsets, np.int64)
    if oracle_mod.ref_available():
        job = oracle_mod.RefJob(dtype, q, None if q_offsets is None else offs.astype(np.int32),
                                kpool, vpool, kv_heads, head_dim, block_size, tables, seq_lens,
                                q_heads, scale, causal)
        try:
            job.run(host_threads())
            return [job.output(i) for i in range(n)]
        finally:
            job.close()

    def one(b):
        L = int(seq_lens[b])
        rows = np.arange(offs[b], offs[b + 1])
        pos = L - len(rows) + np.arange(len(rows))
        return oracle_mod.paged_attention_rows(q[rows], pos, causal, dtype, kpool, vpool,
                                               kv_heads, head_dim, block_size, tables[b], L,
                                               scale)

    with ThreadPoolExecutor(host_threads()) as ex:  # the ctypes calls release the GIL
        return list(ex.map(one, range(n)))


def report(what: str, max_abs: float, max_rel: float) -> None:
    """Prints a full-size parity result beside the tolerances (shown by
    pytest -rP) and appends it to the file PKV_PARITY_LOG names, if set."""
    import os
    line = (f"PARITY {what}: max-abs {max_abs:.3e} (tol {ABS_TOL}), "
            f"max-rel {max_rel:.3e} over |ref| >= {REL_FLOOR} (tol {REL_TOL})")
    print(line)
    log = os.environ.get("PKV_PARITY_LOG")  # optional: collect the lines of a run
    if log:
        with open(log, "a") as f:
            f.write(line + "\n")
