"""Seeded synthetic workloads for the paged-KV path (configs 1-5).

The SDK publishes no benchmark data for this path, so every input is
synthetic: N(0, 1) query/key/value rows rounded to FP16 or BF16 and context
lengths from the distributions each config names.  The small-case generator
is a splitmix64 stream with Box-Muller (pure integer mixing + numpy float64
math), so the same seed yields the same bits on every machine; the golden
fixtures in tests/golden/ are keyed by these seeds.  Full-size benchmark
tensors are drawn on the GPU with torch's seeded generator instead.
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(seed: int, n: int, stream: int = 0) -> np.ndarray:
    """n consecutive splitmix64 outputs of generator (seed, stream)."""
    with np.errstate(over="ignore"):
        base = np.uint64((seed * 0x100000001B3 + stream * 0xD6E8FEB86659FD93) & (2**64 - 1))
        z = base + (np.arange(1, n + 1, dtype=np.uint64) * _GOLDEN)
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def uniform(seed: int, n: int, stream: int = 0) -> np.ndarray:
    """Uniform float64 in [0, 1)."""
    return (splitmix64(seed, n, stream) >> np.uint64(11)).astype(np.float64) * (1.0 / 2**53)


def normal(seed: int, n: int, stream: int = 0) -> np.ndarray:
    """Standard normal float32 via Box-Muller on the splitmix stream."""
    m = (n + 1) // 2
    u = uniform(seed, 2 * m, stream)
    r = np.sqrt(-2.0 * np.log(1.0 - u[0::2]))
    t = 2.0 * math.pi * u[1::2]
    out = np.empty(2 * m, dtype=np.float64)
    out[0::2] = r * np.cos(t)
    out[1::2] = r * np.sin(t)
    return out[:n].astype(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bit patterns (uint16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & np.uint32(0x7FFFFFFF)) > np.uint32(0x7F800000)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)
    r = np.where(nan, (u >> np.uint32(16)) | np.uint32(0x40), r)
    return r.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << np.uint32(16)).view(np.float32)


def storage_bits(x: np.ndarray, dtype: str) -> np.ndarray:
    """float32 values -> uint16 storage bits of 'f16' or 'bf16' (RNE)."""
    if dtype == "f16":
        return x.astype(np.float16).view(np.uint16)
    if dtype == "bf16":
        return f32_to_bf16_bits(x)
    raise ValueError(dtype)


def normal_bits(seed: int, shape, dtype: str, stream: int = 0) -> np.ndarray:
    n = int(np.prod(shape))
    return storage_bits(normal(seed, n, stream), dtype).reshape(shape)


def permutation(seed: int, n: int, stream: int = 0) -> np.ndarray:
    """Seeded Fisher-Yates permutation of range(n) (int64)."""
    u = uniform(seed, max(n, 1), stream)
    p = np.arange(n, dtype=np.int64)
    for i in range(n - 1, 0, -1):
        j = int(u[i] * (i + 1))
        p[i], p[j] = p[j], p[i]
    return p


# ---------------------------------------------------------------------------
# The five configurations
# ---------------------------------------------------------------------------

@dataclasses.dataclass(frozen=True)
class Config:
    name: str
    batch: int
    q_heads: int
    kv_heads: int
    head_dim: int
    block_size: int
    dtype: str  # storage: 'f16' or 'bf16'

    @property
    def kv_width(self) -> int:
        return self.kv_heads * self.head_dim

    @property
    def scale(self) -> float:
        return 1.0 / math.sqrt(self.head_dim)


CONFIGS = {
    1: Config("cfg1: 1 seq, MHA 8x64, 512 appends then decode", 1, 8, 8, 64, 16, "f16"),
    2: Config("cfg2: Llama-3-8B decode layer, B=32, GQA 32/8, d=128, L~U[1024,4096]",
              32, 32, 8, 128, 16, "f16"),
    3: Config("cfg3: B=256, GQA 32/8, d=128, L~LogNormal(ln 8192, 0.5) clipped [512, 32768]",
              256, 32, 8, 128, 16, "f16"),
    4: Config("cfg4: one 131072-token sequence, GQA 64/8, d=128", 1, 64, 8, 128, 16, "f16"),
    5: Config("cfg5: chunked prefill, B=8, 8192 past + 2048 chunk, GQA 32/8, d=128, BF16",
              8, 32, 8, 128, 16, "bf16"),
}

CFG1_POOL_PAGES = 64
CFG1_TABLE_PAGES = 32
CFG1_TOKENS = 512
CFG3_SIGMA = 0.5          # not given by the config; recorded with every number
CFG4_TOKENS = 131072
CFG5_PAST = 8192
CFG5_CHUNK = 2048


def context_lengths(config: int, seed: int, batch: int | None = None) -> np.ndarray:
    """Seeded context lengths (int64) for configs 2-5."""
    c = CONFIGS[config]
    n = c.batch if batch is None else batch
    if config == 2:
        u = uniform(seed, n, stream=11)
        return (1024 + np.floor(u * (4096 - 1024 + 1))).astype(np.int64)
    if config == 3:
        z = normal(seed, n, stream=12).astype(np.float64)
        L = np.exp(math.log(8192.0) + CFG3_SIGMA * z)
        return np.clip(np.rint(L), 512, 32768).astype(np.int64)
    if config == 4:
        return np.full(n, CFG4_TOKENS, dtype=np.int64)
    if config == 5:
        return np.full(n, CFG5_PAST, dtype=np.int64)
    return np.full(n, CFG1_TOKENS, dtype=np.int64)


def shard_by_length(lengths: np.ndarray, ranks: int) -> list[np.ndarray]:
    """Greedy length balancing: longest first onto the least-loaded rank.
    Returns the sequence indices of each rank (ascending)."""
    order = np.argsort(-lengths, kind="stable")
    load = np.zeros(ranks, dtype=np.int64)
    parts: list[list[int]] = [[] for _ in range(ranks)]
    for i in order:
        r = int(np.argmin(load))
        parts[r].append(int(i))
        load[r] += int(lengths[i])
    return [np.array(sorted(p), dtype=np.int64) for p in parts]


def shuffled_tables(lengths: np.ndarray, block_size: int, pool_pages: int, seed: int,
                    stride: int | None = None) -> tuple[np.ndarray, int]:
    """Block tables drawing pages from one shuffled shared pool.

    Returns (tables[batch, stride] uint32, stride).  Pages are dealt from a
    seeded permutation of range(pool_pages) in sequence order, so every
    sequence's pages are scattered over the whole pool."""
    pages = [(int(L) + block_size - 1) // block_size for L in lengths]
    need = sum(pages)
    if need > pool_pages:
        raise ValueError(f"pool of {pool_pages} pages cannot hold {need}")
    perm = permutation(seed, pool_pages, stream=21)
    width = max(1, max(pages)) if stride is None else stride
    tables = np.zeros((len(lengths), width), dtype=np.uint32)
    at = 0
    for b, n in enumerate(pages):
        tables[b, :n] = perm[at:at + n]
        at += n
    return tables, width


def cfg1_table(seed: int) -> np.ndarray:
    """Config 1: 32 distinct pages of a 64-page pool in seeded random order."""
    return permutation(seed, CFG1_POOL_PAGES, stream=31)[:CFG1_TABLE_PAGES].astype(np.uint32)
