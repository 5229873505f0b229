"""ctypes view of the oracle libraries.  TEST INFRASTRUCTURE ONLY.

* ``port``: libpkv_oracle.so, the CPU restatement in pkv_oracle.c.
* ``ref``:  _ref/libref_oracle.so, the inference SDK's own CPU sources
  (tensor_sdpa_f32, the allocator, the f16 conversions) plus ref_harness.c.
  It is built from the SDK's source tree by oracle/Makefile and is absent
  where that tree was never available; ``ref_available()`` says which.
* ``ref_cuda``: _ref/libref_cuda.so, the SDK's own CUDA backend (its paged
  decoder loop) built the same way; it needs a GPU to run.

Only tests/, __graft_entry__.smoke() and bench.py's reference / cpu_baseline
legs use this module, as the checker; the product never does.
"""
from __future__ import annotations

import ctypes
import pathlib
import subprocess
from typing import Optional

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
PORT_PATH = HERE / "libpkv_oracle.so"
REF_PATH = HERE / "_ref" / "libref_oracle.so"
REF_CUDA_PATH = HERE / "_ref" / "libref_cuda.so"

F16, BF16 = 1, 2
_DT = {"f16": F16, "bf16": BF16}

_port = None
_ref = None

_p = ctypes.c_void_p
_s = ctypes.c_size_t
_i = ctypes.c_int
_f = ctypes.c_float


def build() -> None:
    """Runs oracle/Makefile (the SDK part only when its sources exist)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def port() -> ctypes.CDLL:
    global _port
    if _port is None:
        if not PORT_PATH.exists():
            build()
        lib = ctypes.CDLL(str(PORT_PATH))
        lib.orc_f16_to_f32.restype = ctypes.c_float
        lib.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        lib.orc_f32_to_f16.restype = ctypes.c_uint16
        lib.orc_f32_to_f16.argtypes = [ctypes.c_float]
        lib.orc_bf16_to_f32.restype = ctypes.c_float
        lib.orc_bf16_to_f32.argtypes = [ctypes.c_uint16]
        lib.orc_f32_to_bf16.restype = ctypes.c_uint16
        lib.orc_f32_to_bf16.argtypes = [ctypes.c_float]
        lib.orc_kv_rows.restype = _i
        lib.orc_kv_rows.argtypes = [_p, _p, _s, _s, _s, _p, _s, _p, _p, _s, _p, _p, _i, _i]
        lib.orc_sdpa_f32.restype = _i
        lib.orc_sdpa_f32.argtypes = [_p, _p, _p, _p, _p, _s, _s, _s, _s, _s, _s, _s, _f, _i, _p]
        lib.orc_decode_sequence.restype = _i
        lib.orc_decode_sequence.argtypes = [_i, _i, _p, _s, _p, ctypes.c_uint32, _s, _p, _p, _p,
                                            _s, _s, _s, _s, _s, _s, _s, _f, ctypes.c_double, _p,
                                            _p, _s, _p]
        lib.orc_paged_attention_rows.restype = _i
        lib.orc_paged_attention_rows.argtypes = [_p, _p, _s, _i, _i, _p, _p, _s, _s, _s, _s, _p,
                                                 _s, ctypes.c_int64, _s, _f, _p]
        _port = lib
    return _port


def ref_available() -> bool:
    return REF_PATH.exists()


def ref() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        if not REF_PATH.exists():
            raise FileNotFoundError(f"{REF_PATH} not built (needs the SDK sources)")
        lib = ctypes.CDLL(str(REF_PATH))
        lib.ref_sdpa_f32.restype = _i
        lib.ref_sdpa_f32.argtypes = [_p, _p, _p, _p, _p, _s, _s, _s, _s, _s, _s, _s, _f, _i,
                                     ctypes.c_char_p, _s]
        lib.ref_job_prepare.restype = _p
        lib.ref_job_prepare.argtypes = [_i, _p, _p, _p, _p, _s, _s, _s, _s, _p, _s, _p, _s, _s,
                                        _p, _s, _s, _s, _s, _f, _i]
        lib.ref_job_run.restype = _i
        lib.ref_job_run.argtypes = [_p, _i, ctypes.POINTER(ctypes.c_double)]
        lib.ref_job_output.restype = _i
        lib.ref_job_output.argtypes = [_p, _s, _p]
        lib.ref_job_free.restype = None
        lib.ref_job_free.argtypes = [_p]
        # the SDK's own allocator and conversions
        lib.tensor_paged_kv_cache_create.restype = _i
        lib.tensor_paged_kv_cache_create.argtypes = [_s, _s, _s, ctypes.POINTER(_p)]
        lib.tensor_paged_kv_cache_free.argtypes = [_p]
        lib.tensor_paged_kv_sequence_create.restype = _i
        lib.tensor_paged_kv_sequence_create.argtypes = [_p, ctypes.POINTER(ctypes.c_uint64)]
        for n in ("reserve", "set_length"):
            fn = getattr(lib, f"tensor_paged_kv_sequence_{n}")
            fn.restype = _i
            fn.argtypes = [_p, ctypes.c_uint64, _s]
        lib.tensor_paged_kv_sequence_copy_block_table.restype = _i
        lib.tensor_paged_kv_sequence_copy_block_table.argtypes = [_p, ctypes.c_uint64, _p, _s,
                                                                  ctypes.POINTER(_s)]
        lib.tensor_paged_kv_sequence_length.restype = _i
        lib.tensor_paged_kv_sequence_length.argtypes = [_p, ctypes.c_uint64, ctypes.POINTER(_s)]
        for n in ("release", "begin_decode"):
            fn = getattr(lib, f"tensor_paged_kv_sequence_{n}")
            fn.restype = _i
            fn.argtypes = [_p, ctypes.c_uint64]
        lib.tensor_paged_kv_sequence_end_decode.argtypes = [_p, ctypes.c_uint64]
        lib.tensor_paged_kv_cache_free_blocks.restype = _s
        lib.tensor_paged_kv_cache_free_blocks.argtypes = [_p]
        lib.tensor_f16_to_f32.restype = ctypes.c_float
        lib.tensor_f16_to_f32.argtypes = [ctypes.c_uint16]
        lib.tensor_f32_to_f16.restype = ctypes.c_uint16
        lib.tensor_f32_to_f16.argtypes = [ctypes.c_float]
        lib.tensor_bf16_to_f32.restype = ctypes.c_float
        lib.tensor_bf16_to_f32.argtypes = [ctypes.c_uint16]
        _ref = lib
    return _ref


def _a(x: np.ndarray) -> int:
    assert x.flags["C_CONTIGUOUS"]
    return x.ctypes.data


# ---------------------------------------------------------------------------
# Port (restatement) entry points
# ---------------------------------------------------------------------------

def kv_rows(kpool: np.ndarray, vpool: np.ndarray, block_size: int, tables: np.ndarray,
            seq_lens: np.ndarray, row_offsets: Optional[np.ndarray], krows: np.ndarray,
            vrows: np.ndarray, to_pool: bool, tail: bool) -> None:
    """Append (to_pool, tail), import (to_pool) or gather (not to_pool)."""
    kv_width = kpool.shape[1]
    block_count = kpool.shape[0] // block_size
    tables = np.ascontiguousarray(tables, dtype=np.uint32)
    seq_lens = np.ascontiguousarray(seq_lens, dtype=np.int32)
    offs = None if row_offsets is None else np.ascontiguousarray(row_offsets, dtype=np.int32)
    ok = port().orc_kv_rows(_a(kpool), _a(vpool), kv_width, block_size, block_count, _a(tables),
                            tables.shape[1], _a(seq_lens), None if offs is None else _a(offs),
                            len(seq_lens), _a(krows), _a(vrows), int(to_pool), int(tail))
    if not ok:
        raise ValueError("oracle kv_rows: position or page out of range")


def sdpa_f32(q, k, v, scale: float, causal: bool, mask=None) -> np.ndarray:
    """Restated tensor_sdpa_f32 on [B,H,L,d] float32 arrays."""
    q, k, v = (np.ascontiguousarray(x, dtype=np.float32) for x in (q, k, v))
    B, Hq, Lq, d = q.shape
    Hkv, Lk, dv = k.shape[1], k.shape[2], v.shape[3]
    out = np.zeros((B, Hq, Lq, dv), dtype=np.float32)
    scores = np.zeros(Lq * Lk, dtype=np.float32)
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.float32)
    ok = port().orc_sdpa_f32(_a(q), _a(k), _a(v), None if m is None else _a(m), _a(out), B, Hq,
                             Hkv, Lq, Lk, d, dv, scale, int(causal), _a(scores))
    if not ok:
        raise ValueError("oracle sdpa: invalid shape")
    return out


def paged_attention_rows(q_rows: np.ndarray, q_pos: np.ndarray, causal: bool, dtype: str,
                         kpool: np.ndarray, vpool: np.ndarray, kv_heads: int, head_dim: int,
                         block_size: int, table_row: np.ndarray, seq_len: int,
                         scale: float) -> np.ndarray:
    """Paged attention of some query rows ([n, Hq, d] storage bits) of one
    sequence; returns float32 [n, Hq, d]."""
    q_rows = np.ascontiguousarray(q_rows, dtype=np.uint16)
    n, q_heads, _ = q_rows.shape
    q_pos = np.ascontiguousarray(q_pos, dtype=np.int64)
    table_row = np.ascontiguousarray(table_row, dtype=np.uint32)
    out = np.zeros((n, q_heads, head_dim), dtype=np.float32)
    ok = port().orc_paged_attention_rows(_a(q_rows), _a(q_pos), n, int(causal), _DT[dtype],
                                         _a(kpool), _a(vpool), kv_heads, head_dim, block_size,
                                         kpool.shape[0] // block_size, _a(table_row),
                                         len(table_row), seq_len, q_heads, scale, _a(out))
    if not ok:
        raise ValueError("oracle paged attention: addressing error")
    return out


def paged_decode(q: np.ndarray, dtype: str, kpool, vpool, kv_heads: int, head_dim: int,
                 block_size: int, tables: np.ndarray, seq_lens: np.ndarray,
                 scale: float) -> np.ndarray:
    """One query row per sequence: q [B, Hq, d] bits -> float32 [B, Hq, d]."""
    out = np.zeros(q.shape, dtype=np.float32)
    for b in range(q.shape[0]):
        L = int(seq_lens[b])
        out[b] = paged_attention_rows(q[b:b + 1], np.array([L - 1]), False, dtype, kpool, vpool,
                                      kv_heads, head_dim, block_size, tables[b], L, scale)[0]
    return out


# ---------------------------------------------------------------------------
# The SDK's own code (ref)
# ---------------------------------------------------------------------------

def ref_sdpa_f32(q, k, v, scale: float, causal: bool, mask=None) -> np.ndarray:
    q, k, v = (np.ascontiguousarray(x, dtype=np.float32) for x in (q, k, v))
    B, Hq, Lq, d = q.shape
    Hkv, Lk, dv = k.shape[1], k.shape[2], v.shape[3]
    out = np.zeros((B, Hq, Lq, dv), dtype=np.float32)
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.float32)
    err = ctypes.create_string_buffer(256)
    ok = ref().ref_sdpa_f32(_a(q), _a(k), _a(v), None if m is None else _a(m), _a(out), B, Hq,
                            Hkv, Lq, Lk, d, dv, scale, int(causal), err, len(err))
    if not ok:
        raise ValueError(f"tensor_sdpa_f32: {err.value.decode()}")
    return out


class RefJob:
    """Prepared tensor_sdpa_f32 calls over paged sequences (see ref_harness.c)."""

    def __init__(self, dtype: str, q: np.ndarray, q_offsets: Optional[np.ndarray], kpool, vpool,
                 kv_heads: int, head_dim: int, block_size: int, tables: np.ndarray,
                 seq_lens: np.ndarray, q_heads: int, scale: float, causal: bool,
                 subset: Optional[np.ndarray] = None, kv_head0: int = 0,
                 kv_head_n: Optional[int] = None, tail_rows: int = 0):
        lib = ref()
        self._keep = [np.ascontiguousarray(x) for x in (q, kpool, vpool)]
        q, kpool, vpool = self._keep
        tables = np.ascontiguousarray(tables, dtype=np.uint32)
        seq_lens = np.ascontiguousarray(seq_lens, dtype=np.int32)
        offs = None if q_offsets is None else np.ascontiguousarray(q_offsets, dtype=np.int32)
        sub = None if subset is None else np.ascontiguousarray(subset, dtype=np.int32)
        self._keep += [tables, seq_lens, offs, sub]
        kv_head_n = kv_heads if kv_head_n is None else kv_head_n
        self.group = q_heads // kv_heads
        self.q_heads = kv_head_n * self.group
        self.head_dim = head_dim
        self.n_items = len(seq_lens) if sub is None else len(sub)
        self.rows = []
        for i in range(self.n_items):
            b = i if sub is None else int(sub[i])
            r = 1 if offs is None else int(offs[b + 1] - offs[b])
            self.rows.append(min(r, tail_rows) if tail_rows else r)
        self.handle = lib.ref_job_prepare(
            _DT[dtype], _a(q), None if offs is None else _a(offs), _a(kpool), _a(vpool),
            kv_heads, head_dim, block_size, kpool.shape[0] // block_size, _a(tables),
            tables.shape[1], _a(seq_lens), len(seq_lens), q_heads,
            None if sub is None else _a(sub), 0 if sub is None else len(sub), kv_head0,
            kv_head_n, tail_rows, scale, int(causal))
        if not self.handle:
            raise ValueError("ref_job_prepare failed")

    def run(self, threads: int = 1) -> float:
        sec = ctypes.c_double(0.0)
        if not ref().ref_job_run(self.handle, threads, ctypes.byref(sec)):
            raise RuntimeError("ref_job_run failed")
        return sec.value

    def output(self, index: int) -> np.ndarray:
        out = np.zeros((self.rows[index], self.q_heads, self.head_dim), dtype=np.float32)
        ref().ref_job_output(self.handle, index, _a(out))
        return out

    def close(self) -> None:
        if self.handle:
            ref().ref_job_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------------------
# The paged decoder (include/attention.h): restatement and the SDK's own GPU
# ---------------------------------------------------------------------------

def decode_sequence(storage: int, fmt: int, layers, embedding, initial_token: int,
                    token_count: int, kcache, vcache, past: int, capacity: int, hidden: int,
                    inter: int, qh: int, kvh: int, hd: int, eps: float, theta: float,
                    final_norm, lm_head, vocab: int, want_logits: bool = False):
    """orc_decode_sequence.  layers: per layer nine arrays (input_norm, q, k,
    v, o, post_norm, gate, up, down); kcache/vcache: per layer contiguous
    [capacity, kv_width] arrays in the storage type, positions [0, past)
    holding the prefix, updated in place.  Returns the tokens (and every
    step's logits, [token_count, vocab])."""
    keep = []

    def a(x):
        x = np.ascontiguousarray(x)
        keep.append(x)
        return x.ctypes.data

    ptrs = (_p * (9 * len(layers)))(*[a(t) for layer in layers for t in layer])
    for c in list(kcache) + list(vcache):
        assert c.flags["C_CONTIGUOUS"]
    kc = (_p * len(kcache))(*[c.ctypes.data for c in kcache])
    vc = (_p * len(vcache))(*[c.ctypes.data for c in vcache])
    out = np.zeros(token_count, dtype=np.uint32)
    logits = np.zeros((token_count, vocab), dtype=np.float32)
    ok = port().orc_decode_sequence(storage, fmt, ptrs, len(layers), a(embedding), initial_token,
                                    token_count, out.ctypes.data, kc, vc, past, capacity, hidden,
                                    inter, qh, kvh, hd, eps, theta, a(final_norm), a(lm_head),
                                    vocab, logits.ctypes.data)
    if not ok:
        raise ValueError("oracle decode_sequence: invalid arguments")
    tokens = out.tolist()
    return (tokens, logits) if want_logits else tokens


def ref_cuda_available() -> bool:
    return REF_CUDA_PATH.exists()


class _Request(ctypes.Structure):
    """TensorPagedKVDecodeRequest (the SDK's include/attention.h:48-72)."""
    _fields_ = [("cache", _p), ("sequence", ctypes.c_uint64), ("storage", _i), ("layers", _p),
                ("layer_count", _s), ("embedding", _p), ("initial_token", ctypes.c_uint32),
                ("token_count", _s), ("generated_tokens", _p), ("key_cache", _p),
                ("value_cache", _p), ("past_length", _s), ("hidden_size", _s),
                ("intermediate_size", _s), ("query_heads", _s), ("kv_heads", _s),
                ("head_dim", _s), ("rms_norm_epsilon", _f), ("rope_theta", ctypes.c_double),
                ("final_norm", _p), ("lm_head", _p), ("vocabulary_size", _s),
                ("weight_quantization", _i)]


class RefCudaDecoder:
    """One paged cache and sequence inside the SDK's own CUDA build; each
    call runs its tensor_attention_decode_sequence_paged."""

    def __init__(self, block_size: int, block_count: int):
        if not REF_CUDA_PATH.exists():
            raise FileNotFoundError(f"{REF_CUDA_PATH} not built (needs the SDK sources)")
        lib = ctypes.CDLL(str(REF_CUDA_PATH))
        lib.tensor_paged_kv_cache_create.restype = _i
        lib.tensor_paged_kv_cache_create.argtypes = [_s, _s, _s, ctypes.POINTER(_p)]
        lib.tensor_paged_kv_sequence_create.restype = _i
        lib.tensor_paged_kv_sequence_create.argtypes = [_p, ctypes.POINTER(ctypes.c_uint64)]
        lib.tensor_attention_decode_sequence_paged.restype = _i
        lib.tensor_attention_decode_sequence_paged.argtypes = [ctypes.POINTER(_Request)]
        lib.tensor_paged_kv_cache_free.argtypes = [_p]
        lib.tensor_attention_decode_cache_clear.argtypes = []
        self.lib = lib
        h = _p()
        assert lib.tensor_paged_kv_cache_create(block_size, block_count, 1, ctypes.byref(h))
        self.cache = h.value
        seq = ctypes.c_uint64()
        assert lib.tensor_paged_kv_sequence_create(self.cache, ctypes.byref(seq))
        self.seq = seq.value

    def decode(self, storage, fmt, layers, embedding, initial_token, token_count, kcache,
               vcache, past, hidden, inter, qh, kvh, hd, eps, theta, final_norm, lm_head,
               vocab):
        keep = []

        def a(x):
            x = np.ascontiguousarray(x)
            keep.append(x)
            return x.ctypes.data

        # the quantised layer struct keeps both norms first (attention.h:38-42)
        order = [0, 5, 1, 2, 3, 4, 6, 7, 8] if storage == 2 else list(range(9))
        ptrs = (_p * (9 * len(layers)))(*[a(layer[i]) for layer in layers for i in order])
        kc = (_p * len(kcache))(*[a(c) for c in kcache])
        vc = (_p * len(vcache))(*[a(c) for c in vcache])
        out = np.zeros(token_count, dtype=np.uint32)
        rq = _Request(self.cache, self.seq, storage, ctypes.addressof(ptrs), len(layers),
                      a(embedding), initial_token, token_count, out.ctypes.data,
                      ctypes.addressof(kc), ctypes.addressof(vc), past, hidden, inter, qh, kvh,
                      hd, eps, theta, a(final_norm), a(lm_head), vocab, fmt)
        ok = self.lib.tensor_attention_decode_sequence_paged(ctypes.byref(rq))
        return out.tolist() if ok else None

    def close(self):
        if self.cache:
            self.lib.tensor_paged_kv_cache_free(self.cache)
            self.lib.tensor_attention_decode_cache_clear()
            self.cache = None


class _Ops(ctypes.Structure):
    """The head of TensorAttentionBackendOps (the SDK's src/attention_backend.h)."""
    _fields_ = [("kind", _i), ("name", ctypes.c_char_p), ("is_available", _p), ("run", _p),
                ("run_f16", _p)]


_RUN_F16 = ctypes.CFUNCTYPE(_i, _p, _p, _p, _p, _p, _s, _s, _s, _s, _s, _s, _s, _f, _i)


def ref_cuda_sdpa_f16(q, k, v, scale: float, causal: bool, mask=None):
    """The SDK CUDA backend's run_f16 (dense sdpa, attention_cuda.cu:71-99)
    on host uint16 arrays (mask: None or [Lq, Lk] FP16 bits); returns the
    output bits or None."""
    lib = ctypes.CDLL(str(REF_CUDA_PATH))
    lib.tensor_attention_cuda_backend.restype = ctypes.POINTER(_Ops)
    ops = lib.tensor_attention_cuda_backend().contents
    run = _RUN_F16(ops.run_f16)
    B, Hq, Lq, d = q.shape
    Hkv, Lk, dv = k.shape[1], k.shape[2], v.shape[3]
    q, k, v = (np.ascontiguousarray(a, dtype=np.uint16) for a in (q, k, v))
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint16)
    out = np.zeros((B, Hq, Lq, dv), dtype=np.uint16)
    ok = run(q.ctypes.data, k.ctypes.data, v.ctypes.data, None if m is None else m.ctypes.data,
             out.ctypes.data, B, Hq, Hkv, Lq, Lk, d, dv, scale, int(causal))
    return out if ok else None
