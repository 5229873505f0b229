"""B200 (sm_100a) paged-KV attention behind the inference SDK's C API.

The product is the shared library ``inference_c_b200/lib/libpkv_b200.so``:
C11 host code (page allocator with the SDK's ``tensor_paged_kv_*`` API, the
device pool and the batch step transaction) and the CUDA kernels, exported
through ``include/paged_kv_cache.h``, ``include/pkv_b200.h`` and
``include/attention.h`` (the SDK's paged decoder entry point).  This module
is the Python view of that ABI, via ctypes: tests and ``bench.py`` use it,
with torch only for device memory and streams.  Nothing here computes
attention; there is no CPU fallback, and every call raises when the library
is missing or a C call reports failure.
"""
from __future__ import annotations

import ctypes
import pathlib
from typing import Optional, Sequence

LIB_PATH = pathlib.Path(__file__).resolve().parent / "lib" / "libpkv_b200.so"

PKV_DTYPE_F16 = 1
PKV_DTYPE_BF16 = 2
PKV_DTYPE_F32 = 3

TENSOR_PAGED_KV_BACKEND_CUDA = 1

_c_size = ctypes.c_size_t
_c_ptr = ctypes.c_void_p
_c_u64 = ctypes.c_uint64
_c_int = ctypes.c_int
_c_char_p = ctypes.c_char_p


class PkvPagedLayer(ctypes.Structure):
    _fields_ = [
        ("key_pool", _c_ptr),
        ("value_pool", _c_ptr),
        ("block_size", _c_size),
        ("block_count", _c_size),
        ("kv_heads", _c_size),
        ("head_dim", _c_size),
        ("dtype", _c_int),
    ]


class PkvBatch(ctypes.Structure):
    _fields_ = [
        ("block_tables", _c_ptr),
        ("table_stride", _c_size),
        ("seq_lens", _c_ptr),
        ("batch", _c_size),
    ]


# include/attention.h: TENSOR_PAGED_KV_* storage kinds and the request struct
TENSOR_PAGED_KV_F32 = 0
TENSOR_PAGED_KV_F16 = 1
TENSOR_PAGED_KV_QUANT_F16 = 2
TENSOR_WEIGHT_Q8_0 = 1
TENSOR_WEIGHT_Q4_0 = 2


class TensorAttentionDecoderLayer(ctypes.Structure):
    """TensorAttentionDecoderLayer / ...LayerF16: nine pointers in this order."""
    _fields_ = [(n, _c_ptr) for n in ("input_norm", "q_weight", "k_weight", "v_weight",
                                      "o_weight", "post_norm", "gate_weight", "up_weight",
                                      "down_weight")]


class TensorAttentionDecoderLayerQuantF16(ctypes.Structure):
    """The quantised layer struct keeps both norms first."""
    _fields_ = [(n, _c_ptr) for n in ("input_norm", "post_norm", "q_weight", "k_weight",
                                      "v_weight", "o_weight", "gate_weight", "up_weight",
                                      "down_weight")]


class TensorPagedKVDecodeRequest(ctypes.Structure):
    _fields_ = [
        ("cache", _c_ptr),
        ("sequence", _c_u64),
        ("storage", _c_int),
        ("layers", _c_ptr),
        ("layer_count", _c_size),
        ("embedding", _c_ptr),
        ("initial_token", ctypes.c_uint32),
        ("token_count", _c_size),
        ("generated_tokens", _c_ptr),
        ("key_cache", _c_ptr),
        ("value_cache", _c_ptr),
        ("past_length", _c_size),
        ("hidden_size", _c_size),
        ("intermediate_size", _c_size),
        ("query_heads", _c_size),
        ("kv_heads", _c_size),
        ("head_dim", _c_size),
        ("rms_norm_epsilon", ctypes.c_float),
        ("rope_theta", ctypes.c_double),
        ("final_norm", _c_ptr),
        ("lm_head", _c_ptr),
        ("vocabulary_size", _c_size),
        ("weight_quantization", _c_int),
    ]


_LP = ctypes.POINTER(PkvPagedLayer)
_BP = ctypes.POINTER(PkvBatch)
_ERR = [_c_char_p, _c_size]

# name -> (restype, argtypes).  Every symbol declared in include/*.h.
EXPORTS = {
    # include/paged_kv_cache.h
    "tensor_paged_kv_cache_create": (_c_int, [_c_size, _c_size, _c_size, ctypes.POINTER(_c_ptr)]),
    "tensor_paged_kv_cache_free": (None, [_c_ptr]),
    "tensor_paged_kv_sequence_create": (_c_int, [_c_ptr, ctypes.POINTER(_c_u64)]),
    "tensor_paged_kv_sequence_reserve": (_c_int, [_c_ptr, _c_u64, _c_size]),
    "tensor_paged_kv_sequence_set_length": (_c_int, [_c_ptr, _c_u64, _c_size]),
    "tensor_paged_kv_sequence_copy_block_table": (
        _c_int, [_c_ptr, _c_u64, _c_ptr, _c_size, ctypes.POINTER(_c_size)]),
    "tensor_paged_kv_sequence_length": (_c_int, [_c_ptr, _c_u64, ctypes.POINTER(_c_size)]),
    "tensor_paged_kv_sequence_release": (_c_int, [_c_ptr, _c_u64]),
    "tensor_paged_kv_sequence_begin_decode": (_c_int, [_c_ptr, _c_u64]),
    "tensor_paged_kv_sequence_end_decode": (None, [_c_ptr, _c_u64]),
    "tensor_paged_kv_cache_free_blocks": (_c_size, [_c_ptr]),
    "tensor_paged_kv_cache_block_size": (_c_size, [_c_ptr]),
    "tensor_paged_kv_cache_block_count": (_c_size, [_c_ptr]),
    "tensor_paged_kv_cache_backend_state": (_c_ptr, [_c_ptr, _c_int]),
    "tensor_paged_kv_cache_set_backend_state": (_c_int, [_c_ptr, _c_int, _c_ptr, _c_ptr, _c_ptr]),
    # include/attention.h
    "tensor_attention_decode_sequence_paged": (
        _c_int, [ctypes.POINTER(TensorPagedKVDecodeRequest)]),
    "tensor_attention_decode_cache_clear": (None, []),
    # include/pkv_b200.h -- kernels
    "pkv_kv_append": (_c_int, [_LP, _BP, _c_ptr, _c_ptr, _c_ptr, _c_size, _c_ptr, *_ERR]),
    "pkv_kv_import": (_c_int, [_LP, _BP, _c_ptr, _c_ptr, _c_ptr, _c_size, _c_ptr, *_ERR]),
    "pkv_kv_gather": (_c_int, [_LP, _BP, _c_ptr, _c_ptr, _c_ptr, _c_size, _c_ptr, *_ERR]),
    "pkv_decode_workspace_bytes": (_c_size, [_c_size, _c_size, _c_size, _c_size, _c_size]),
    "pkv_decode_workspace_init": (_c_int, [_c_ptr, _c_size, _c_ptr, *_ERR]),
    "pkv_paged_decode": (_c_int, [_LP, _BP, _c_size, _c_ptr, ctypes.c_float, _c_ptr, _c_int,
                                  _c_size, _c_size, _c_ptr, _c_size, _c_ptr, *_ERR]),
    "pkv_paged_decode_append": (_c_int, [_LP, _BP, _c_ptr, _c_ptr, _c_size, _c_ptr,
                                         ctypes.c_float, _c_ptr, _c_int, _c_size, _c_size,
                                         _c_ptr, _c_size, _c_ptr, *_ERR]),
    "pkv_paged_decode_static_scratch": (_c_int, [_LP, _BP, _c_size, _c_ptr, ctypes.c_float,
                                                 _c_ptr, _c_int, _c_size, _c_ptr, *_ERR]),
    "pkv_paged_prefill": (_c_int, [_LP, _BP, _c_size, _c_ptr, _c_ptr, _c_size, _c_size,
                                   ctypes.c_float, _c_int, _c_ptr, _c_int, _c_ptr, *_ERR]),
    "pkv_device_fault": (_c_int, [_c_int, ctypes.POINTER(ctypes.c_uint32), *_ERR]),
    "pkv_selftest_wait_timeout": (_c_int, [ctypes.POINTER(ctypes.c_uint32), *_ERR]),
    "pkv_sdpa_workspace_bytes": (_c_size, [_c_size, _c_size, _c_size, _c_size, _c_size]),
    "pkv_sdpa_f16": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_size, _c_size, _c_size,
                              _c_size, _c_size, _c_size, ctypes.c_float, _c_int, _c_ptr, _c_size,
                              _c_ptr, *_ERR]),
    "pkv_sdpa_f16_host": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_size, _c_size,
                                   _c_size, _c_size, _c_size, _c_size, _c_size, ctypes.c_float,
                                   _c_int]),
    # include/pkv_b200.h -- host transaction layer
    "pkv_pool_create": (_c_int, [_c_ptr, _c_int, _c_int, _c_size, _c_size, _c_size, _c_size,
                                 _c_size, ctypes.POINTER(_c_ptr), *_ERR]),
    "pkv_pool_from_cache": (_c_ptr, [_c_ptr]),
    "pkv_pool_layer": (_c_int, [_c_ptr, _c_size, _LP]),
    "pkv_step_begin": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_size, _c_ptr, *_ERR]),
    "pkv_step_batch": (_c_int, [_c_ptr, _BP]),
    "pkv_step_row_offsets": (_c_ptr, [_c_ptr]),
    "pkv_step_end": (_c_int, [_c_ptr, _c_int, *_ERR]),
    # include/pkv_b200.h -- NCCL all-gather with a host deadline
    "pkv_comm_unique_id": (_c_int, [_c_ptr, _c_size, *_ERR]),
    "pkv_comm_init": (_c_int, [_c_ptr, _c_size, _c_int, _c_int, _c_int, ctypes.c_double,
                               ctypes.POINTER(_c_ptr), *_ERR]),
    "pkv_comm_all_gather": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_size, _c_ptr, ctypes.c_double,
                                     *_ERR]),
    "pkv_comm_wait": (_c_int, [_c_ptr, _c_ptr, ctypes.c_double, *_ERR]),
    "pkv_comm_aborted": (_c_int, [_c_ptr]),
    "pkv_comm_destroy": (None, [_c_ptr]),
    # include/pkv_b200.h -- all-gather by peer stores
    "pkv_peer_gather_create": (_c_int, [_c_int, _c_int, _c_int, _c_size, ctypes.POINTER(_c_ptr),
                                        _c_ptr, _c_size, *_ERR]),
    "pkv_peer_gather_connect": (_c_int, [_c_ptr, _c_ptr, _c_size, *_ERR]),
    "pkv_peer_all_gather": (_c_int, [_c_ptr, _c_ptr, _c_ptr, ctypes.c_double, _c_ptr, *_ERR]),
    "pkv_peer_gather_destroy": (None, [_c_ptr]),
}

_lib: Optional[ctypes.CDLL] = None


def load() -> ctypes.CDLL:
    """Loads libpkv_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: run inference_c_b200/_build.py "
                           "(or __graft_entry__.build()) first; there is no fallback")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in EXPORTS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class PkvError(RuntimeError):
    """A C entry point returned 0."""


def _call(name: str, *args):
    lib = load()
    err = ctypes.create_string_buffer(512)
    ok = getattr(lib, name)(*args, err, len(err))
    if not ok:
        raise PkvError(f"{name}: {err.value.decode(errors='replace')}")
    return ok


# ---------------------------------------------------------------------------
# Allocator: the SDK's tensor_paged_kv_* API, one method per C function.
# ---------------------------------------------------------------------------

class PagedKVCache:
    """Owns one TensorPagedKVCache*.  Methods return the C result (1/0)."""

    def __init__(self, block_size: int, block_count: int, max_sequences: int):
        lib = load()
        h = _c_ptr()
        if not lib.tensor_paged_kv_cache_create(block_size, block_count, max_sequences,
                                                ctypes.byref(h)):
            raise PkvError("tensor_paged_kv_cache_create failed")
        self.handle = h.value
        self._lib = lib

    def free(self) -> None:
        if self.handle:
            self._lib.tensor_paged_kv_cache_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def sequence_create(self) -> int:
        s = _c_u64(0)
        return s.value if self._lib.tensor_paged_kv_sequence_create(self.handle, ctypes.byref(s)) else 0

    def reserve(self, seq: int, tokens: int) -> int:
        return self._lib.tensor_paged_kv_sequence_reserve(self.handle, seq, tokens)

    def set_length(self, seq: int, tokens: int) -> int:
        return self._lib.tensor_paged_kv_sequence_set_length(self.handle, seq, tokens)

    def length(self, seq: int) -> Optional[int]:
        n = _c_size(0)
        return n.value if self._lib.tensor_paged_kv_sequence_length(self.handle, seq, ctypes.byref(n)) else None

    def block_table(self, seq: int) -> Optional[list[int]]:
        n = _c_size(0)
        if not self._lib.tensor_paged_kv_sequence_copy_block_table(self.handle, seq, None, 0,
                                                                   ctypes.byref(n)):
            return None
        buf = (ctypes.c_uint32 * max(1, n.value))()
        if not self._lib.tensor_paged_kv_sequence_copy_block_table(self.handle, seq, buf, n.value,
                                                                   ctypes.byref(n)):
            return None
        return list(buf[: n.value])

    def copy_block_table(self, seq: int, capacity: int) -> tuple[int, list[int], int]:
        buf = (ctypes.c_uint32 * max(1, capacity))()
        n = _c_size(0)
        ok = self._lib.tensor_paged_kv_sequence_copy_block_table(self.handle, seq, buf, capacity,
                                                                 ctypes.byref(n))
        return ok, list(buf[: min(n.value, capacity)]), n.value

    def release(self, seq: int) -> int:
        return self._lib.tensor_paged_kv_sequence_release(self.handle, seq)

    def begin_decode(self, seq: int) -> int:
        return self._lib.tensor_paged_kv_sequence_begin_decode(self.handle, seq)

    def end_decode(self, seq: int) -> None:
        self._lib.tensor_paged_kv_sequence_end_decode(self.handle, seq)

    def free_blocks(self) -> int:
        return self._lib.tensor_paged_kv_cache_free_blocks(self.handle)

    def block_size(self) -> int:
        return self._lib.tensor_paged_kv_cache_block_size(self.handle)

    def block_count(self) -> int:
        return self._lib.tensor_paged_kv_cache_block_count(self.handle)


# ---------------------------------------------------------------------------
# Kernel entry points over torch tensors (device memory only).
# ---------------------------------------------------------------------------

def _ptr(x) -> Optional[int]:
    """Device address of a tensor, or an int address passed through."""
    if x is None or isinstance(x, int):
        return x
    return x.data_ptr()


def _dtype_code(t) -> int:
    import torch
    return {torch.float16: PKV_DTYPE_F16, torch.bfloat16: PKV_DTYPE_BF16,
            torch.float32: PKV_DTYPE_F32}[t.dtype]


def _stream_ptr(stream) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def make_layer(key_pool, value_pool, block_size: int, kv_heads: int, head_dim: int) -> PkvPagedLayer:
    """Layer view of two [block_count*block_size, kv_heads*head_dim] pools."""
    assert key_pool.shape == value_pool.shape and key_pool.is_cuda
    rows = key_pool.shape[0]
    assert rows % block_size == 0 and key_pool.shape[1] == kv_heads * head_dim
    return PkvPagedLayer(key_pool.data_ptr(), value_pool.data_ptr(), block_size,
                         rows // block_size, kv_heads, head_dim, _dtype_code(key_pool))


def make_batch(block_tables, seq_lens) -> PkvBatch:
    """Batch view of a [batch, stride] int32 table and [batch] int32 lengths."""
    assert block_tables.dim() == 2 and block_tables.is_contiguous() and seq_lens.is_contiguous()
    return PkvBatch(block_tables.data_ptr(), block_tables.shape[1], seq_lens.data_ptr(),
                    block_tables.shape[0])


def kv_append(layer: PkvPagedLayer, batch: PkvBatch, key_rows, value_rows, row_offsets=None,
              stream=None) -> None:
    _call("pkv_kv_append", ctypes.byref(layer), ctypes.byref(batch), _ptr(row_offsets),
          key_rows.data_ptr(), value_rows.data_ptr(), key_rows.shape[0], _stream_ptr(stream))


def kv_import(layer: PkvPagedLayer, batch: PkvBatch, key_rows, value_rows, row_offsets,
              stream=None) -> None:
    _call("pkv_kv_import", ctypes.byref(layer), ctypes.byref(batch), _ptr(row_offsets),
          key_rows.data_ptr(), value_rows.data_ptr(), key_rows.shape[0], _stream_ptr(stream))


def kv_gather(layer: PkvPagedLayer, batch: PkvBatch, key_out, value_out, row_offsets,
              stream=None) -> None:
    _call("pkv_kv_gather", ctypes.byref(layer), ctypes.byref(batch), _ptr(row_offsets),
          key_out.data_ptr(), value_out.data_ptr(), key_out.shape[0], _stream_ptr(stream))


def decode_workspace_bytes(batch: int, q_heads: int, head_dim: int, max_seq_len: int,
                           chunk_tokens: int = 0) -> int:
    return load().pkv_decode_workspace_bytes(batch, q_heads, head_dim, max_seq_len, chunk_tokens)


def decode_workspace(batch: int, q_heads: int, head_dim: int, max_seq_len: int,
                     chunk_tokens: int = 0, device=None, stream=None):
    """Zero-initialised decode scratch as a uint8 CUDA tensor."""
    import torch
    n = decode_workspace_bytes(batch, q_heads, head_dim, max_seq_len, chunk_tokens)
    ws = torch.empty(n, dtype=torch.uint8, device=device or "cuda")
    _call("pkv_decode_workspace_init", ws.data_ptr(), n, _stream_ptr(stream))
    return ws


def paged_decode(layer: PkvPagedLayer, batch: PkvBatch, query, output, scale: float,
                 max_seq_len: int, workspace, chunk_tokens: int = 0, stream=None) -> None:
    q_heads = query.shape[-2]
    _call("pkv_paged_decode", ctypes.byref(layer), ctypes.byref(batch), q_heads,
          query.data_ptr(), ctypes.c_float(scale), output.data_ptr(), _dtype_code(output),
          max_seq_len, chunk_tokens, workspace.data_ptr(), workspace.numel(), _stream_ptr(stream))


def paged_decode_append(layer: PkvPagedLayer, batch: PkvBatch, key_rows, value_rows, query,
                        output, scale: float, max_seq_len: int, workspace, chunk_tokens: int = 0,
                        stream=None) -> None:
    """pkv_paged_decode_append: kv_append of one new row per sequence and
    paged_decode in one call (one launch on the tensor-core path)."""
    if key_rows.shape[0] != batch.batch or value_rows.shape[0] != batch.batch:
        raise ValueError("one new K and V row per sequence")
    q_heads = query.shape[-2]
    _call("pkv_paged_decode_append", ctypes.byref(layer), ctypes.byref(batch),
          key_rows.data_ptr(), value_rows.data_ptr(), q_heads, query.data_ptr(),
          ctypes.c_float(scale), output.data_ptr(), _dtype_code(output), max_seq_len,
          chunk_tokens, workspace.data_ptr(), workspace.numel(), _stream_ptr(stream))


def paged_decode_static_scratch(layer: PkvPagedLayer, batch: PkvBatch, query, output,
                                scale: float, max_seq_len: int, stream=None) -> None:
    """pkv_paged_decode with the library's static device scratch (no workspace)."""
    q_heads = query.shape[-2]
    _call("pkv_paged_decode_static_scratch", ctypes.byref(layer), ctypes.byref(batch), q_heads,
          query.data_ptr(), ctypes.c_float(scale), output.data_ptr(), _dtype_code(output),
          max_seq_len, _stream_ptr(stream))


def paged_prefill(layer: PkvPagedLayer, batch: PkvBatch, query, query_offsets, output,
                  scale: float, max_query_len: int, causal: bool = True, stream=None) -> None:
    q_heads = query.shape[-2]
    _call("pkv_paged_prefill", ctypes.byref(layer), ctypes.byref(batch), q_heads,
          _ptr(query_offsets), query.data_ptr(), query.shape[0], max_query_len,
          ctypes.c_float(scale), int(causal), output.data_ptr(), _dtype_code(output),
          _stream_ptr(stream))


def device_fault(device: int = 0) -> int:
    code = ctypes.c_uint32(0)
    _call("pkv_device_fault", device, ctypes.byref(code))
    return code.value


def selftest_wait_timeout() -> int:
    """Runs the bounded-wait self-test on the current device; returns the
    fault code it recorded (4: the wait gave up as designed)."""
    code = ctypes.c_uint32(0)
    _call("pkv_selftest_wait_timeout", ctypes.byref(code))
    return code.value


# ---------------------------------------------------------------------------
# Host transaction layer.
# ---------------------------------------------------------------------------

class PagedPool:
    """Device pool attached to a PagedKVCache (freed with the cache)."""

    def __init__(self, cache: PagedKVCache, device: int, dtype: int, layer_count: int,
                 kv_heads: int, head_dim: int, max_batch: int, max_pages_per_seq: int):
        h = _c_ptr()
        _call("pkv_pool_create", cache.handle, device, dtype, layer_count, kv_heads, head_dim,
              max_batch, max_pages_per_seq, ctypes.byref(h))
        self.handle = h.value
        self.cache = cache
        self.max_batch = max_batch
        self._lib = load()

    def layer(self, index: int) -> PkvPagedLayer:
        out = PkvPagedLayer()
        if not self._lib.pkv_pool_layer(self.handle, index, ctypes.byref(out)):
            raise PkvError(f"pkv_pool_layer({index}) failed")
        return out

    def step_begin(self, sequences: Sequence[int], new_tokens: Sequence[int],
                   past_lengths: Optional[Sequence[int]] = None, stream=None) -> None:
        n = len(sequences)
        seqs = (_c_u64 * n)(*sequences)
        new = (_c_size * n)(*new_tokens)
        past = None if past_lengths is None else (_c_size * n)(*past_lengths)
        _call("pkv_step_begin", self.handle, seqs, past, new, n, _stream_ptr(stream))

    def step_batch(self) -> PkvBatch:
        out = PkvBatch()
        if not self._lib.pkv_step_batch(self.handle, ctypes.byref(out)):
            raise PkvError("pkv_step_batch: no open step")
        return out

    def step_row_offsets(self) -> int:
        return self._lib.pkv_step_row_offsets(self.handle)

    def step_end(self, commit: bool) -> None:
        _call("pkv_step_end", self.handle, int(commit))


class DecodeStepper:
    """One decode step of a fixed batch -- pkv_step_begin (one new token per
    sequence), pkv_paged_decode_append (or, with fused=False, pkv_kv_append
    then pkv_paged_decode), pkv_step_end -- with every argument converted
    once.  A step of a short batch runs for tens of microseconds on the GPU;
    building the ctypes arguments, stream and dtype lookups of the one-call
    wrappers again for each call would make the Python host, not the GPU, set
    the step rate.  A failed call rolls the open step back (pkv_step_end(0))
    and raises."""

    def __init__(self, pool: PagedPool, layer: PkvPagedLayer, sequences: Sequence[int], query,
                 key_rows, value_rows, output, scale: float, max_seq_len: int, workspace,
                 chunk_tokens: int = 0, stream=None, fused: bool = True):
        lib = load()
        self.fused = fused
        n = len(sequences)
        self._lib = lib
        self._pool = pool.handle
        self._n = n
        self._seqs = (_c_u64 * n)(*sequences)
        self._new = (_c_size * n)(*([1] * n))
        self._stream = _stream_ptr(stream)
        self._err = ctypes.create_string_buffer(512)
        self._layer = layer
        self._layer_ref = ctypes.byref(layer)
        self._batch = PkvBatch()
        self._batch_ref = ctypes.byref(self._batch)
        self._q_heads = query.shape[-2]
        self._scale = ctypes.c_float(scale)
        self._out_dtype = _dtype_code(output)
        self._max_len = max_seq_len
        self._chunk = chunk_tokens
        self._ws = workspace.data_ptr()
        self._ws_bytes = workspace.numel()
        self.bind(query, key_rows, value_rows, output)

    def bind(self, query, key_rows, value_rows, output) -> None:
        """Device buffers of the next steps (same shapes and dtypes)."""
        if key_rows.shape[0] != self._n or value_rows.shape[0] != self._n:
            raise ValueError("one new K and V row per sequence")
        self._q, self._k, self._v = query.data_ptr(), key_rows.data_ptr(), value_rows.data_ptr()
        self._o = output.data_ptr()

    def _fail(self, name: str, opened: bool):
        msg = self._err.value.decode(errors="replace")
        if opened:
            self._lib.pkv_step_end(self._pool, 0, self._err, 512)
        raise PkvError(f"{name}: {msg}")

    def step(self) -> None:
        lib, err = self._lib, self._err
        if not lib.pkv_step_begin(self._pool, self._seqs, None, self._new, self._n, self._stream,
                                  err, 512):
            self._fail("pkv_step_begin", False)
        lib.pkv_step_batch(self._pool, self._batch_ref)
        if self.fused:
            if not lib.pkv_paged_decode_append(self._layer_ref, self._batch_ref, self._k, self._v,
                                               self._q_heads, self._q, self._scale, self._o,
                                               self._out_dtype, self._max_len, self._chunk,
                                               self._ws, self._ws_bytes, self._stream, err, 512):
                self._fail("pkv_paged_decode_append", True)
        else:
            if not lib.pkv_kv_append(self._layer_ref, self._batch_ref, None, self._k, self._v,
                                     self._n, self._stream, err, 512):
                self._fail("pkv_kv_append", True)
            if not lib.pkv_paged_decode(self._layer_ref, self._batch_ref, self._q_heads, self._q,
                                        self._scale, self._o, self._out_dtype, self._max_len,
                                        self._chunk, self._ws, self._ws_bytes, self._stream, err,
                                        512):
                self._fail("pkv_paged_decode", True)
        if not lib.pkv_step_end(self._pool, 1, err, 512):
            self._fail("pkv_step_end", False)


# ---------------------------------------------------------------------------
# include/attention.h: the SDK's paged decoder (greedy tokens of one sequence)
# ---------------------------------------------------------------------------

def decode_sequence_paged(cache: "PagedKVCache", sequence: int, storage: int, layers,
                          embedding, initial_token: int, token_count: int, key_cache,
                          value_cache, past_length: int, hidden_size: int,
                          intermediate_size: int, query_heads: int, kv_heads: int,
                          head_dim: int, rms_norm_epsilon: float, rope_theta: float,
                          final_norm, lm_head, vocabulary_size: int,
                          weight_quantization: int = 0) -> Optional[list]:
    """tensor_attention_decode_sequence_paged with host numpy arrays.

    layers: one sequence of nine arrays per layer (input_norm, q, k, v, o,
    post_norm, gate, up, down, whatever the storage's struct order) in the
    storage's element type (float32 or
    uint16 half bits; uint8 blocks for quantised matrices); key_cache /
    value_cache: one host array per layer holding at least past_length rows.
    Returns the generated tokens, or None when the call returns 0 (the SDK
    reports failure only through the return value)."""
    import numpy as np
    lib = load()
    keep = []

    def ptr(a):
        a = np.ascontiguousarray(a)
        keep.append(a)
        return a.ctypes.data

    kind = (TensorAttentionDecoderLayerQuantF16 if storage == TENSOR_PAGED_KV_QUANT_F16
            else TensorAttentionDecoderLayer)
    order = ("input_norm", "q_weight", "k_weight", "v_weight", "o_weight", "post_norm",
             "gate_weight", "up_weight", "down_weight")
    layer_arr = (kind * len(layers))()
    for i, tensors in enumerate(layers):
        assert len(tensors) == 9
        for name, t in zip(order, tensors):
            setattr(layer_arr[i], name, ptr(t))
    kc = (_c_ptr * len(key_cache))(*[ptr(a) for a in key_cache])
    vc = (_c_ptr * len(value_cache))(*[ptr(a) for a in value_cache])
    out = np.zeros(max(token_count, 1), dtype=np.uint32)
    rq = TensorPagedKVDecodeRequest()
    rq.cache = cache.handle if cache is not None else None
    rq.sequence = sequence
    rq.storage = storage
    rq.layers = ctypes.addressof(layer_arr)
    rq.layer_count = len(layers)
    rq.embedding = ptr(embedding)
    rq.initial_token = initial_token
    rq.token_count = token_count
    rq.generated_tokens = out.ctypes.data
    rq.key_cache = ctypes.addressof(kc)
    rq.value_cache = ctypes.addressof(vc)
    rq.past_length = past_length
    rq.hidden_size = hidden_size
    rq.intermediate_size = intermediate_size
    rq.query_heads = query_heads
    rq.kv_heads = kv_heads
    rq.head_dim = head_dim
    rq.rms_norm_epsilon = rms_norm_epsilon
    rq.rope_theta = rope_theta
    rq.final_norm = ptr(final_norm)
    rq.lm_head = ptr(lm_head)
    rq.vocabulary_size = vocabulary_size
    rq.weight_quantization = weight_quantization
    ok = lib.tensor_attention_decode_sequence_paged(ctypes.byref(rq))
    return out[:token_count].tolist() if ok else None


def decode_cache_clear() -> None:
    load().tensor_attention_decode_cache_clear()


# ---------------------------------------------------------------------------
# Dense FP16 SDPA (tensor_sdpa_f16's backend) on the prefill kernel
# ---------------------------------------------------------------------------

def sdpa_f16(query, key, value, output, scale: float, causal: bool, stream=None,
             mask=None) -> None:
    """query/output [B, Hq, Lq, d], key/value [B, Hkv, Lk, d] float16 CUDA tensors
    (d = 64 or 128); mask: None or an additive float16 CUDA tensor [Lq, Lk]."""
    import torch
    B, Hq, Lq, d = query.shape
    Hkv, Lk = key.shape[1], key.shape[2]
    n = load().pkv_sdpa_workspace_bytes(B, Hq, Hkv, Lq, Lk, d)
    ws = torch.empty(n, dtype=torch.uint8, device=query.device)
    _call("pkv_sdpa_f16", query.data_ptr(), key.data_ptr(), value.data_ptr(),
          None if mask is None else mask.data_ptr(), output.data_ptr(), B, Hq, Hkv, Lq, Lk, d,
          ctypes.c_float(scale), int(causal), ws.data_ptr(), n, _stream_ptr(stream))


def sdpa_f16_host(query, key, value, scale: float, causal: bool, mask=None):
    """The run_f16 backend hook with host numpy uint16 (FP16 bits) arrays;
    returns the output bits or None when the call returns 0."""
    import numpy as np
    B, Hq, Lq, d = query.shape
    Hkv, Lk, dv = key.shape[1], key.shape[2], value.shape[3]
    q, k, v = (np.ascontiguousarray(a, dtype=np.uint16) for a in (query, key, value))
    m = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint16)
    out = np.zeros((B, Hq, Lq, dv), dtype=np.uint16)
    ok = load().pkv_sdpa_f16_host(q.ctypes.data, k.ctypes.data, v.ctypes.data,
                                  None if m is None else m.ctypes.data, out.ctypes.data, B, Hq,
                                  Hkv, Lq, Lk, d, dv, ctypes.c_float(scale), int(causal))
    return out if ok else None


# ---------------------------------------------------------------------------
# NCCL all-gather with a host deadline (multi-GPU head split)
# ---------------------------------------------------------------------------

COMM_ID_BYTES = 256


def comm_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(COMM_ID_BYTES)
    _call("pkv_comm_unique_id", buf, COMM_ID_BYTES)
    return buf.raw


class Comm:
    """One rank of a non-blocking NCCL communicator (pkv_comm_*): every call
    waits at most its timeout and raises PkvError (the communicator then
    aborted) when a peer never joins or stalls."""

    def __init__(self, unique_id: bytes, nranks: int, rank: int, device: int,
                 timeout_s: float):
        if len(unique_id) != COMM_ID_BYTES:
            raise ValueError(f"unique id must be {COMM_ID_BYTES} bytes")
        self._id = ctypes.create_string_buffer(unique_id, COMM_ID_BYTES)
        h = _c_ptr()
        _call("pkv_comm_init", self._id, COMM_ID_BYTES, nranks, rank, device,
              ctypes.c_double(timeout_s), ctypes.byref(h))
        self.handle = h.value

    def all_gather(self, send, recv, stream=None, timeout_s: float = 10.0) -> None:
        """send: a CUDA tensor; recv: nranks x send (rank order)."""
        _call("pkv_comm_all_gather", self.handle, send.data_ptr(), recv.data_ptr(),
              send.numel() * send.element_size(), _stream_ptr(stream),
              ctypes.c_double(timeout_s))

    def wait(self, stream=None, timeout_s: float = 10.0) -> None:
        _call("pkv_comm_wait", self.handle, _stream_ptr(stream), ctypes.c_double(timeout_s))

    @property
    def aborted(self) -> bool:
        return bool(load().pkv_comm_aborted(self.handle))

    def destroy(self) -> None:
        if self.handle:
            load().pkv_comm_destroy(self.handle)
            self.handle = None


PEER_HANDLE_BYTES = 64


class PeerGather:
    """pkv_peer_gather_*: all-gather of `nbytes` per rank by peer stores over
    NVLink.  Create on every rank, exchange `handle` (bytes), then connect
    with all ranks' handles in rank order."""

    def __init__(self, device: int, nranks: int, rank: int, nbytes: int):
        h = _c_ptr()
        buf = ctypes.create_string_buffer(PEER_HANDLE_BYTES)
        _call("pkv_peer_gather_create", device, nranks, rank, nbytes, ctypes.byref(h), buf,
              PEER_HANDLE_BYTES)
        self.handle = h.value
        self.ipc_handle = buf.raw

    def connect(self, handles: list) -> None:
        blob = b"".join(handles)
        buf = ctypes.create_string_buffer(blob, len(blob))
        _call("pkv_peer_gather_connect", self.handle, buf, len(blob))

    def all_gather(self, send, recv, stream=None, timeout_s: float = 1.0) -> None:
        _call("pkv_peer_all_gather", self.handle, send.data_ptr(), recv.data_ptr(),
              ctypes.c_double(timeout_s), _stream_ptr(stream))

    def destroy(self) -> None:
        if self.handle:
            load().pkv_peer_gather_destroy(self.handle)
            self.handle = None
