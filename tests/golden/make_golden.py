"""Generates the golden fixtures in tests/golden/ from the inference SDK's own
CPU code (oracle/_ref/libref_oracle.so, built from the SDK sources by
oracle/Makefile).  Run from the repository root:

    python tests/golden/make_golden.py

Fixtures (inputs are regenerated from the recorded seeds with
inference_c_b200.workloads, which is bit-reproducible on any machine):
  known_answer.json    the SDK's dense SDPA known-answer case
                       (tests/test_attention.c:441-496): inputs, SDK outputs
  cfg1.json            config 1: 512 one-token appends into a seeded
                       32-of-64-page table, sha256 of the K and V pools
                       afterwards, and the SDK's FP32 decode output
  decode_small.json    ragged GQA decode (lengths on and across page edges)
  prefill_small.json   causal chunked prefill, BF16, two sequences
  allocator_trace.json a seeded trace of allocator calls with the SDK
                       allocator's result and full state after every call
"""
from __future__ import annotations

import base64
import ctypes
import hashlib
import json
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from inference_c_b200 import workloads as W  # noqa: E402
from oracle import oracle as O  # noqa: E402


def b64(a: np.ndarray) -> str:
    return base64.b64encode(np.ascontiguousarray(a).tobytes()).decode()


def known_answer() -> dict:
    q = np.array([1, 0, 0, 1, 1, 0, 0, 1], np.float32).reshape(1, 2, 2, 2)
    k = np.array([1, 0, 0, 1], np.float32).reshape(1, 1, 2, 2)
    v = np.array([1, 0, 0, 2], np.float32).reshape(1, 1, 2, 2)
    mask = np.array([-np.inf, 0, 0, 0], np.float32).reshape(2, 2)
    allmask = np.full((2, 2), -np.inf, np.float32)
    out = {
        "q": q.ravel().tolist(), "k": k.ravel().tolist(), "v": v.ravel().tolist(),
        "noncausal": O.ref_sdpa_f32(q, k, v, 1.0, False).ravel().tolist(),
        "causal": O.ref_sdpa_f32(q, k, v, 1.0, True).ravel().tolist(),
        "masked": O.ref_sdpa_f32(q, k, v, 1.0, False, mask).ravel().tolist(),
        "all_masked": O.ref_sdpa_f32(q, k, v, 1.0, False, allmask).ravel().tolist(),
        # the literal expectations of the SDK test
        "sdk_expected_noncausal": [0.73105858, 0.53788284, 0.26894143, 1.4621172],
        "sdk_expected_causal": [1.0, 0.0, 0.26894143, 1.4621172],
        "sdk_expected_masked_first": [0.0, 2.0],
        "sdk_tolerance": 1e-5,
    }
    return out


def cfg1(seed: int = 2024) -> dict:
    c = W.CONFIGS[1]
    table = W.cfg1_table(seed)
    rows = W.CFG1_POOL_PAGES * c.block_size
    kpool = np.zeros((rows, c.kv_width), np.uint16)
    vpool = np.zeros((rows, c.kv_width), np.uint16)
    krows = W.normal_bits(seed, (W.CFG1_TOKENS, c.kv_width), "f16", stream=41)
    vrows = W.normal_bits(seed, (W.CFG1_TOKENS, c.kv_width), "f16", stream=42)
    q = W.normal_bits(seed, (1, c.q_heads, c.head_dim), "f16", stream=43)
    tables = table.reshape(1, -1)
    for t in range(W.CFG1_TOKENS):
        O.kv_rows(kpool, vpool, c.block_size, tables, np.array([t + 1]), None,
                  np.ascontiguousarray(krows[t:t + 1]), np.ascontiguousarray(vrows[t:t + 1]),
                  to_pool=True, tail=True)
    job = O.RefJob("f16", q, None, kpool, vpool, c.kv_heads, c.head_dim, c.block_size, tables,
                   np.array([W.CFG1_TOKENS]), c.q_heads, c.scale, False)
    job.run(1)
    out = job.output(0)[0]
    return {
        "seed": seed, "table": table.tolist(),
        "k_pool_sha256": hashlib.sha256(kpool.tobytes()).hexdigest(),
        "v_pool_sha256": hashlib.sha256(vpool.tobytes()).hexdigest(),
        "decode_out_f32_b64": b64(out), "shape": list(out.shape),
    }


def decode_small(seed: int = 7) -> dict:
    q_heads, kv_heads, d, bs = 8, 2, 128, 16
    lengths = np.array([1, 15, 16, 17, 300], np.int64)
    pool_pages = 64
    tables, stride = W.shuffled_tables(lengths, bs, pool_pages, seed)
    kv = kv_heads * d
    kpool = W.normal_bits(seed, (pool_pages * bs, kv), "f16", stream=51)
    vpool = W.normal_bits(seed, (pool_pages * bs, kv), "f16", stream=52)
    q = W.normal_bits(seed, (len(lengths), q_heads, d), "f16", stream=53)
    scale = 1.0 / np.sqrt(d)
    job = O.RefJob("f16", q, None, kpool, vpool, kv_heads, d, bs, tables, lengths, q_heads,
                   float(scale), False)
    job.run(1)
    out = np.stack([job.output(i)[0] for i in range(len(lengths))])
    return {"seed": seed, "q_heads": q_heads, "kv_heads": kv_heads, "head_dim": d,
            "block_size": bs, "pool_pages": pool_pages, "lengths": lengths.tolist(),
            "out_f32_b64": b64(out), "shape": list(out.shape)}


def prefill_small(seed: int = 11) -> dict:
    q_heads, kv_heads, d, bs = 4, 2, 128, 16
    past = np.array([40, 5], np.int64)
    chunk = np.array([24, 19], np.int64)
    lengths = past + chunk
    pool_pages = 16
    tables, stride = W.shuffled_tables(lengths, bs, pool_pages, seed)
    kv = kv_heads * d
    kpool = W.normal_bits(seed, (pool_pages * bs, kv), "bf16", stream=61)
    vpool = W.normal_bits(seed, (pool_pages * bs, kv), "bf16", stream=62)
    offs = np.concatenate([[0], np.cumsum(chunk)]).astype(np.int32)
    q = W.normal_bits(seed, (int(offs[-1]), q_heads, d), "bf16", stream=63)
    scale = 1.0 / np.sqrt(d)
    job = O.RefJob("bf16", q, offs, kpool, vpool, kv_heads, d, bs, tables, lengths, q_heads,
                   float(scale), True)
    job.run(1)
    out = np.concatenate([job.output(i) for i in range(len(lengths))])
    return {"seed": seed, "q_heads": q_heads, "kv_heads": kv_heads, "head_dim": d,
            "block_size": bs, "pool_pages": pool_pages, "past": past.tolist(),
            "chunk": chunk.tolist(), "out_f32_b64": b64(out), "shape": list(out.shape)}


def allocator_trace(seed: int = 3, steps: int = 400) -> dict:
    """Random allocator calls against the SDK's allocator."""
    lib = O.ref()
    block_size, block_count, max_seq = 4, 24, 3
    cache = ctypes.c_void_p()
    assert lib.tensor_paged_kv_cache_create(block_size, block_count, max_seq, ctypes.byref(cache))
    u = W.uniform(seed, steps * 3, stream=71)
    handles: list[int] = []
    stale_handles: list[int] = []
    ops = []
    for i in range(steps):
        kind = int(u[3 * i] * 7)
        pick = handles[int(u[3 * i + 1] * len(handles))] if handles else 0
        arg = int(u[3 * i + 2] * 40)
        if kind == 0 or not handles:
            h = ctypes.c_uint64(0)
            r = lib.tensor_paged_kv_sequence_create(cache, ctypes.byref(h))
            if r:
                handles.append(h.value)
            op = {"op": "create", "result": r, "handle": h.value if r else 0}
        elif kind == 1:
            op = {"op": "reserve", "seq": pick, "arg": arg,
                  "result": lib.tensor_paged_kv_sequence_reserve(cache, pick, arg)}
        elif kind == 2:
            op = {"op": "set_length", "seq": pick, "arg": arg,
                  "result": lib.tensor_paged_kv_sequence_set_length(cache, pick, arg)}
        elif kind == 3:
            r = lib.tensor_paged_kv_sequence_release(cache, pick)
            if r:
                handles.remove(pick)
                stale_handles.append(pick)
            op = {"op": "release", "seq": pick, "result": r}
        elif kind == 4:
            op = {"op": "begin_decode", "seq": pick,
                  "result": lib.tensor_paged_kv_sequence_begin_decode(cache, pick)}
        elif kind == 5:
            lib.tensor_paged_kv_sequence_end_decode(cache, pick)
            op = {"op": "end_decode", "seq": pick, "result": None}
        else:
            # a released handle, or one whose generation never existed
            stale = stale_handles[arg % len(stale_handles)] if stale_handles else pick ^ (1 << 40)
            op = {"op": "reserve", "seq": stale, "arg": arg,
                  "result": lib.tensor_paged_kv_sequence_reserve(cache, stale, arg)}
        state = {"free": lib.tensor_paged_kv_cache_free_blocks(cache), "seqs": {}}
        for h in handles + stale_handles:
            n = ctypes.c_size_t(0)
            if lib.tensor_paged_kv_sequence_copy_block_table(cache, h, None, 0, ctypes.byref(n)):
                buf = (ctypes.c_uint32 * max(1, n.value))()
                lib.tensor_paged_kv_sequence_copy_block_table(cache, h, buf, n.value,
                                                              ctypes.byref(n))
                ln = ctypes.c_size_t(0)
                lib.tensor_paged_kv_sequence_length(cache, h, ctypes.byref(ln))
                state["seqs"][str(h)] = {"table": list(buf[: n.value]), "length": ln.value}
        op["state"] = state
        ops.append(op)
    lib.tensor_paged_kv_cache_free(cache)
    return {"block_size": block_size, "block_count": block_count, "max_sequences": max_seq,
            "ops": ops}


def main() -> None:
    O.build()
    if not O.ref_available():
        raise SystemExit("the SDK-source oracle (oracle/_ref) is not built")
    for name, fn in [("known_answer", known_answer), ("cfg1", cfg1),
                     ("decode_small", decode_small), ("prefill_small", prefill_small),
                     ("allocator_trace", allocator_trace)]:
        path = HERE / f"{name}.json"
        path.write_text(json.dumps(fn(), indent=1, sort_keys=True) + "\n")
        print(f"wrote {path.relative_to(ROOT)} ({path.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
