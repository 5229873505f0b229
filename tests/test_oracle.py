"""Pins the CPU oracle to the inference SDK: golden fixtures made by the SDK's
own code (tests/golden/make_golden.py), the SDK test's literal expectations,
and -- where the SDK sources were available to build oracle/_ref -- a live
bit-for-bit comparison with the SDK's tensor_sdpa_f32 and conversions."""
from __future__ import annotations

import base64
import hashlib
import json
import pathlib

import numpy as np
import pytest

from inference_c_b200 import workloads as W

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


def _fixture(name):
    return json.loads((GOLDEN / f"{name}.json").read_text())


def _f32(b64: str, shape) -> np.ndarray:
    return np.frombuffer(base64.b64decode(b64), dtype=np.float32).reshape(shape)


def test_known_answer_matches_sdk_test(oracle_mod):
    fx = _fixture("known_answer")
    q = np.array(fx["q"], np.float32).reshape(1, 2, 2, 2)
    k = np.array(fx["k"], np.float32).reshape(1, 1, 2, 2)
    v = np.array(fx["v"], np.float32).reshape(1, 1, 2, 2)
    nc = oracle_mod.sdpa_f32(q, k, v, 1.0, False).ravel()
    c = oracle_mod.sdpa_f32(q, k, v, 1.0, True).ravel()
    mask = np.array([-np.inf, 0, 0, 0], np.float32).reshape(2, 2)
    m = oracle_mod.sdpa_f32(q, k, v, 1.0, False, mask).ravel()
    am = oracle_mod.sdpa_f32(q, k, v, 1.0, False, np.full((2, 2), -np.inf, np.float32)).ravel()
    tol = fx["sdk_tolerance"]
    # the SDK test's literal values (test_attention.c:441-496), both heads
    assert np.all(np.abs(nc[:4] - fx["sdk_expected_noncausal"]) < tol)
    assert np.all(np.abs(nc[4:] - nc[:4]) < tol)
    assert np.all(np.abs(c[:4] - fx["sdk_expected_causal"]) < tol)
    assert np.all(np.abs(m[:2] - fx["sdk_expected_masked_first"]) < tol)
    assert np.all(am == 0.0)
    # and the SDK's own outputs, bit for bit
    assert np.array_equal(nc, np.array(fx["noncausal"], np.float32))
    assert np.array_equal(c, np.array(fx["causal"], np.float32))
    assert np.array_equal(m, np.array(fx["masked"], np.float32))
    assert np.array_equal(am, np.array(fx["all_masked"], np.float32))


def test_f16_widening_all_patterns(oracle_mod):
    lib = oracle_mod.port()
    bits = np.arange(65536, dtype=np.uint32)
    ours = np.array([lib.orc_f16_to_f32(int(b)) for b in bits], np.float32)
    npv = bits.astype(np.uint16).view(np.float16).astype(np.float32)
    nan = np.isnan(npv)
    assert np.array_equal(ours[~nan].view(np.uint32), npv[~nan].view(np.uint32))
    assert np.all(np.isnan(ours[nan]))
    if oracle_mod.ref_available():
        ref = oracle_mod.ref()
        sdk = np.array([ref.tensor_f16_to_f32(int(b)) for b in bits], np.float32)
        assert np.array_equal(ours.view(np.uint32), sdk.view(np.uint32))


def test_f16_rounding(oracle_mod):
    lib = oracle_mod.port()
    u = W.splitmix64(5, 20000).astype(np.uint64) & np.uint64(0xFFFFFFFF)
    vals = u.astype(np.uint32).view(np.float32)
    edge = np.array([0.0, -0.0, 65504.0, 65520.0, 65519.99, 6.1e-5, 5.96e-8, 2.98e-8, 2.99e-8,
                     1.0 + 2**-11, 1.0 + 3 * 2**-11, np.inf, -np.inf], np.float32)
    vals = np.concatenate([vals, edge, W.normal(5, 5000) * 1000])
    ours = np.array([lib.orc_f32_to_f16(float(v)) for v in vals], np.uint16)
    npb = vals.astype(np.float16).view(np.uint16)
    nan = np.isnan(vals)
    assert np.array_equal(ours[~nan], npb[~nan])
    assert np.all((ours[nan] & 0x7C00) == 0x7C00) and np.all((ours[nan] & 0x3FF) != 0)
    if oracle_mod.ref_available():
        ref = oracle_mod.ref()
        sdk = np.array([ref.tensor_f32_to_f16(float(v)) for v in vals], np.uint16)
        assert np.array_equal(ours, sdk)


def test_bf16_rounding(oracle_mod):
    lib = oracle_mod.port()
    vals = np.concatenate([W.normal(9, 4000), W.normal(9, 100, stream=1) * 1e30,
                           np.array([0.0, -0.0, np.inf, -np.inf, 3.4e38], np.float32)])
    ours = np.array([lib.orc_f32_to_bf16(float(v)) for v in vals], np.uint16)
    assert np.array_equal(ours, W.f32_to_bf16_bits(vals))
    back = np.array([lib.orc_bf16_to_f32(int(b)) for b in ours], np.float32)
    assert np.array_equal(back, W.bf16_bits_to_f32(ours))


def test_cfg1_pages_and_decode(oracle_mod):
    fx = _fixture("cfg1")
    c = W.CONFIGS[1]
    seed = fx["seed"]
    table = W.cfg1_table(seed)
    assert table.tolist() == fx["table"]
    assert len(set(fx["table"])) == W.CFG1_TABLE_PAGES
    rows = W.CFG1_POOL_PAGES * c.block_size
    kpool = np.zeros((rows, c.kv_width), np.uint16)
    vpool = np.zeros((rows, c.kv_width), np.uint16)
    krows = W.normal_bits(seed, (W.CFG1_TOKENS, c.kv_width), "f16", stream=41)
    vrows = W.normal_bits(seed, (W.CFG1_TOKENS, c.kv_width), "f16", stream=42)
    for t in range(W.CFG1_TOKENS):
        oracle_mod.kv_rows(kpool, vpool, c.block_size, table.reshape(1, -1), np.array([t + 1]),
                           None, np.ascontiguousarray(krows[t:t + 1]),
                           np.ascontiguousarray(vrows[t:t + 1]), to_pool=True, tail=True)
    assert hashlib.sha256(kpool.tobytes()).hexdigest() == fx["k_pool_sha256"]
    assert hashlib.sha256(vpool.tobytes()).hexdigest() == fx["v_pool_sha256"]
    q = W.normal_bits(seed, (1, c.q_heads, c.head_dim), "f16", stream=43)
    out = oracle_mod.paged_decode(q, "f16", kpool, vpool, c.kv_heads, c.head_dim, c.block_size,
                                  table.reshape(1, -1), np.array([W.CFG1_TOKENS]), c.scale)
    assert np.array_equal(out[0], _f32(fx["decode_out_f32_b64"], fx["shape"]))


def test_decode_small_fixture(oracle_mod):
    fx = _fixture("decode_small")
    seed, bs, d = fx["seed"], fx["block_size"], fx["head_dim"]
    lengths = np.array(fx["lengths"], np.int64)
    tables, _ = W.shuffled_tables(lengths, bs, fx["pool_pages"], seed)
    kv = fx["kv_heads"] * d
    kpool = W.normal_bits(seed, (fx["pool_pages"] * bs, kv), "f16", stream=51)
    vpool = W.normal_bits(seed, (fx["pool_pages"] * bs, kv), "f16", stream=52)
    q = W.normal_bits(seed, (len(lengths), fx["q_heads"], d), "f16", stream=53)
    out = oracle_mod.paged_decode(q, "f16", kpool, vpool, fx["kv_heads"], d, bs, tables, lengths,
                                  float(1.0 / np.sqrt(d)))
    assert np.array_equal(out, _f32(fx["out_f32_b64"], fx["shape"]))


def test_prefill_small_fixture(oracle_mod):
    fx = _fixture("prefill_small")
    seed, bs, d = fx["seed"], fx["block_size"], fx["head_dim"]
    past, chunk = np.array(fx["past"]), np.array(fx["chunk"])
    lengths = past + chunk
    tables, _ = W.shuffled_tables(lengths, bs, fx["pool_pages"], seed)
    kv = fx["kv_heads"] * d
    kpool = W.normal_bits(seed, (fx["pool_pages"] * bs, kv), "bf16", stream=61)
    vpool = W.normal_bits(seed, (fx["pool_pages"] * bs, kv), "bf16", stream=62)
    offs = np.concatenate([[0], np.cumsum(chunk)]).astype(np.int32)
    q = W.normal_bits(seed, (int(offs[-1]), fx["q_heads"], d), "bf16", stream=63)
    want = _f32(fx["out_f32_b64"], fx["shape"])
    for b in range(len(lengths)):
        rows = q[offs[b]:offs[b + 1]]
        pos = np.arange(past[b], lengths[b])
        got = oracle_mod.paged_attention_rows(rows, pos, True, "bf16", kpool, vpool,
                                              fx["kv_heads"], d, bs, tables[b], int(lengths[b]),
                                              float(1.0 / np.sqrt(d)))
        # cutting the key range at the causal limit instead of masking with
        # -inf only changes additions of exact zeros
        assert np.max(np.abs(got - want[offs[b]:offs[b + 1]])) <= 1e-6


@pytest.mark.skipif(not (pathlib.Path(__file__).resolve().parents[1] / "oracle" / "_ref" /
                         "libref_oracle.so").exists(), reason="SDK-source oracle not built here")
@pytest.mark.parametrize("group,dtype,causal", [(1, "f16", False), (4, "f16", False),
                                                (8, "bf16", False), (2, "bf16", True)])
def test_port_equals_sdk_live(oracle_mod, group, dtype, causal):
    """The restatement against the SDK's tensor_sdpa_f32 on seeded paged data."""
    seed, bs, d, kvh = 100 + group, 16, 64, 2
    qh = kvh * group
    lengths = np.array([3, 33, 70], np.int64)
    tables, _ = W.shuffled_tables(lengths, bs, 16, seed)
    kpool = W.normal_bits(seed, (16 * bs, kvh * d), dtype, stream=1)
    vpool = W.normal_bits(seed, (16 * bs, kvh * d), dtype, stream=2)
    nq = np.array([1, 5, 9]) if causal else np.ones(3, np.int64)
    offs = np.concatenate([[0], np.cumsum(nq)]).astype(np.int32)
    q = W.normal_bits(seed, (int(offs[-1]), qh, d), dtype, stream=3)
    job = oracle_mod.RefJob(dtype, q, offs, kpool, vpool, kvh, d, bs, tables, lengths, qh, 0.125,
                            causal)
    job.run(2)
    for b in range(3):
        pos = np.arange(lengths[b] - nq[b], lengths[b])
        got = oracle_mod.paged_attention_rows(q[offs[b]:offs[b + 1]], pos, causal, dtype, kpool,
                                              vpool, kvh, d, bs, tables[b], int(lengths[b]), 0.125)
        want = job.output(b)
        if causal:
            assert np.max(np.abs(got - want)) <= 1e-6
        else:
            assert np.array_equal(got, want)


def test_threaded_sdk_reference_splits_a_causal_chunk_exactly(oracle_mod):
    """The full-size GPU tests cut a causal chunk into row blocks, block j a
    sequence of length past + its last row, so the host threads share the
    SDK's tensor_sdpa_f32 calls; that must give the same bits as the
    restatement on the whole chunk, and the decode form (one row per
    sequence) the same as paged_decode."""
    from tests.gpu_cases import sdk_paged_attention
    lengths = np.array([300 + 64], np.int64)
    tables, _ = W.shuffled_tables(lengths, 16, 40, seed=4)
    kp = W.normal_bits(4, (40 * 16, 2 * 64), "bf16", stream=1)
    vp = W.normal_bits(4, (40 * 16, 2 * 64), "bf16", stream=2)
    q = W.normal_bits(4, (64, 8, 64), "bf16", stream=3)
    whole = oracle_mod.paged_attention_rows(q, 300 + np.arange(64), True, "bf16", kp, vp, 2, 64,
                                            16, tables[0], 364, 0.125)
    blk = 16
    outs = sdk_paged_attention(oracle_mod, "bf16", q, blk * np.arange(5), kp, vp, 2, 64, 16,
                               np.repeat(tables, 4, axis=0), 300 + blk * np.arange(1, 5), 8,
                               0.125, True)
    assert np.array_equal(np.concatenate(outs), whole)
    lens = np.array([5, 200, 17], np.int64)
    t3, _ = W.shuffled_tables(lens, 16, 40, seed=5)
    q3 = W.normal_bits(5, (3, 8, 64), "bf16", stream=3)
    dec = sdk_paged_attention(oracle_mod, "bf16", q3, None, kp, vp, 2, 64, 16, t3, lens, 8,
                              0.125, False)
    want = oracle_mod.paged_decode(q3, "bf16", kp, vp, 2, 64, 16, t3, lens, 0.125)
    assert np.array_equal(np.stack([o[0] for o in dec]), want)
