"""The CPU restatement of the SDK's paged decoder (orc_decode_sequence)
against an independent float64 numpy model of the same math, and its own
continuation property (the SDK's test_attention.c checks that decoding in two
calls gives the tokens of one call)."""
from __future__ import annotations

import numpy as np
import pytest

from tests.decoder_cases import Model


def numpy_step(m: Model, token: int, kcache, vcache, pos: int, eps=1e-5, theta=10000.0):
    """One decode step in float64 with no storage rounding: returns logits.
    kcache/vcache: lists of float64 [capacity, kv_width], updated at pos."""
    x = m.embedding[token].astype(np.float64)
    hd, half = m.hd, m.hd // 2

    def rms(v, w):
        return v / np.sqrt(np.mean(v * v) + eps) * w

    def rope(v):
        out = v.copy()
        for base in range(0, len(v), hd):
            for dim in range(hd):
                f = dim if dim < half else dim - half
                ang = pos / theta ** (2.0 * f / hd)
                pair = base + (dim + half if dim < half else dim - half)
                sign = -1.0 if dim < half else 1.0
                out[base + dim] = v[base + dim] * np.cos(ang) + sign * v[pair] * np.sin(ang)
        return out

    for l, t in enumerate(m.layers):
        n = rms(x, t[0])
        q, k, v = t[1] @ n, t[2] @ n, t[3] @ n
        q, k = rope(q), rope(k)
        kcache[l][pos], vcache[l][pos] = k, v
        att = np.zeros(m.hidden)
        g = m.qh // m.kvh
        for h in range(m.qh):
            kh = h // g
            K = kcache[l][:pos + 1, kh * hd:(kh + 1) * hd]
            V = vcache[l][:pos + 1, kh * hd:(kh + 1) * hd]
            s = K @ q[h * hd:(h + 1) * hd] / np.sqrt(hd)
            p = np.exp(s - s.max())
            att[h * hd:(h + 1) * hd] = (p / p.sum()) @ V
        r = t[4] @ att + x
        n2 = rms(r, t[5])
        gate, up = t[6] @ n2, t[7] @ n2
        x = t[8] @ (gate / (1 + np.exp(-gate)) * up) + r
    return m.lm_head @ rms(x, m.final_norm)


def test_oracle_matches_float64_model(oracle_mod):
    m = Model("f32", 2, 64, 96, 4, 2, 16, 50, seed=1)
    cap = 8
    kc = [np.zeros((cap, m.kvw), np.float32) for _ in range(2)]
    vc = [np.zeros((cap, m.kvw), np.float32) for _ in range(2)]
    toks, logits, _, _ = m.oracle(oracle_mod, 3, 4, kc, vc, 0, cap)
    k64 = [np.zeros((cap, m.kvw)) for _ in range(2)]
    v64 = [np.zeros((cap, m.kvw)) for _ in range(2)]
    token = 3
    for t in range(4):
        ref = numpy_step(m, token, k64, v64, t)
        np.testing.assert_allclose(logits[t], ref, rtol=1e-4, atol=1e-4)
        assert toks[t] == int(np.argmax(ref))
        token = toks[t]


@pytest.mark.parametrize("kind", ["f32", "f16", "q8", "q4"])
def test_two_calls_equal_one(oracle_mod, kind):
    m = Model(kind, 2, 64, 128, 4, 2, 16, 40, seed=2)
    cap = 16
    kc = [np.zeros((cap, m.kvw), m.cache_dtype()) for _ in range(2)]
    vc = [np.zeros((cap, m.kvw), m.cache_dtype()) for _ in range(2)]
    full, _, _, _ = m.oracle(oracle_mod, 5, 6, kc, vc, 0, cap)
    first, _, k1, v1 = m.oracle(oracle_mod, 5, 3, kc, vc, 0, cap)
    second, _, _, _ = m.oracle(oracle_mod, first[-1], 3, k1, v1, 3, cap)
    assert first + second == full


def test_prefix_rows_are_kept(oracle_mod):
    m = Model("f16", 1, 32, 64, 2, 1, 16, 20, seed=3)
    cap = 12
    kc, vc = m.prefix(5, cap, seed=4)
    _, _, k2, v2 = m.oracle(oracle_mod, 1, 3, kc, vc, 5, cap)
    assert np.array_equal(k2[0][:5], kc[0][:5]) and np.array_equal(v2[0][:5], vc[0][:5])
    assert (k2[0][5:8] != 0).any() and not k2[0][8:].any()
