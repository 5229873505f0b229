"""Seeded dense decoder models for the paged decoder entry point
(tensor_attention_decode_sequence_paged): weights in the three storage kinds
of include/attention.h, Q8_0/Q4_0 block packing, and the token comparison
the tests use.

Weights are synthetic (seeded normal); no checkpoint is involved.  Q*_0
blocks follow the GGML layout the SDK consumes (a half scale, then 32 int8
values or 16 bytes of nibbles with value q - 8; attention_cuda.cu:197-206);
the packing here is this file's own (round to nearest of x / scale).
"""
from __future__ import annotations

import numpy as np

from inference_c_b200 import workloads as W

STORAGE = {"f32": 0, "f16": 1, "q8": 2, "q4": 2}
QUANT = {"f32": 0, "f16": 0, "q8": 1, "q4": 2}


def f16_bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, np.float32).astype(np.float16)).view(np.uint16)


def quantize(m: np.ndarray, fmt: str) -> np.ndarray:
    """[out, in] float matrix (in % 32 == 0) -> [out, in/32, 34|18] uint8 blocks."""
    out, inp = m.shape
    blocks = m.reshape(out, inp // 32, 32).astype(np.float32)
    if fmt == "q8":
        amax = np.abs(blocks).max(axis=2, keepdims=True)
        scale = (amax / 127.0).astype(np.float16).astype(np.float32)
        q = np.where(scale > 0, np.rint(blocks / np.where(scale > 0, scale, 1)), 0)
        q = np.clip(q, -127, 127).astype(np.int8)
        res = np.zeros((out, inp // 32, 34), np.uint8)
        res[:, :, 0:2] = scale.astype(np.float16).view(np.uint8).reshape(out, inp // 32, 2)
        res[:, :, 2:] = q.view(np.uint8)
        return res
    amax = np.abs(blocks).max(axis=2, keepdims=True)
    scale = (amax / 7.0).astype(np.float16).astype(np.float32)
    q = np.where(scale > 0, np.rint(blocks / np.where(scale > 0, scale, 1)), 0)
    q = (np.clip(q, -8, 7) + 8).astype(np.uint8)
    res = np.zeros((out, inp // 32, 18), np.uint8)
    res[:, :, 0:2] = scale.astype(np.float16).view(np.uint8).reshape(out, inp // 32, 2)
    res[:, :, 2:] = (q[:, :, :16] & 15) | ((q[:, :, 16:] & 15) << 4)
    return res


class Model:
    """A seeded decoder stack in one storage kind ('f32', 'f16', 'q8', 'q4')."""

    def __init__(self, kind: str, layers: int, hidden: int, inter: int, qh: int, kvh: int,
                 hd: int, vocab: int, seed: int, logit_scale: float = 4.0):
        assert qh * hd == hidden and qh % kvh == 0
        self.kind, self.storage, self.fmt = kind, STORAGE[kind], QUANT[kind]
        self.n_layers, self.hidden, self.inter = layers, hidden, inter
        self.qh, self.kvh, self.hd, self.vocab = qh, kvh, hd, vocab
        self.kvw = kvh * hd
        rng = np.random.default_rng(seed)

        def mat(o, i, gain=1.0):
            return (rng.standard_normal((o, i)) * gain / np.sqrt(i)).astype(np.float32)

        def norm(n):
            return (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)

        self.layers = []
        for _ in range(layers):
            self.layers.append([norm(hidden), mat(hidden, hidden), mat(self.kvw, hidden),
                                mat(self.kvw, hidden), mat(hidden, hidden, 0.5), norm(hidden),
                                mat(inter, hidden), mat(inter, hidden), mat(hidden, inter, 0.5)])
        self.embedding = rng.standard_normal((vocab, hidden)).astype(np.float32)
        self.final_norm = norm(hidden)
        self.lm_head = mat(vocab, hidden, logit_scale)

    # storage-format arrays
    def _vec(self, v):
        return v if self.kind == "f32" else f16_bits(v)

    def _mat(self, m):
        if self.kind == "f32":
            return m
        if self.kind == "f16":
            return f16_bits(m)
        return quantize(m, self.kind)

    def layer_tensors(self):
        out = []
        for t in self.layers:
            out.append([self._vec(t[0]), self._mat(t[1]), self._mat(t[2]), self._mat(t[3]),
                        self._mat(t[4]), self._vec(t[5]), self._mat(t[6]), self._mat(t[7]),
                        self._mat(t[8])])
        return out

    def embedding_s(self):
        return self._vec(self.embedding)

    def final_norm_s(self):
        return self._vec(self.final_norm)

    def lm_head_s(self):
        return self._mat(self.lm_head)

    def cache_dtype(self):
        return np.float32 if self.kind == "f32" else np.uint16

    def prefix(self, past: int, capacity: int, seed: int):
        """Host prefix K/V per layer ([capacity, kv_width], rows < past set)."""
        rng = np.random.default_rng(seed)
        ks, vs = [], []
        for _ in range(self.n_layers):
            k = np.zeros((capacity, self.kvw), np.float32)
            v = np.zeros((capacity, self.kvw), np.float32)
            k[:past] = rng.standard_normal((past, self.kvw))
            v[:past] = rng.standard_normal((past, self.kvw))
            ks.append(k if self.kind == "f32" else f16_bits(k))
            vs.append(v if self.kind == "f32" else f16_bits(v))
        return ks, vs

    def request_args(self):
        return dict(hidden=self.hidden, inter=self.inter, qh=self.qh, kvh=self.kvh, hd=self.hd,
                    vocab=self.vocab)

    def oracle(self, oracle_mod, initial_token, count, kcache, vcache, past, capacity,
               eps=1e-5, theta=10000.0):
        """Runs orc_decode_sequence on copies of the caches; returns
        (tokens, logits per step, kcache, vcache)."""
        kc = [np.ascontiguousarray(k.copy()) for k in kcache]
        vc = [np.ascontiguousarray(v.copy()) for v in vcache]
        toks, logits = oracle_mod.decode_sequence(
            self.storage, self.fmt, self.layer_tensors(), self.embedding_s(), initial_token,
            count, kc, vc, past, capacity, self.hidden, self.inter, self.qh, self.kvh, self.hd,
            eps, theta, self.final_norm_s(), self.lm_head_s(), self.vocab, want_logits=True)
        return toks, logits, kc, vc


def assert_tokens_agree(got, want, logits, what=""):
    """Tokens must be equal; the only tolerated difference is a near-tie of
    the oracle's logits at the first step where they differ (the GPU's sums
    differ from the oracle's in the last bits), after which the two
    trajectories are no longer comparable."""
    assert got is not None, f"{what}: the call returned 0"
    assert len(got) == len(want), (got, want)
    for t, (g, w) in enumerate(zip(got, want)):
        if g == w:
            continue
        lg, lw = float(logits[t][g]), float(logits[t][w])
        assert abs(lg - lw) <= 2e-3 + 2e-3 * abs(lw), (
            f"{what}: step {t} token {g} vs oracle {w} (logits {lg} vs {lw}); got {got}, "
            f"want {want}")
        return t
    return len(got)


__all__ = ["Model", "quantize", "f16_bits", "assert_tokens_agree", "W"]
