"""Timed CPU baselines of the reference algorithm (oracle port; used only by
bench.py's ``cpu_baseline`` leg, its per-config CPU figures and its
``--impl reference`` arm).  Every sample is numpy on the host cores, with the
work the reference's CPU torch path does for the same step:

* ``LayerSample`` -- one decode token of the Qwen3-VL-4B config: one decoder
  layer at the given context (NF4 dequant of every linear on every call, as
  the reference's 4-bit path does, then fp32 matmul; int8 KV prefix dequant +
  fp32 attention over the prefix and the fp16 ring) plus 1/num_layers of the
  4-bit lm_head rows, for ``batch`` rows (the weights dequantized once per
  step; ``attn_rows`` of the rows' attentions timed and scaled to ``batch``).
  ``seconds_per_step = num_layers * sample``.
* ``Config1Sample``: the decode append of a token that
  completes a 64-token group (the group requantized) + attention of 32 q heads
  over 8 int8 KV heads at ctx 4096.
* ``GemvSample`` -- one NF4 projection at batch 1: dequant + fp32 matmul.
* ``AttnSlice`` -- the decode attention of one batch row and one KV head (its
  4 query heads) over ``ctx`` int8 tokens (+ window); scaled by batch x KV heads.
"""

from __future__ import annotations

import os
import statistics
import time

import numpy as np

from . import kvquant as okv
from .attention import streaming_attend
from .nf4 import dequantize_nf4, nf4_codebook, quantize_nf4
from .norm import apply_rope, rms_norm, rope_cos_sin, silu_mul


def _rand_nf4(rng, n, k, code):
    w = (rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float16)
    return quantize_nf4(w, code)


def _lin(x, w, code):
    return (np.asarray(x, np.float32) @ dequantize_nf4(w[0], w[1], code).T).astype(np.float16)


def median_time(fn, budget_s: float = 2.0, max_runs: int = 50, min_runs: int = 3) -> tuple[float, int]:
    """Median wall time of ``fn()`` over as many runs as fit ``budget_s`` (after
    one untimed run), at least ``min_runs``; returns (seconds, runs)."""
    fn()
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < min_runs or (time.perf_counter() < t_end and len(times) < max_runs):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    return statistics.median(times), len(times)


class LayerSample:
    def __init__(self, ctx: int = 8192, hidden: int = 2560, q_heads: int = 32, kv_heads: int = 8, d: int = 128,
                 inter: int = 9728, vocab: int = 151936, layers: int = 36, seed: int = 0, batch: int = 1,
                 attn_rows: int | None = None) -> None:
        rng = np.random.default_rng(seed)
        self.code = nf4_codebook()
        self.layers, self.batch = layers, int(batch)
        self.attn_rows = self.batch if attn_rows is None else max(1, min(int(attn_rows), self.batch))
        self.hidden, self.hq, self.hkv, self.d, self.inter = hidden, q_heads, kv_heads, d, inter
        qd, kd = q_heads * d, kv_heads * d
        self.qkv = _rand_nf4(rng, qd + 2 * kd, hidden, self.code)
        self.o = _rand_nf4(rng, hidden, qd, self.code)
        self.gate = _rand_nf4(rng, inter, hidden, self.code)
        self.up = _rand_nf4(rng, inter, hidden, self.code)
        self.down = _rand_nf4(rng, hidden, inter, self.code)
        rows = -(-vocab // layers) // 16 * 16
        self.head = _rand_nf4(rng, rows, hidden, self.code)
        self.ones = np.ones(hidden, np.float16)
        self.ones_d = np.ones(d, np.float16)
        q_len = ctx // 64 * 64
        kv = (rng.standard_normal((2, 1, kv_heads, q_len, d), dtype=np.float32) * 0.7).astype(np.float16)
        self.kq, self.kmn, self.kst = okv.quantize_int8_token(kv[0], 64)
        self.vq, self.vmn, self.vst = okv.quantize_int8_token(kv[1], 64)
        self.tail_k = (rng.standard_normal((1, kv_heads, 64, d), dtype=np.float32) * 0.7).astype(np.float16)
        self.tail_v = self.tail_k.copy()
        self.ctx, self.q_len = ctx, q_len
        self.h = (rng.standard_normal((self.batch, hidden), dtype=np.float32)).astype(np.float16)
        self.cos, self.sin = rope_cos_sin([ctx], d)

    def run(self) -> float:
        """One sample; returns the seconds of one layer's step for ``batch``
        rows (the timed attentions scaled to all rows)."""
        hq, hkv, d, B = self.hq, self.hkv, self.d, self.batch
        t0 = time.perf_counter()
        x = rms_norm(self.h, self.ones)
        qkv = _lin(x, self.qkv, self.code)
        q = rms_norm(qkv[:, :hq * d].reshape(B, hq, d), self.ones_d)
        k = rms_norm(qkv[:, hq * d:(hq + hkv) * d].reshape(B, hkv, d), self.ones_d)
        q = apply_rope(q, self.cos[0], self.sin[0])
        self.tail_k[:, :, self.ctx % 64] = apply_rope(k[:1], self.cos[0], self.sin[0])
        t_lin = time.perf_counter() - t0
        t1 = time.perf_counter()
        outs = [streaming_attend(q[r:r + 1], self.kq, self.kmn, self.kst, self.vq, self.vmn, self.vst, self.tail_k,
                                 self.tail_v, written=self.ctx + 1, qlen=self.q_len)[0] for r in range(self.attn_rows)]
        t_att = (time.perf_counter() - t1) * B / self.attn_rows
        t2 = time.perf_counter()
        o = np.concatenate([outs[r % len(outs)] for r in range(B)]).reshape(B, -1)
        h = (self.h.astype(np.float32) + _lin(o, self.o, self.code).astype(np.float32)).astype(np.float16)
        x2 = rms_norm(h, self.ones)
        act = silu_mul(_lin(x2, self.gate, self.code), _lin(x2, self.up, self.code))
        h = (h.astype(np.float32) + _lin(act, self.down, self.code).astype(np.float32)).astype(np.float16)
        _ = _lin(rms_norm(h, self.ones), self.head, self.code)
        return t_lin + t_att + (time.perf_counter() - t2)


class Config1Sample:
    """Append (group-completing token, ring requantized) + attention at ctx 4096."""

    def __init__(self, ctx: int = 4096, q_heads: int = 32, kv_heads: int = 8, d: int = 128, seed: int = 0) -> None:
        rng = np.random.default_rng(seed)
        q_len = ctx - 64
        kv = rng.standard_normal((2, 1, kv_heads, q_len, d), dtype=np.float32).astype(np.float16)
        self.kq = np.zeros((1, kv_heads, ctx, d), np.uint8)
        self.vq = np.zeros_like(self.kq)
        self.kmn, self.kst, self.vmn, self.vst = (np.zeros((1, kv_heads, ctx // 64, d), np.float16) for _ in range(4))
        c, m, s = okv.quantize_int8_token(kv[0], 64)
        self.kq[:, :, :q_len], self.kmn[:, :, :-1], self.kst[:, :, :-1] = c, m, s
        c, m, s = okv.quantize_int8_token(kv[1], 64)
        self.vq[:, :, :q_len], self.vmn[:, :, :-1], self.vst[:, :, :-1] = c, m, s
        self.tail_k = rng.standard_normal((1, kv_heads, 64, d), dtype=np.float32).astype(np.float16)
        self.tail_v = rng.standard_normal((1, kv_heads, 64, d), dtype=np.float32).astype(np.float16)
        self.q = rng.standard_normal((1, q_heads, d), dtype=np.float32).astype(np.float16)
        self.ctx, self.g = ctx, ctx // 64 - 1

    def run(self) -> None:
        g = self.g
        for ring, codes, mn, st in ((self.tail_k, self.kq, self.kmn, self.kst),
                                    (self.tail_v, self.vq, self.vmn, self.vst)):
            c, m, s = okv.quantize_ring(ring)
            codes[:, :, g * 64:(g + 1) * 64], mn[:, :, g], st[:, :, g] = c, m, s
        streaming_attend(self.q, self.kq, self.kmn, self.kst, self.vq, self.vmn, self.vst, self.tail_k, self.tail_v,
                         written=self.ctx, qlen=self.ctx)


class GemvSample:
    """One NF4 projection [n, k] at batch 1: dequant + fp32 matmul -> fp16.
    ``rows`` < n times that many output rows (the cost is linear in them);
    ``scale`` = n / rows converts a sample to the whole projection."""

    def __init__(self, n: int, k: int, seed: int = 0, rows: int | None = None) -> None:
        rng = np.random.default_rng(seed)
        self.code = nf4_codebook()
        rows = n if rows is None else min(n, int(rows))
        self.scale = n / rows
        self.w = _rand_nf4(rng, rows, k, self.code)
        self.x = rng.standard_normal((1, k), dtype=np.float32).astype(np.float16)

    def run(self) -> None:
        _lin(self.x, self.w, self.code)


class AttnSlice:
    """Decode attention of one batch row and one KV head (4 q heads) over ctx
    int8 tokens (window: only the last ``window`` positions); the full case is
    ``batch * kv_heads`` of these."""

    def __init__(self, ctx: int, window: int = 0, gq: int = 4, d: int = 128, seed: int = 0) -> None:
        rng = np.random.default_rng(seed)
        self.kq = rng.integers(0, 256, (1, 1, ctx, d), dtype=np.uint8)
        self.vq = rng.integers(0, 256, (1, 1, ctx, d), dtype=np.uint8)
        self.sc = [(rng.random((1, 1, ctx // 64, d), dtype=np.float32) * 0.01).astype(np.float16) for _ in range(4)]
        self.q = rng.standard_normal((1, gq, d), dtype=np.float32).astype(np.float16)
        self.ctx, self.window = ctx, window

    def run(self) -> None:
        streaming_attend(self.q, self.kq, self.sc[0], self.sc[1], self.vq, self.sc[2], self.sc[3], None, None,
                         written=self.ctx, qlen=self.ctx, window=self.window)


def host_threads() -> int:
    return len(os.sched_getaffinity(0))
