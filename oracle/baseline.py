"""Timed CPU baseline of the reference decode algorithm (oracle port; used only
by bench.py's ``cpu_baseline`` leg and its ``--impl reference`` arm).

A bounded sample of one decode token of the full Qwen3-VL-4B config: one
decoder layer at the given context (NF4 dequant of every linear on every
call, as the reference's 4-bit path does, then fp32 matmul; int8 KV prefix
dequant + fp32 attention over the prefix and the fp16 ring) plus 1/num_layers
of the 4-bit lm_head rows.  With ``slice = S`` every linear keeps 1/S of its
output rows and the attention 1/S of the KV heads (the work is linear in
both), so ``seconds_per_token = num_layers * S * sample``.
"""

from __future__ import annotations

import os
import time

import numpy as np

from . import kvquant as okv
from .attention import streaming_attend
from .nf4 import dequantize_nf4, nf4_codebook, quantize_nf4
from .norm import apply_rope, rms_norm, rope_cos_sin, silu_mul


def _rand_nf4(rng, n, k, code):
    w = (rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float16)
    return quantize_nf4(w, code)


class LayerSample:
    def __init__(self, ctx: int = 8192, hidden: int = 2560, q_heads: int = 32, kv_heads: int = 8, d: int = 128,
                 inter: int = 9728, vocab: int = 151936, layers: int = 36, seed: int = 0, slice: int = 1) -> None:
        rng = np.random.default_rng(seed)
        self.code = nf4_codebook()
        self.layers, self.slice = layers, int(slice)
        S = self.slice
        if q_heads % S or kv_heads % S or hidden % (64 * S) or inter % (64 * S):
            raise ValueError(f"slice {S} must divide the heads and the hidden / intermediate blocks")
        q_heads, kv_heads = q_heads // S, kv_heads // S
        self.hidden, self.hq, self.hkv, self.d, self.inter = hidden, q_heads, kv_heads, d, inter
        qd, kd = q_heads * d, kv_heads * d
        self.qkv = _rand_nf4(rng, qd + 2 * kd, hidden, self.code)
        self.o = _rand_nf4(rng, hidden // S, qd * S, self.code)
        self.gate = _rand_nf4(rng, inter // S, hidden, self.code)
        self.up = _rand_nf4(rng, inter // S, hidden, self.code)
        self.down = _rand_nf4(rng, hidden // S, inter, self.code)
        rows = -(-vocab // (layers * S)) // 16 * 16
        self.head = _rand_nf4(rng, rows, hidden, self.code)
        self.ones = np.ones(hidden, np.float16)
        self.ones_d = np.ones(d, np.float16)
        q_len = ctx // 64 * 64
        kv = (rng.standard_normal((2, 1, kv_heads, q_len, d), dtype=np.float32) * 0.7).astype(np.float16)
        self.seconds_scale = layers * S
        self.kq, self.kmn, self.kst = okv.quantize_int8_token(kv[0], 64)
        self.vq, self.vmn, self.vst = okv.quantize_int8_token(kv[1], 64)
        self.tail_k = (rng.standard_normal((1, kv_heads, 64, d), dtype=np.float32) * 0.7).astype(np.float16)
        self.tail_v = self.tail_k.copy()
        self.ctx, self.q_len = ctx, q_len
        self.h = (rng.standard_normal((1, hidden), dtype=np.float32)).astype(np.float16)
        self.cos, self.sin = rope_cos_sin([ctx], d)

    def _lin(self, x, w):
        return (np.asarray(x, np.float32) @ dequantize_nf4(w[0], w[1], self.code).T).astype(np.float16)

    def run(self) -> float:
        """One sample; returns its wall time in seconds."""
        t0 = time.perf_counter()
        hq, hkv, d = self.hq, self.hkv, self.d
        x = rms_norm(self.h, self.ones)
        qkv = self._lin(x, self.qkv)
        q = rms_norm(qkv[:, :hq * d].reshape(1, hq, d), self.ones_d)
        k = rms_norm(qkv[:, hq * d:(hq + hkv) * d].reshape(1, hkv, d), self.ones_d)
        q = apply_rope(q, self.cos[0], self.sin[0])
        self.tail_k[:, :, self.ctx % 64] = apply_rope(k, self.cos[0], self.sin[0])
        o, _ = streaming_attend(q, self.kq, self.kmn, self.kst, self.vq, self.vmn, self.vst, self.tail_k,
                                self.tail_v, written=self.ctx + 1, qlen=self.q_len)
        S = self.slice
        o_in = np.tile(o.reshape(1, -1), (1, S))                  # o_proj reads all q heads
        oo = self._lin(o_in, self.o)
        h = self.h.copy()
        h[:, :oo.shape[1]] = (h[:, :oo.shape[1]].astype(np.float32) + oo.astype(np.float32)).astype(np.float16)
        x2 = rms_norm(h, self.ones)
        act = silu_mul(self._lin(x2, self.gate), self._lin(x2, self.up))
        act = np.tile(act, (1, S))                                 # down reads the full intermediate
        dd = self._lin(act, self.down)
        h[:, :dd.shape[1]] = (h[:, :dd.shape[1]].astype(np.float32) + dd.astype(np.float32)).astype(np.float16)
        _ = self._lin(rms_norm(h, self.ones), self.head)
        return time.perf_counter() - t0


def host_threads() -> int:
    return len(os.sched_getaffinity(0))
