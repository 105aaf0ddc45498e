"""One greedy decode step of the lean Qwen3-VL text decoder with NF4 linears
and the streaming int8 KV cache, restated in numpy (oracle; test
infrastructure only).

Per layer (src/nova/layers.py:195-218, :99-174):
    x = input_layernorm(h)                          RMSNorm, HF order
    q, k, v = q_proj(x), k_proj(x), v_proj(x)       NF4 linear, fp16 out
    q, k = q_norm(q), k_norm(k)                     per-head RMSNorm
    q, k = RoPE(q, k) at position pos               fp16 op by op
    cache.update(k, v); o = cache.attend(q)         int8 prefix + fp16 ring
    h = h + o_proj(o)                               fp16 add
    h = h + down(silu(gate(x2)) * up(x2)),  x2 = post_attention_layernorm(h)
then final norm, the 4-bit lm_head (NF4 copy of embed_tokens), greedy argmax
(first maximal index) and pos += 1 (src/nova/model.py:115-204,
src/nova/decode.py:301-320).

Prefill (src/nova/decode.py:224-297, src/nova/kvattn.py:745-815): the prompt
attends causally over its own fp16 K/V; afterwards the complete 64-token
groups are quantized and the remaining tokens go to the ring.
"""

from __future__ import annotations

import numpy as np

from . import kvquant as okv
from .attention import attend, ring_positions, streaming_attend
from .nf4 import dequantize_nf4
from .norm import apply_rope, rms_norm, rope_cos_sin, silu_mul

GT = 64


def _f16(a):
    return np.asarray(a, np.float32).astype(np.float16)


class OracleDecoder:
    """``W`` is the dict of NF4 weights produced by
    ``nova_b200.decoder.weights_to_numpy`` (packed + absmax per linear)."""

    def __init__(self, W: dict, *, hidden: int, q_heads: int, kv_heads: int, head_dim: int = 128,
                 eps: float = 1e-6, theta: float = 5_000_000.0, max_len: int = 512, batch: int = 1) -> None:
        self.W = W
        self.code = np.asarray(W["code"], np.float32)
        self.hidden, self.hq, self.hkv, self.d = hidden, q_heads, kv_heads, head_dim
        self.eps, self.theta, self.max_len, self.batch = eps, theta, max_len, batch
        self._deq = {}
        L = len(W["layers"])
        ng = -(-max_len // GT)
        self.kq = [np.zeros((batch, kv_heads, max_len, head_dim), np.uint8) for _ in range(L)]
        self.vq = [np.zeros_like(self.kq[0]) for _ in range(L)]
        self.kmn, self.kst, self.vmn, self.vst = ([np.zeros((batch, kv_heads, ng, head_dim), np.float16)
                                                   for _ in range(L)] for _ in range(4))
        self.tail_k = [np.zeros((batch, kv_heads, GT, head_dim), np.float16) for _ in range(L)]
        self.tail_v = [np.zeros_like(self.tail_k[0]) for _ in range(L)]
        self.pos = 0

    # ---- weights
    def _w(self, key, pa):
        if key not in self._deq:
            self._deq[key] = dequantize_nf4(pa[0], pa[1], self.code).T.copy()   # [K, N] fp32
        return self._deq[key]

    def _lin(self, x, key, pa):
        """NF4 linear with fp32 accumulation, fp16 output (src/nova/kernels.py:187-240)."""
        return _f16(np.asarray(x, np.float32) @ self._w(key, pa))

    # ---- state exchange with the GPU decoder
    def load_state(self, st: dict) -> None:
        for name in ("kq", "vq", "kmn", "kst", "vmn", "vst", "tail_k", "tail_v"):
            setattr(self, name, [np.array(a) for a in st[name]])
        self.pos = int(st["pos"])

    # ---- one layer's attention block for a single query position
    def _attn_decode(self, li, lw, x, pos):
        B, hq, hkv, d = x.shape[0], self.hq, self.hkv, self.d
        qkv = self._lin(x, ("qkv", li), lw["qkv"])
        q = qkv[:, :hq * d].reshape(B, hq, d)
        k = qkv[:, hq * d:(hq + hkv) * d].reshape(B, hkv, d)
        v = qkv[:, (hq + hkv) * d:].reshape(B, hkv, d)
        q = rms_norm(q, lw["q_norm"], self.eps)
        k = rms_norm(k, lw["k_norm"], self.eps)
        cos, sin = rope_cos_sin([pos], d, self.theta)
        q = apply_rope(q, cos[0], sin[0])
        k = apply_rope(k, cos[0], sin[0])
        slot = pos % GT
        self.tail_k[li][:, :, slot] = k
        self.tail_v[li][:, :, slot] = v
        if slot == GT - 1:
            g = pos // GT
            for ring, codes, mn, st in ((self.tail_k[li], self.kq[li], self.kmn[li], self.kst[li]),
                                        (self.tail_v[li], self.vq[li], self.vmn[li], self.vst[li])):
                c, m, s = okv.quantize_ring(ring)
                codes[:, :, g * GT:(g + 1) * GT] = c
                mn[:, :, g] = m
                st[:, :, g] = s
        written = pos + 1
        qlen = written // GT * GT
        out, _ = streaming_attend(q, self.kq[li], self.kmn[li], self.kst[li], self.vq[li], self.vmn[li],
                                  self.vst[li], self.tail_k[li], self.tail_v[li], written=written, qlen=qlen)
        return out.reshape(B, hq * d)

    def _mlp(self, li, lw, h):
        x2 = rms_norm(h, lw["post_ln"], self.eps)
        gate = self._lin(x2, ("gate", li), lw["gate"])
        up = self._lin(x2, ("up", li), lw["up"])
        return self._lin(silu_mul(gate, up), ("down", li), lw["down"])

    def step(self, tokens: np.ndarray):
        """Decode one token per row at ``self.pos``; returns (logits fp16
        ``[B, V]``, greedy tokens ``[B]``)."""
        pos = self.pos
        h = np.asarray(self.W["embed"])[np.asarray(tokens)]                     # fp16 [B, H]
        for li, lw in enumerate(self.W["layers"]):
            x = rms_norm(h, lw["input_ln"], self.eps)
            o = self._attn_decode(li, lw, x, pos)
            h = _f16(h.astype(np.float32) + self._lin(o, ("o", li), lw["o"]).astype(np.float32))
            h = _f16(h.astype(np.float32) + self._mlp(li, lw, h).astype(np.float32))
        x = rms_norm(h, self.W["final_norm"], self.eps)
        logits = self._lin(x, ("lm_head", -1), self.W["lm_head"])
        self.pos = pos + 1
        return logits, np.argmax(logits.astype(np.float32), axis=-1)

    def prefill_chunked(self, ids: np.ndarray, chunk: int):
        """Prefill straight into the int8 cache in chunks of ``chunk`` tokens
        (a multiple of 64; reports/kv-int8-streaming-cache.md section 5.1 of
        the reference): each chunk attends to the int8 prefix of the earlier
        chunks, dequantized (src/nova/kvquant.py:166-176), and to its own fp16
        K/V, causally; its complete groups are quantized (token axis, 64-token
        groups) once the layer is done; the prompt's last <= 64 tokens go into
        the ring.  Returns (last-position logits, first greedy token)."""
        ids = np.asarray(ids)
        B, T = ids.shape
        hq, hkv, d = self.hq, self.hkv, self.d
        take0 = T - min(T, GT)
        for c0 in range(0, T, chunk):
            c1 = min(T, c0 + chunk)
            n = c1 - c0
            cos, sin = rope_cos_sin(np.arange(c0, c1), d, self.theta)
            h = np.asarray(self.W["embed"])[ids[:, c0:c1]]
            for li, lw in enumerate(self.W["layers"]):
                x = rms_norm(h, lw["input_ln"], self.eps)
                qkv = self._lin(x, ("qkv", li), lw["qkv"])
                q = rms_norm(qkv[..., :hq * d].reshape(B, n, hq, d), lw["q_norm"], self.eps)
                k = rms_norm(qkv[..., hq * d:(hq + hkv) * d].reshape(B, n, hkv, d), lw["k_norm"], self.eps)
                v = qkv[..., (hq + hkv) * d:].reshape(B, n, hkv, d)
                q = apply_rope(q, cos[None, :, None], sin[None, :, None]).transpose(0, 2, 1, 3)
                k = apply_rope(k, cos[None, :, None], sin[None, :, None]).transpose(0, 2, 1, 3)
                v = v.transpose(0, 2, 1, 3)
                K, V = k, v
                if c0:
                    g0 = c0 // GT
                    pk = okv.dequantize_int8_token(self.kq[li][:, :, :c0], self.kmn[li][:, :, :g0],
                                                   self.kst[li][:, :, :g0], GT)
                    pv = okv.dequantize_int8_token(self.vq[li][:, :, :c0], self.vmn[li][:, :, :g0],
                                                   self.vst[li][:, :, :g0], GT)
                    K, V = np.concatenate([pk, k], axis=2), np.concatenate([pv, v], axis=2)
                o = np.empty((B, n, hq * d), np.float16)
                for t in range(n):
                    ot, _ = attend(q[:, :, t], K[:, :, :c0 + t + 1], V[:, :, :c0 + t + 1])
                    o[:, t] = ot.reshape(B, hq * d)
                h = _f16(h.astype(np.float32) + self._lin(o, ("o", li), lw["o"]).astype(np.float32))
                h = _f16(h.astype(np.float32) + self._mlp(li, lw, h).astype(np.float32))
                full = n // GT * GT
                if full:
                    for src, codes, mn, st in ((k, self.kq[li], self.kmn[li], self.kst[li]),
                                               (v, self.vq[li], self.vmn[li], self.vst[li])):
                        c, m, s_ = okv.quantize_int8_token(np.ascontiguousarray(src[:, :, :full]), GT)
                        codes[:, :, c0:c0 + full] = c
                        mn[:, :, c0 // GT:(c0 + full) // GT] = m
                        st[:, :, c0 // GT:(c0 + full) // GT] = s_
                for p in range(max(c0, take0), c1):
                    self.tail_k[li][:, :, p % GT] = k[:, :, p - c0]
                    self.tail_v[li][:, :, p % GT] = v[:, :, p - c0]
        x = rms_norm(h[:, -1], self.W["final_norm"], self.eps)
        logits = self._lin(x, ("lm_head", -1), self.W["lm_head"])
        self.pos = T
        return logits, np.argmax(logits.astype(np.float32), axis=-1)

    def prefill(self, ids: np.ndarray):
        """Causal prefill over fp16 K/V from position 0; fills the int8 cache
        and the ring; returns (last-position logits, first greedy token)."""
        ids = np.asarray(ids)
        B, T = ids.shape
        hq, hkv, d = self.hq, self.hkv, self.d
        cos, sin = rope_cos_sin(np.arange(T), d, self.theta)
        h = np.asarray(self.W["embed"])[ids]                                     # [B, T, H]
        q_full = T // GT * GT
        for li, lw in enumerate(self.W["layers"]):
            x = rms_norm(h, lw["input_ln"], self.eps)
            qkv = self._lin(x, ("qkv", li), lw["qkv"])
            q = rms_norm(qkv[..., :hq * d].reshape(B, T, hq, d), lw["q_norm"], self.eps)
            k = rms_norm(qkv[..., hq * d:(hq + hkv) * d].reshape(B, T, hkv, d), lw["k_norm"], self.eps)
            v = qkv[..., (hq + hkv) * d:].reshape(B, T, hkv, d)
            q = apply_rope(q, cos[None, :, None], sin[None, :, None]).transpose(0, 2, 1, 3)   # [B, hq, T, d]
            k = apply_rope(k, cos[None, :, None], sin[None, :, None]).transpose(0, 2, 1, 3)   # [B, hkv, T, d]
            v = v.transpose(0, 2, 1, 3)
            o = np.empty((B, T, hq * d), np.float16)
            for t in range(T):
                ot, _ = attend(q[:, :, t], k[:, :, :t + 1], v[:, :, :t + 1])
                o[:, t] = ot.reshape(B, hq * d)
            h = _f16(h.astype(np.float32) + self._lin(o, ("o", li), lw["o"]).astype(np.float32))
            h = _f16(h.astype(np.float32) + self._mlp(li, lw, h).astype(np.float32))
            if q_full:
                for src, codes, mn, st in ((k, self.kq[li], self.kmn[li], self.kst[li]),
                                           (v, self.vq[li], self.vmn[li], self.vst[li])):
                    c, m, s = okv.quantize_int8_token(np.ascontiguousarray(src[:, :, :q_full]), GT)
                    codes[:, :, :q_full] = c
                    mn[:, :, :q_full // GT] = m
                    st[:, :, :q_full // GT] = s
            pos_ring = ring_positions(T)
            for slot in range(GT):
                p = pos_ring[slot]
                if 0 <= p < T and p >= T - GT:
                    self.tail_k[li][:, :, slot] = k[:, :, p]
                    self.tail_v[li][:, :, slot] = v[:, :, p]
        x = rms_norm(h[:, -1], self.W["final_norm"], self.eps)
        logits = self._lin(x, ("lm_head", -1), self.W["lm_head"])
        self.pos = T
        return logits, np.argmax(logits.astype(np.float32), axis=-1)
