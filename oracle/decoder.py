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
from .nf4 import dequantize_nf4, nf4_codebook, quantize_nf4
from .norm import apply_rope, rms_norm, rope_cos_sin, silu_mul

GT = 64
LM_HEAD_ROWS = 16384   # lm_head rows dequantized at a time by the batched path (bounds host memory)


def random_weights(*, vocab: int, hidden: int, layers: int, q_heads: int, kv_heads: int, inter: int,
                   head_dim: int = 128, seed: int = 0, std: float = 0.02, norm_jitter: float = 0.1) -> dict:
    """Seeded random-init decoder weights in the layout ``OracleDecoder`` takes
    (the dict ``nova_b200.decoder.weights_to_numpy`` produces): every linear
    N(0, std) in fp32, rounded to fp16, NF4-quantized with fp16 absmax; norm
    weights 1 + norm_jitter * N(0, 1) in fp16; the embedding N(0, std) fp16
    with its NF4 copy as the tied lm_head.  numpy's PCG64 stream, so the same
    seed gives the same weights on any host."""
    rng = np.random.default_rng(seed)
    code = nf4_codebook()

    def lin(n, k):
        w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(std)).astype(np.float16)
        return quantize_nf4(w, code, absmax_dtype=np.float16)

    def norm(n):
        return (1.0 + norm_jitter * rng.standard_normal(n, dtype=np.float32)).astype(np.float16)

    out = {"code": code, "layers": []}
    qd, kvd = q_heads * head_dim, kv_heads * head_dim
    for _ in range(layers):
        q, k, v = lin(qd, hidden), lin(kvd, hidden), lin(kvd, hidden)
        out["layers"].append({
            "qkv": (np.concatenate([q[0], k[0], v[0]]), np.concatenate([q[1], k[1], v[1]], axis=1)),
            "o": lin(hidden, qd), "gate": lin(inter, hidden), "up": lin(inter, hidden), "down": lin(hidden, inter),
            "input_ln": norm(hidden), "post_ln": norm(hidden), "q_norm": norm(head_dim), "k_norm": norm(head_dim)})
    out["embed"] = (rng.standard_normal((vocab, hidden), dtype=np.float32) * np.float32(std)).astype(np.float16)
    out["lm_head"] = quantize_nf4(out["embed"], code, absmax_dtype=np.float16)
    out["final_norm"] = norm(hidden)
    return out


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

    def _lin_once(self, x, pa, rows: int | None = None):
        """``_lin`` without keeping the dequantized weight (the batched path
        uses each weight once); ``rows`` dequantizes that many output rows at a
        time."""
        packed, absmax = pa
        n = packed.shape[0]
        rows = n if rows is None else rows
        xf = np.asarray(x, np.float32)
        out = np.empty((*xf.shape[:-1], n), np.float16)
        for r0 in range(0, n, rows):
            r1 = min(n, r0 + rows)
            w = dequantize_nf4(packed[r0:r1], absmax[:, r0:r1], self.code)
            out[..., r0:r1] = _f16(xf @ w.T)
            del w
        return out

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

    def decode_teacher_forced(self, tokens: np.ndarray):
        """``len(tokens)`` decode steps from the current state, step i fed
        ``tokens[i]`` (``[S, B]`` ids): the same results as calling
        :meth:`step` S times with those inputs, computed one layer at a time
        for all steps at once (each weight dequantized once, one matmul per
        linear).  Step i attends, as the streaming cache does at that step,
        to the int8 form of every group complete at position p_i = pos + i
        and to the fp16 K/V of the rest; a group is quantized from the fp16
        K/V of its 64 positions (the ring the step completing it holds).
        Returns (logits fp16 ``[S, B, V]``, greedy tokens ``[S, B]``) and leaves
        the cache and ``pos`` as after the S steps."""
        tokens = np.asarray(tokens)
        S, B = tokens.shape
        hq, hkv, d = self.hq, self.hkv, self.d
        gq = hq // hkv
        pos0 = self.pos
        end = pos0 + S                                   # positions written after the last step
        q0 = pos0 // GT * GT                             # int8 prefix before the first step
        if end > self.max_len:
            raise ValueError(f"{S} steps from position {pos0} exceed the capacity {self.max_len}")
        steps_pos = pos0 + np.arange(S)
        cos, sin = rope_cos_sin(steps_pos, d, self.theta)
        h = np.asarray(self.W["embed"])[tokens]          # fp16 [S, B, H]
        scale = np.float32(d ** -0.5)
        for li, lw in enumerate(self.W["layers"]):
            x = rms_norm(h, lw["input_ln"], self.eps)
            qkv = self._lin_once(x, lw["qkv"])
            q = rms_norm(qkv[..., :hq * d].reshape(S, B, hq, d), lw["q_norm"], self.eps)
            k = rms_norm(qkv[..., hq * d:(hq + hkv) * d].reshape(S, B, hkv, d), lw["k_norm"], self.eps)
            v = qkv[..., (hq + hkv) * d:].reshape(S, B, hkv, d)
            q = apply_rope(q, cos[:, None, None], sin[:, None, None])
            k = apply_rope(k, cos[:, None, None], sin[:, None, None])
            # fp16 K/V of positions [q0, end): the prompt's open group from the ring, then the steps
            fk = np.empty((B, hkv, end - q0, d), np.float16)
            fv = np.empty_like(fk)
            for p in range(q0, pos0):
                fk[:, :, p - q0] = self.tail_k[li][:, :, p % GT]
                fv[:, :, p - q0] = self.tail_v[li][:, :, p % GT]
            fk[:, :, pos0 - q0:] = k.transpose(1, 2, 0, 3)
            fv[:, :, pos0 - q0:] = v.transpose(1, 2, 0, 3)
            for g in range(q0 // GT, end // GT):         # groups completed during these steps
                for src, codes, mn, st in ((fk, self.kq[li], self.kmn[li], self.kst[li]),
                                           (fv, self.vq[li], self.vmn[li], self.vst[li])):
                    c, m_, s_ = okv.quantize_ring(src[:, :, g * GT - q0:(g + 1) * GT - q0])
                    codes[:, :, g * GT:(g + 1) * GT] = c
                    mn[:, :, g] = m_
                    st[:, :, g] = s_
            qmax = end // GT * GT
            kd = okv.dequantize_int8_token(self.kq[li][:, :, :qmax], self.kmn[li][:, :, :qmax // GT],
                                           self.kst[li][:, :, :qmax // GT], GT).astype(np.float32)
            vd = okv.dequantize_int8_token(self.vq[li][:, :, :qmax], self.vmn[li][:, :, :qmax // GT],
                                           self.vst[li][:, :, :qmax // GT], GT).astype(np.float32)
            fkf, fvf = fk.astype(np.float32), fv.astype(np.float32)
            o = np.empty((S, B, hq * d), np.float16)
            qf = q.astype(np.float32)                    # [S, B, hq, d]
            i = 0
            while i < S:                                 # steps that share one int8 prefix length
                ql = (steps_pos[i] + 1) // GT * GT
                j = i
                while j < S and (steps_pos[j] + 1) // GT * GT == ql:
                    j += 1
                last = steps_pos[j - 1]
                n_f = last + 1 - ql                      # fp16 keys [ql, last]
                fpos = ql + np.arange(n_f)
                ok = fpos[None, :] <= steps_pos[i:j, None]          # [steps, n_f] causal
                for b in range(B):
                    for hh in range(hkv):
                        kk = np.concatenate([kd[b, hh, :ql], fkf[b, hh, ql - q0:last + 1 - q0]])
                        vv = np.concatenate([vd[b, hh, :ql], fvf[b, hh, ql - q0:last + 1 - q0]])
                        qq = qf[i:j, b, hh * gq:(hh + 1) * gq].reshape(-1, d)        # [steps*gq, d]
                        sc = (qq @ kk.T) * scale
                        valid = np.concatenate([np.ones((j - i, ql), bool), ok], axis=1)
                        sc = np.where(np.repeat(valid, gq, axis=0), sc, -np.inf)
                        mx = sc.max(axis=-1, keepdims=True)
                        pr = np.exp(sc - mx).astype(np.float32)
                        res = (pr @ vv) / pr.sum(axis=-1, keepdims=True)
                        o[i:j, b, hh * gq * d:(hh + 1) * gq * d] = res.reshape(j - i, gq * d).astype(np.float16)
                i = j
            h = _f16(h.astype(np.float32) + self._lin_once(o, lw["o"]).astype(np.float32))
            x2 = rms_norm(h, lw["post_ln"], self.eps)
            act = silu_mul(self._lin_once(x2, lw["gate"]), self._lin_once(x2, lw["up"]))
            h = _f16(h.astype(np.float32) + self._lin_once(act, lw["down"]).astype(np.float32))
            u = end - 1
            for slot in range(GT):                       # the ring as the last step leaves it
                p = u - (u - slot) % GT
                if p >= q0:
                    self.tail_k[li][:, :, slot] = fk[:, :, p - q0]
                    self.tail_v[li][:, :, slot] = fv[:, :, p - q0]
        x = rms_norm(h, self.W["final_norm"], self.eps)
        logits = self._lin_once(x, self.W["lm_head"], rows=LM_HEAD_ROWS)
        self.pos = end
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

    def capture_kv(self, ids: np.ndarray, span: tuple[int, int]):
        """K after k_norm and before RoPE, and V, of positions [span[0],
        span[1]) on every layer, from a causal forward over ``ids`` ``[1, T]``
        that leaves the cache untouched (capture_qkv / capture_kv,
        src/nova/memory.py:176-217, which hooks LeanAttention before RoPE,
        src/nova/layers.py:113-122).  Returns fp16 ``[layers, kv_heads, m, d]``."""
        ids = np.asarray(ids)
        B, T = ids.shape
        s0, s1 = int(span[0]), int(span[1])
        if B != 1 or not 0 <= s0 < s1 <= T:
            raise ValueError(f"capture needs batch 1 and 0 <= {s0} < {s1} <= {T}")
        hq, hkv, d = self.hq, self.hkv, self.d
        cos, sin = rope_cos_sin(np.arange(T), d, self.theta)
        h = np.asarray(self.W["embed"])[ids]
        ks, vs = [], []
        for li, lw in enumerate(self.W["layers"]):
            x = rms_norm(h, lw["input_ln"], self.eps)
            qkv = self._lin(x, ("qkv", li), lw["qkv"])
            q = rms_norm(qkv[..., :hq * d].reshape(B, T, hq, d), lw["q_norm"], self.eps)
            k = rms_norm(qkv[..., hq * d:(hq + hkv) * d].reshape(B, T, hkv, d), lw["k_norm"], self.eps)
            v = qkv[..., (hq + hkv) * d:].reshape(B, T, hkv, d)
            ks.append(k[0, s0:s1].transpose(1, 0, 2))
            vs.append(v[0, s0:s1].transpose(1, 0, 2))
            q = apply_rope(q, cos[None, :, None], sin[None, :, None]).transpose(0, 2, 1, 3)
            kr = apply_rope(k, cos[None, :, None], sin[None, :, None]).transpose(0, 2, 1, 3)
            vt = v.transpose(0, 2, 1, 3)
            o = np.empty((B, T, hq * d), np.float16)
            for t in range(T):
                ot, _ = attend(q[:, :, t], kr[:, :, :t + 1], vt[:, :, :t + 1])
                o[:, t] = ot.reshape(B, hq * d)
            h = _f16(h.astype(np.float32) + self._lin(o, ("o", li), lw["o"]).astype(np.float32))
            h = _f16(h.astype(np.float32) + self._mlp(li, lw, h).astype(np.float32))
        return np.stack(ks), np.stack(vs)

    def inject(self, k: np.ndarray, v: np.ndarray, offset: int = 0) -> int:
        """MemoryStore.inject (src/nova/memory.py:447-475) onto the streaming
        int8 cache: K (``[layers, kv_heads, m, d]``, before RoPE) rotated to
        positions [offset, offset + m) with the fp16 op-by-op RoPE
        (src/nova/layers.py:30-36), K/V appended to the fp16 K/V already
        written by earlier injections (offset must equal their length; 0
        starts afresh), then the cache as a prefill of [0, offset + m) leaves
        it (src/nova/kvattn.py:745-783): every complete 64-token group
        quantized on the token axis, the last <= 64 positions in the ring.
        Returns offset + m.  Batch 1."""
        L, hkv, m, d = k.shape
        offset = int(offset)
        have = 0 if offset == 0 or getattr(self, "_staged", None) is None else self._staged[0][0].shape[2]
        if offset != have:
            raise ValueError(f"offset {offset}: {have} positions written")
        total = offset + m
        cos, sin = rope_cos_sin(np.arange(offset, total), d, self.theta)
        staged = []
        for li in range(L):
            kr = apply_rope(np.asarray(k[li], np.float16), cos[None], sin[None])[None]
            vv = np.asarray(v[li], np.float16)[None]
            if offset:
                kr = np.concatenate([self._staged[li][0], kr], axis=2)
                vv = np.concatenate([self._staged[li][1], vv], axis=2)
            staged.append((kr, vv))
            full = total // GT * GT
            for src, codes, mn, st in ((kr, self.kq[li], self.kmn[li], self.kst[li]),
                                       (vv, self.vq[li], self.vmn[li], self.vst[li])):
                if full:
                    c, m_, s_ = okv.quantize_int8_token(np.ascontiguousarray(src[:, :, :full]), GT)
                    codes[:, :, :full], mn[:, :, :full // GT], st[:, :, :full // GT] = c, m_, s_
            for p in range(max(0, total - GT), total):
                self.tail_k[li][:, :, p % GT] = kr[:, :, p]
                self.tail_v[li][:, :, p % GT] = vv[:, :, p]
        self._staged = staged
        self.pos = total
        return total

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
