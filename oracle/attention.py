"""Decode attention over the streaming int8 KV cache, restated in numpy
(oracle; test infrastructure only).

The reference computes one decode step as
  * int8 prefix ``[0, qlen)``: dequantize to fp16 (src/nova/kvquant.py:152-176)
    and attend in fp32 (SDPA math backend upcasts fp16 to fp32,
    tests/test_kvattn.py:62-71),
  * fp16 tail ring: the <=63 newest tokens, slot i holding absolute position
    ``p_i = u - ((u - i) mod 64)`` with ``u = written - 1``, valid when
    ``qlen <= p_i <= u`` and ``p_i >= first`` (src/nova/kvattn.py:819-833),
  * both merged by log-sum-exp (src/nova/kvattn.py:835-862).
Mathematically that is one softmax over the union of prefix tokens and valid
ring slots, which is what ``streaming_attend`` evaluates (the reference's own
streaming test uses exactly this single-softmax form as its ground truth,
tests/test_kvattn_stream.py:68-83).

The sliding-window variant keeps only positions with ``q - p < window``
(src/nova/decode.py:207-220, applied here to the int8 prefix as well).
"""

from __future__ import annotations

import numpy as np

from .kvquant import dequantize_int8_token


def attend(q: np.ndarray, k: np.ndarray, v: np.ndarray, valid: np.ndarray | None = None):
    """fp32 softmax attention for one query token.

    q: fp16 ``[B, Hq, D]``; k, v: fp16 ``[B, Hkv, T, D]``; valid: bool ``[B, T]``
    or ``[T]`` (None = all valid).  Query head h reads KV head ``h // (Hq/Hkv)``
    (repeat_kv, src/nova/layers.py:39-45).  Returns (out fp16 ``[B, Hq, D]``,
    lse fp32 ``[B, Hq]``); rows with no valid key give out=0, lse=-inf
    (src/nova/kvattn.py:241-253).
    """
    B, Hq, D = q.shape
    Hkv, T = k.shape[1], k.shape[2]
    gq = Hq // Hkv
    scale = np.float32(D ** -0.5)
    qf = q.astype(np.float32).reshape(B, Hkv, gq, D)
    kf = k.astype(np.float32)
    vf = v.astype(np.float32)
    s = np.einsum("bhgd,bhtd->bhgt", qf, kf, dtype=np.float32) * scale
    if valid is not None:
        vm = np.broadcast_to(np.asarray(valid, bool), (B, T))
        s = np.where(vm[:, None, None, :], s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    m_safe = np.where(np.isfinite(m), m, 0.0).astype(np.float32)
    p = np.exp(s - m_safe).astype(np.float32)
    l = p.sum(axis=-1, keepdims=True)
    o = np.einsum("bhgt,bhtd->bhgd", p, vf, dtype=np.float32)
    with np.errstate(invalid="ignore", divide="ignore"):
        out = np.where(l > 0, o / np.where(l > 0, l, 1), 0.0)
        lse = np.where(l[..., 0] > 0, m_safe[..., 0] + np.log(np.where(l[..., 0] > 0, l[..., 0], 1)), -np.inf)
    return out.reshape(B, Hq, D).astype(np.float16), lse.reshape(B, Hq).astype(np.float32)


def ring_positions(written: int, group: int = 64) -> np.ndarray:
    """Absolute position held by each ring slot (src/nova/kvattn.py:826)."""
    u = written - 1
    i = np.arange(group)
    return u - np.mod(u - i, group)


def streaming_attend(q, kq, kmn, kst, vq, vmn, vst, tail_k, tail_v, *, written: int, qlen: int,
                     first: int = 0, window: int = 0, group: int = 64):
    """One decode step of ``KVInt8Cache.attend`` as a single softmax.

    q fp16 ``[B,Hq,D]``; kq/vq uint8 ``[B,Hkv,L,D]``; scales fp16
    ``[B,Hkv,ceil(L/64),D]``; tail_k/v fp16 ``[B,Hkv,64,D]``.
    ``written`` = tokens written (the query sits at ``written-1``), ``qlen`` =
    int8 prefix length (a multiple of ``group`` in the cache path, any value
    for the plain fused-kernel API).  Returns (out fp16, lse fp32).
    """
    B = q.shape[0]
    u = written - 1
    kp = dequantize_int8_token(kq[:, :, :qlen], kmn, kst, group) if qlen else kq[:, :, :0].astype(np.float16)
    vp = dequantize_int8_token(vq[:, :, :qlen], vmn, vst, group) if qlen else vq[:, :, :0].astype(np.float16)
    pos_p = np.arange(qlen)
    valid_p = pos_p >= first
    if window:
        valid_p &= (u - pos_p) < window
    if tail_k is not None:
        pos_t = ring_positions(written, group)
        valid_t = (pos_t >= qlen) & (pos_t <= u) & (pos_t >= first)
        if window:
            valid_t &= (u - pos_t) < window
        k = np.concatenate([kp, tail_k], axis=2)
        v = np.concatenate([vp, tail_v], axis=2)
        valid = np.concatenate([valid_p, valid_t])
    else:
        k, v, valid = kp, vp, valid_p
    return attend(q, k, v, np.broadcast_to(valid, (B, valid.shape[0])))


def fused_prefix_attend(q, kq, kmn, kst, vq, vmn, vst, used: int, group: int = 64, window: int = 0,
                        qpos: int | None = None):
    """``int8_attn_decode(q, ..., used=used)`` semantics: attend over the int8
    codes ``[0, used)`` only (tests/test_kvattn.py:62-71).  ``window`` keeps
    positions ``p > qpos - window`` (``qpos`` defaults to ``used - 1``)."""
    k = dequantize_int8_token(np.ascontiguousarray(kq[:, :, :used]), kmn, kst, group)
    v = dequantize_int8_token(np.ascontiguousarray(vq[:, :, :used]), vmn, vst, group)
    valid = np.ones(used, bool)
    if window:
        qp = used - 1 if qpos is None else qpos
        valid &= (qp - np.arange(used)) < window
    return attend(q, k, v, np.broadcast_to(valid, (q.shape[0], used)))
