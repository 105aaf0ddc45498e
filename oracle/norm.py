"""RMSNorm and RoPE, restated in numpy (oracle; test infrastructure only)."""

from __future__ import annotations

import numpy as np


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """HF-order RMSNorm (src/nova/norm.py:37-42, kernel variant
    src/nova/kernels.py:51-69): fp32 variance, ``h = fp16(x * rsqrt(var+eps))``,
    then ``fp16(w * h)``.  ``rsqrt`` is ``1/sqrt`` with two IEEE roundings."""
    xf = np.asarray(x).astype(np.float32)
    var = np.mean(xf * xf, axis=-1, keepdims=True, dtype=np.float32)
    r = (np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)
    h = (xf * r).astype(np.float16)
    return (np.asarray(w).astype(np.float32) * h.astype(np.float32)).astype(np.float16)


def rope_inv_freq(head_dim: int = 128, theta: float = 5_000_000.0) -> np.ndarray:
    """``1 / theta**(arange(0, d, 2)/d)`` in fp32, the HF default RoPE init
    (transformers Qwen3VLTextRotaryEmbedding.compute_default_rope_parameters).
    The power is evaluated the way torch's CPU ``float ** tensor`` does:
    ``pow`` in fp32 of an fp32 exponent."""
    import torch

    e = torch.arange(0, head_dim, 2, dtype=torch.int64).to(dtype=torch.float) / head_dim
    return (1.0 / (theta ** e)).numpy().astype(np.float32)


def rope_cos_sin(positions, head_dim: int = 128, theta: float = 5_000_000.0):
    """fp16 cos/sin ``[len(positions), head_dim]`` exactly as the HF rotary does
    for text tokens (all three M-RoPE rows equal, so the interleave is a no-op):
    fp32 ``freqs = pos * inv_freq``, ``emb = cat(freqs, freqs)``, fp32
    cos/sin, cast to fp16.  Evaluated with torch on the CPU so the values are
    the reference's own (src/nova/model.py:144, src/nova/layers.py:124)."""
    import torch

    inv = torch.from_numpy(rope_inv_freq(head_dim, theta))
    pos = torch.as_tensor(np.asarray(positions), dtype=torch.float32)
    freqs = pos[:, None] * inv[None, :]
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(torch.float16).numpy(), emb.sin().to(torch.float16).numpy()


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """``(x*cos) + (rotate_half(x)*sin)`` with fp16 rounding after every op
    (src/nova/layers.py:24-36).  x fp16 ``[..., D]``; cos/sin fp16 ``[D]`` or
    broadcastable."""
    x = np.asarray(x, np.float16)
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    a = (x.astype(np.float32) * cos.astype(np.float32)).astype(np.float16)
    b = (rot.astype(np.float32) * sin.astype(np.float32)).astype(np.float16)
    return (a.astype(np.float32) + b.astype(np.float32)).astype(np.float16)


def silu_mul(gate16: np.ndarray, up16: np.ndarray) -> np.ndarray:
    """``act_fn(gate) * up`` on fp16 tensors (src/nova/layers.py:174): SiLU in
    fp32 rounded to fp16, then an fp16 multiply."""
    g = gate16.astype(np.float32)
    s = (g / (np.float32(1.0) + np.exp(-g))).astype(np.float16)
    return (s.astype(np.float32) * up16.astype(np.float32)).astype(np.float16)
