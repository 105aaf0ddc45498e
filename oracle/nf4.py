"""NF4 weights, restated in numpy (oracle; test infrastructure only).

Layout (reference src/nova/quant.py:39-69, src/nova/kernels.py:126-139):
  packed  uint8 ``[N, K/2]``, K-contiguous; byte j of a row holds element 2j in
          the HIGH nibble and element 2j+1 in the LOW nibble
  absmax  ``[K/64, N]`` (one scale per 64 consecutive K elements of a row),
          fp32 in the reference, fp16 in the B200-native format
  code    16-entry NF4 codebook; the kernels use it rounded to fp16
          (build_nf4_lut, src/nova/kernels.py:170-182)
  W[n,k] = code16[idx(n,k)] * absmax[k//64, n]

Codebook: bitsandbytes provides it at run time (src/nova/quant.py:67) and is
not part of the reference tree nor installed here.  ``nf4_codebook`` rebuilds
it from the published QLoRA construction (Dettmers et al. 2023, "QLoRA",
Sec. 3 / Appendix: normal-distribution quantiles, 8 positive + 7 negative
levels from ``offset = 1 - (1/30 + 1/32)/2``, plus an exact zero, normalised to
[-1, 1]).  The quantizer (``quantize_nf4``) is the bitsandbytes blockwise
scheme restated: absmax per 64-element block, then nearest codebook level by
midpoint thresholds, ties toward the lower level.
"""

from __future__ import annotations

import numpy as np
from scipy.special import ndtri

NF4_BLOCK = 64
NF4_OFFSET = 0.9677083


def nf4_codebook() -> np.ndarray:
    """16 NF4 levels, ascending, fp32 (QLoRA construction, see module doc)."""
    pos = ndtri(np.linspace(NF4_OFFSET, 0.5, 9)[:-1])        # 8 positive quantiles
    neg = -ndtri(np.linspace(NF4_OFFSET, 0.5, 8)[:-1])       # 7 negative quantiles
    v = np.sort(np.concatenate([pos, [0.0], neg]))
    v = v / np.abs(v).max()
    return v.astype(np.float32)


def nf4_midpoints(code: np.ndarray) -> np.ndarray:
    """fp32 decision thresholds between consecutive levels."""
    c = code.astype(np.float32)
    return ((c[:-1] + c[1:]) * np.float32(0.5)).astype(np.float32)


def build_nf4_lut(code: np.ndarray) -> np.ndarray:
    """256-entry int32 table, low 16 bits = fp16 bits of code[b >> 4], high 16
    bits = fp16 bits of code[b & 15] (src/nova/kernels.py:170-182)."""
    c16 = np.asarray(code, np.float32).astype(np.float16).view(np.uint16).astype(np.uint32)
    b = np.arange(256)
    val = c16[b >> 4] | (c16[b & 15] << 16)
    return val.astype(np.uint32).view(np.int32)


def quantize_nf4(w: np.ndarray, code: np.ndarray | None = None, absmax_dtype=np.float16):
    """Blockwise NF4 quantization of ``w`` ``[N, K]`` (fp16 or fp32).

    Returns (packed uint8 ``[N, K/2]``, absmax ``[K/64, N]`` in
    ``absmax_dtype``).  The level index is chosen from ``w / absmax`` with the
    fp32 absmax; the stored absmax is that value cast to ``absmax_dtype``.
    An all-zero block maps to the zero level.
    """
    code = nf4_codebook() if code is None else np.asarray(code, np.float32)
    n, k = w.shape
    if k % NF4_BLOCK:
        raise ValueError(f"K={k} is not a multiple of {NF4_BLOCK}")
    wf = np.asarray(w).astype(np.float32).reshape(n, k // NF4_BLOCK, NF4_BLOCK)
    am = np.abs(wf).max(axis=-1)                                   # [N, K/64] fp32
    safe = np.where(am > 0, am, np.float32(1.0)).astype(np.float32)
    v = (wf / safe[..., None]).astype(np.float32)
    idx = np.zeros(v.shape, np.uint8)
    for mid in nf4_midpoints(code):       # level = number of thresholds strictly below v (ties go low)
        idx += v > mid
    idx = idx.reshape(n, k)
    packed = ((idx[:, 0::2] << 4) | idx[:, 1::2]).astype(np.uint8)
    return packed, np.ascontiguousarray(am.T).astype(absmax_dtype)


def unpack_nf4(packed: np.ndarray) -> np.ndarray:
    """uint8 ``[N, K/2]`` -> level indices ``[N, K]`` (tests/test_nf4_linear.py:50-54)."""
    n, k2 = packed.shape
    idx = np.empty((n, 2 * k2), np.uint8)
    idx[:, 0::2] = packed >> 4
    idx[:, 1::2] = packed & 0x0F
    return idx


def dequantize_nf4(packed: np.ndarray, absmax: np.ndarray, code: np.ndarray, round_fp16: bool = False,
                   code_fp16: bool = True) -> np.ndarray:
    """``W = code[idx] * absmax`` in fp32 -> ``[N, K]``.

    ``code_fp16=True`` uses the codebook rounded to fp16, which is what the
    reference GEMV kernel multiplies by (its LUT, src/nova/kernels.py:170-182);
    ``code_fp16=False, round_fp16=True`` is exactly the reference test's
    dequant (tests/test_nf4_linear.py:46-57, fp32 code, product cast to fp16)."""
    c = np.asarray(code, np.float32)
    if code_fp16:
        c = c.astype(np.float16).astype(np.float32)
    vals = c[unpack_nf4(packed)]
    am = np.repeat(absmax.astype(np.float32).T, NF4_BLOCK, axis=1)
    w = (vals * am).astype(np.float32)
    return w.astype(np.float16) if round_fp16 else w


def nf4_linear(x: np.ndarray, packed: np.ndarray, absmax: np.ndarray, code: np.ndarray,
               bias: np.ndarray | None = None) -> np.ndarray:
    """``fused_nf4_linear`` semantics: fp32 accumulation of x * W, + bias, cast
    to fp16 (src/nova/kernels.py:187-240).  Returns fp32 before the cast so the
    caller can compare with a tolerance; use ``.astype(np.float16)`` for the
    fp16 output."""
    w = dequantize_nf4(packed, absmax, code)
    y = np.asarray(x, np.float32) @ w.T
    if bias is not None:
        y = y + np.asarray(bias, np.float32)
    return y.astype(np.float32)
