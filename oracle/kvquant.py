"""int8 KV quantization, restated in numpy (oracle; test infrastructure only).

Format ("int8t64", reference decision D38): asymmetric uint8 codes, one
(min, step) pair per (KV head, channel d, group of ``group`` consecutive
tokens), both stored as fp16.  Codes are computed from the fp32 min/step, the
dequant uses the fp16-stored ones.

    step = max((max - min) / 255, 1e-8)            fp32
    q    = clamp(round_half_even((x - min) / step), 0, 255)
    x'   = fp16( fp32(q) * fp32(step16) + fp32(min16) )

Reference: src/nova/kvquant.py:118-149 (quantize_int8, axis="token"),
:152-176 (dequantize_int8), src/nova/kvattn.py:716-743 (_quantize_ring).
"""

from __future__ import annotations

import numpy as np

BYTE_MAX = 255.0
STEP_FLOOR = np.float32(1e-8)


def _group_stats(xf: np.ndarray, axis: int):
    """fp32 min / step along ``axis`` (src/nova/kvquant.py:143-144)."""
    xmin = xf.min(axis=axis)
    xmax = xf.max(axis=axis)
    step = np.maximum((xmax - xmin) / np.float32(BYTE_MAX), STEP_FLOOR).astype(np.float32)
    return xmin.astype(np.float32), step


def _codes(xf: np.ndarray, xmin: np.ndarray, step: np.ndarray) -> np.ndarray:
    """clamp(round((x - min) / step), 0, 255) in fp32 (src/nova/kvquant.py:145)."""
    q = np.rint((xf - xmin) / step)          # np.rint = round half to even, like torch.round
    return np.clip(q, 0, 255).astype(np.uint8)


def quantize_int8_token(x: np.ndarray, group: int = 64):
    """Token-axis quantizer: ``x`` fp16 ``[..., n, dim]`` ->
    (codes uint8 ``[..., n, dim]``, mins fp16 ``[..., ceil(n/g), dim]``, steps fp16).

    A ragged last group is padded by repeating the last token
    (src/nova/kvquant.py:133-139); repeating an existing token leaves the
    group's min/max unchanged, so the pad is never materialised here.
    """
    x = np.asarray(x)
    if x.dtype != np.float16:
        raise ValueError("x must be float16")
    *lead, n, dim = x.shape
    g = int(group or n)
    ng = -(-n // g) if n else 0
    xf = x.astype(np.float32)
    codes = np.zeros(x.shape, np.uint8)
    mins = np.zeros((*lead, ng, dim), np.float16)
    steps = np.zeros((*lead, ng, dim), np.float16)
    for gi in range(ng):
        t0, t1 = gi * g, min(n, (gi + 1) * g)
        blk = xf[..., t0:t1, :]
        xmin, step = _group_stats(blk, axis=-2)
        codes[..., t0:t1, :] = _codes(blk, xmin[..., None, :], step[..., None, :])
        mins[..., gi, :] = xmin.astype(np.float16)
        steps[..., gi, :] = step.astype(np.float16)
    return codes, mins, steps


def dequantize_int8_token(q: np.ndarray, mins: np.ndarray, steps: np.ndarray, group: int = 64) -> np.ndarray:
    """Inverse of :func:`quantize_int8_token` -> fp16 (src/nova/kvquant.py:166-176).

    ``q*step`` is exact in fp32 (8-bit x 11-bit significands), so the fp32
    multiply-then-add equals a single fp32 rounding of ``q*step+min``.
    """
    *lead, n, dim = q.shape
    g = int(group or n)
    gi = np.arange(n) // g
    st = steps.astype(np.float32)[..., gi, :]
    mn = mins.astype(np.float32)[..., gi, :]
    return (q.astype(np.float32) * st + mn).astype(np.float16)


def quantize_ring(ring: np.ndarray):
    """Requantize one full 64-slot fp16 ring ``[..., 64, dim]`` into a group:
    -> (codes ``[..., 64, dim]``, min fp16 ``[..., dim]``, step fp16 ``[..., dim]``).
    Slot order equals in-group token order because a group starts at a multiple
    of 64 (src/nova/kvattn.py:716-743)."""
    rf = ring.astype(np.float32)
    xmin, step = _group_stats(rf, axis=-2)
    codes = _codes(rf, xmin[..., None, :], step[..., None, :])
    return codes, xmin.astype(np.float16), step.astype(np.float16)
