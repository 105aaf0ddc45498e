"""int8 KV quantization on the GPU, keeping the reference signatures of
``quantize_int8`` / ``dequantize_int8`` (src/nova/kvquant.py:118-176).

Only ``axis="token"`` (the "int8t64" KV format, reference decision D38) is on
the B200 path; the channel-axis, int4 and fp8 variants of the reference module
are rejected formats and are not provided here.
"""

from __future__ import annotations

import torch

from . import _lib

GROUP_K = 32  # reference default group (channel axis, src/nova/kvquant.py:48)
GROUP_T = 64  # token-axis group of the int8t64 KV format
BYTE_MAX = 255


def _check_axis(axis: str) -> None:
    if axis not in ("channel", "token"):
        raise ValueError(f"axis must be 'channel' or 'token', got {axis!r}")
    if axis != "token":
        raise ValueError("only axis='token' (the int8t64 KV format) is implemented on the B200 path")


def quantize_int8(x: torch.Tensor, group_size: int = GROUP_K, axis: str = "channel"):
    """Same defaults as the reference (``axis="channel"``, which is rejected
    here: pass ``group_size=64, axis="token"``).

    Asymmetric int8 along the token axis: ``x`` fp16 ``[..., n, dim]`` ->
    ``(codes uint8 [..., n, dim], mins fp16 [..., ceil(n/g), dim], steps fp16)``.
    Bit-identical to the reference quantizer (src/nova/kvquant.py:130-149)."""
    _check_axis(axis)
    _lib.require_cuda(x, names=("x",))
    if x.dtype != torch.float16:
        raise ValueError(f"x must be float16, got {x.dtype}")
    *lead, n, dim = x.shape
    g = int(group_size or n)
    x = x.contiguous()
    rows = 1
    for s in lead:
        rows *= int(s)
    ng = -(-n // g) if n else 0
    q = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    mins = torch.empty((*lead, ng, dim), dtype=torch.float16, device=x.device)
    steps = torch.empty_like(mins)
    if rows and n:
        _lib.call("nova_kv_quant_int8", x.data_ptr(), n * dim, q.data_ptr(), n * dim, mins.data_ptr(),
                  steps.data_ptr(), ng * dim, rows, n, dim, g, _lib.stream_of(x.device))
    return q, mins, steps


def dequantize_int8(q: torch.Tensor, mins: torch.Tensor, steps: torch.Tensor, group_size: int = GROUP_K,
                    axis: str = "channel", dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """Inverse of :func:`quantize_int8`: ``fp16(q*step + min)`` (src/nova/kvquant.py:166-176)."""
    _check_axis(axis)
    _lib.require_cuda(q, mins, steps, names=("q", "mins", "steps"))
    if dtype != torch.float16:
        raise ValueError("only float16 output is supported")
    *lead, n, dim = q.shape
    g = int(group_size or n)
    ng = -(-n // g) if n else 0
    if tuple(mins.shape) != (*lead, ng, dim) or mins.shape != steps.shape:
        raise ValueError(f"scale shape {tuple(mins.shape)} does not match codes {tuple(q.shape)}")
    q, mins, steps = q.contiguous(), mins.contiguous(), steps.contiguous()
    rows = 1
    for s in lead:
        rows *= int(s)
    out = torch.empty(q.shape, dtype=torch.float16, device=q.device)
    if rows and n:
        _lib.call("nova_kv_dequant_int8", q.data_ptr(), n * dim, mins.data_ptr(), steps.data_ptr(), ng * dim,
                  out.data_ptr(), n * dim, rows, n, dim, g, _lib.stream_of(q.device))
    return out


def bytes_per_token(num_slots: int = 36, num_kv_heads: int = 8, head_dim: int = 128, group: int = GROUP_T) -> dict:
    """Resident bytes per cached token (K+V codes + the fp16 min/step vectors
    amortised over the group), cf. src/nova/kvquant.py:232-289."""
    codes = 2 * num_slots * num_kv_heads * head_dim
    scales = 4 * num_slots * num_kv_heads * head_dim * 2 / group
    fp16 = 2 * num_slots * num_kv_heads * head_dim * 2
    return {"int8t64_kv": codes + scales, "fp16_kv": fp16, "ratio": fp16 / (codes + scales)}
