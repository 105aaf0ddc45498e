"""NF4 linear layers on B200 (drop-in for ``nova.quant``, src/nova/quant.py).

* ``NF4Linear(packed, absmax, code, shape, bias=None)`` -- same constructor and
  ``forward`` as the reference; forward runs ``nova_nf4_gemv``.
* ``extract_nf4(weight, quant_state)`` -- the reference's layout transform of a
  bitsandbytes ``Params4bit`` (duck-typed: only the attributes it reads).
* ``nf4_codebook()`` / ``quantize_nf4(w)`` / ``dequantize_nf4(...)`` -- the NF4
  levels and the blockwise quantizer for random-init models (bitsandbytes is
  not part of the reference tree).  The levels follow the published QLoRA
  construction (Dettmers et al. 2023): standard-normal quantiles at 8
  positive and 7 negative probabilities spaced from ``1 - (1/30 + 1/32)/2`` to
  1/2, plus an exact zero, normalised to [-1, 1].
"""

from __future__ import annotations

import torch
import torch.nn as nn

from . import _lib
from .kernels import build_nf4_lut, fused_nf4_linear

NF4_BLOCK = 64
_NF4_OFFSET = 0.9677083


def nf4_codebook() -> torch.Tensor:
    """The 16 NF4 levels, ascending, fp32 (computed in fp64 on the CPU)."""
    pos = torch.special.ndtri(torch.linspace(_NF4_OFFSET, 0.5, 9, dtype=torch.float64)[:-1])
    neg = -torch.special.ndtri(torch.linspace(_NF4_OFFSET, 0.5, 8, dtype=torch.float64)[:-1])
    v = torch.sort(torch.cat([pos, torch.zeros(1, dtype=torch.float64), neg])).values
    return (v / v.abs().max()).to(torch.float32)


def nf4_midpoints(code: torch.Tensor) -> torch.Tensor:
    c = code.to(torch.float32).cpu()
    return ((c[:-1] + c[1:]) * 0.5).to(torch.float32)


def quantize_nf4(w: torch.Tensor, code: torch.Tensor | None = None, absmax_dtype: torch.dtype = torch.float16):
    """Blockwise NF4 of fp16 ``w`` ``[N, K]`` on the GPU -> (packed uint8
    ``[N, K/2]``, absmax ``[K/64, N]``)."""
    _lib.require_cuda(w, names=("w",))
    if w.dtype != torch.float16 or w.dim() != 2:
        raise ValueError("w must be a 2-D float16 tensor")
    n, k = w.shape
    if k % NF4_BLOCK:
        raise ValueError(f"K={k} is not a multiple of {NF4_BLOCK}")
    code = nf4_codebook() if code is None else code
    mid = nf4_midpoints(code).to(w.device)
    w = w.contiguous()
    packed = torch.empty((n, k // 2), dtype=torch.uint8, device=w.device)
    absmax = torch.empty((k // NF4_BLOCK, n), dtype=absmax_dtype, device=w.device)
    _lib.call("nova_nf4_quantize", w.data_ptr(), n, k, mid.data_ptr(), packed.data_ptr(), absmax.data_ptr(),
              int(absmax_dtype == torch.float32), _lib.stream_of(w.device))
    return packed, absmax


def dequantize_nf4(packed: torch.Tensor, absmax: torch.Tensor, lut: torch.Tensor) -> torch.Tensor:
    """NF4 -> fp16 ``[N, K]`` (code16 * absmax rounded to fp16)."""
    _lib.require_cuda(packed, absmax, lut, names=("packed", "absmax", "lut"))
    n, k2 = packed.shape
    out = torch.empty((n, 2 * k2), dtype=torch.float16, device=packed.device)
    _lib.call("nova_nf4_dequant", packed.contiguous().data_ptr(), absmax.contiguous().data_ptr(),
              int(absmax.dtype == torch.float32), lut.contiguous().data_ptr(), out.data_ptr(), n, 2 * k2,
              _lib.stream_of(packed.device))
    return out


def extract_nf4(weight, quant_state):
    """bitsandbytes ``Params4bit`` -> ``(packed [N, K/2], absmax [K/64, N] fp32,
    code [16], (N, K))`` with double quantization undone (src/nova/quant.py:39-69)."""
    qs = quant_state
    n, k = int(qs.shape[0]), int(qs.shape[1])
    if k % NF4_BLOCK or k % 2:
        raise ValueError(f"K={k} must be a multiple of {NF4_BLOCK}")
    packed = weight.reshape(-1).view(torch.uint8)
    if packed.numel() != n * k // 2:
        raise ValueError(f"packed has {packed.numel()} bytes, expected {n * k // 2}")
    n_blocks = n * k // NF4_BLOCK
    if getattr(qs, "nested", False):
        s2 = qs.state2
        qa = qs.absmax.reshape(-1).long()
        a2 = s2.absmax.reshape(-1).repeat_interleave(int(s2.blocksize))[:n_blocks]
        absmax = s2.code.reshape(-1)[qa] * a2 + qs.offset
    else:
        absmax = qs.absmax.reshape(-1).float()
    packed = packed.reshape(n, k // 2).contiguous()
    absmax = absmax.reshape(n, k // NF4_BLOCK).t().contiguous()
    code = qs.code.reshape(-1).float().contiguous()
    if code.numel() != 16:
        raise ValueError(f"codebook has {code.numel()} entries, expected 16")
    return packed, absmax, code, (n, k)


class NF4Linear(nn.Module):
    """``nn.Linear``-compatible layer with NF4 weights; forward = one
    ``nova_nf4_gemv`` launch per 8 input rows (src/nova/quant.py:72-106)."""

    def __init__(self, packed: torch.Tensor, absmax: torch.Tensor, code: torch.Tensor, shape: tuple[int, int],
                 bias: torch.Tensor | None = None) -> None:
        super().__init__()
        self.out_features, self.in_features = int(shape[0]), int(shape[1])
        self.register_buffer("packed", packed, persistent=False)
        self.register_buffer("absmax", absmax, persistent=False)
        self.register_buffer("code", code, persistent=False)
        self.register_buffer("lut", build_nf4_lut(code).to(packed.device), persistent=False)
        if bias is None:
            self.bias = None
        else:
            self.bias = nn.Parameter(bias.detach().clone().to(torch.float16), requires_grad=False)

    @classmethod
    def from_bnb(cls, lin: nn.Module) -> "NF4Linear":
        packed, absmax, code, shape = extract_nf4(lin.weight.data, lin.weight.quant_state)
        bias = lin.bias.data if getattr(lin, "bias", None) is not None else None
        return cls(packed, absmax, code, shape, bias)

    @classmethod
    def from_float(cls, weight: torch.Tensor, bias: torch.Tensor | None = None,
                   absmax_dtype: torch.dtype = torch.float16) -> "NF4Linear":
        """Quantize an fp16 ``[N, K]`` CUDA weight with the NF4 quantizer."""
        code = nf4_codebook()
        packed, absmax = quantize_nf4(weight.to(torch.float16), code, absmax_dtype)
        return cls(packed, absmax, code.to(weight.device), tuple(weight.shape), bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return fused_nf4_linear(x, self.packed, self.absmax, self.lut, self.out_features, self.bias)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, nf4=sm_100a")


def convert_to_nf4(model: nn.Module, verbose: bool = False, skip: set[str] | None = None) -> int:
    """Replace every bitsandbytes-style 4-bit linear (a module whose ``weight``
    carries a ``quant_state``) with :class:`NF4Linear` (src/nova/quant.py:
    109-135).  Unlike the reference, ``lm_head4`` is converted too by default:
    the B200 GEMV is faster than the reference's fallback on that shape."""
    skip = set() if skip is None else skip
    n_done = 0
    for name, module in list(model.named_modules()):
        for child_name, child in list(module.named_children()):
            if child_name in skip:
                continue
            w = getattr(child, "weight", None)
            if w is not None and getattr(w, "quant_state", None) is not None:
                setattr(module, child_name, NF4Linear.from_bnb(child))
                n_done += 1
                if verbose:
                    print(f"  nf4: {name}.{child_name} -> {tuple(w.quant_state.shape)}")
    return n_done
