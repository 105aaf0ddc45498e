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
from .kernels import MAX_GEMV_M, build_nf4_lut, fused_nf4_linear, nf4_gemv, pack_native

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
    """``nn.Linear`` replacement holding NF4 weights (the reference's
    ``NF4Linear(packed, absmax, code, shape, bias)``, src/nova/quant.py:72-106).

    The reference-layout buffers ``packed`` / ``absmax`` / ``code`` / ``lut``
    are kept under the reference's names (callers and state dicts read them);
    with fp16 absmax the first forward on a device also packs the B200 unit
    stream (1088-byte 32 x 64 units, ``nova_nf4_pack_native``) and every later
    forward streams that, one ``nova_nf4_gemv`` launch per 8 input rows;
    leading dimensions of ``x`` are kept."""

    def __init__(self, packed: torch.Tensor, absmax: torch.Tensor, code: torch.Tensor, shape: tuple[int, int],
                 bias: torch.Tensor | None = None) -> None:
        super().__init__()
        n, k = (int(v) for v in shape)
        if tuple(packed.shape) != (n, k // 2) or tuple(absmax.shape) != (k // NF4_BLOCK, n):
            raise ValueError(f"packed {tuple(packed.shape)} / absmax {tuple(absmax.shape)} do not describe a "
                             f"[{n}, {k}] NF4 weight")
        self.out_features, self.in_features = n, k
        tensors = {"packed": packed, "absmax": absmax, "code": code,
                   "lut": build_nf4_lut(code).to(packed.device),
                   "bias": None if bias is None else bias.detach().to(torch.float16).clone()}
        for name, t in tensors.items():
            self.register_buffer(name, t, persistent=False)
        self._units: torch.Tensor | None = None

    @classmethod
    def from_bnb(cls, lin: nn.Module) -> "NF4Linear":
        """From a bitsandbytes ``Linear4bit`` (duck-typed: ``weight`` with a
        ``quant_state``, optional ``bias``)."""
        b = lin.bias.data if getattr(lin, "bias", None) is not None else None
        return cls(*extract_nf4(lin.weight.data, lin.weight.quant_state), bias=b)

    @classmethod
    def from_float(cls, weight: torch.Tensor, bias: torch.Tensor | None = None,
                   absmax_dtype: torch.dtype = torch.float16) -> "NF4Linear":
        """Quantize an fp16 ``[N, K]`` CUDA weight with the NF4 quantizer."""
        code = nf4_codebook()
        packed, absmax = quantize_nf4(weight.to(torch.float16), code, absmax_dtype)
        return cls(packed, absmax, code.to(weight.device), tuple(weight.shape), bias)

    def units(self) -> torch.Tensor:
        """The B200 unit stream of this weight, packed on first use.  Used when
        N is a multiple of 32 and absmax is fp16 (the units store fp16 absmax);
        otherwise forward streams the reference layout as it is."""
        if self._units is None or self._units.device != self.packed.device:
            self._units = pack_native(self.packed, self.absmax)
        return self._units

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.out_features % 32 or self.absmax.dtype != torch.float16:
            return fused_nf4_linear(x, self.packed, self.absmax, self.lut, self.out_features, self.bias)
        if x.shape[-1] != self.in_features:
            raise ValueError(f"x has {x.shape[-1]} features, the layer expects {self.in_features}")
        rows = x.reshape(-1, self.in_features)
        if not rows.is_contiguous() or rows.data_ptr() % 16:
            rows = rows.contiguous()
        y = torch.empty((rows.shape[0], self.out_features), dtype=torch.float16, device=x.device)
        units = self.units()
        for r0 in range(0, rows.shape[0], MAX_GEMV_M):
            nf4_gemv(rows[r0:r0 + MAX_GEMV_M], units, None, self.lut, y[r0:r0 + MAX_GEMV_M], bias=self.bias,
                     n=self.out_features)
        return y.view(*x.shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return f"{self.in_features} -> {self.out_features}, NF4 blocks of {NF4_BLOCK}, bias={self.bias is not None}"


def _quantized_linears(model: nn.Module):
    """(parent module, attribute name, child) for every child whose weight
    carries a bitsandbytes ``quant_state``, collected before any replacement."""
    found = []
    for parent in model.modules():
        for attr, child in parent.named_children():
            if getattr(getattr(child, "weight", None), "quant_state", None) is not None:
                found.append((parent, attr, child))
    return found


def convert_to_nf4(model: nn.Module, verbose: bool = False, skip: set[str] | None = None) -> int:
    """Swap every bitsandbytes-style 4-bit linear in ``model`` for
    :class:`NF4Linear` and return how many were swapped (the reference's
    ``convert_to_nf4``, src/nova/quant.py:109-135).  Children named in ``skip``
    stay as they are; unlike the reference, ``lm_head4`` is not skipped by
    default (the B200 GEMV is the fast path for that shape too)."""
    skip = set(skip or ())
    todo = [(parent, attr, child) for parent, attr, child in _quantized_linears(model) if attr not in skip]
    for parent, attr, child in todo:
        setattr(parent, attr, NF4Linear.from_bnb(child))
    if verbose:
        shapes = sorted({tuple(child.weight.quant_state.shape) for _, _, child in todo})
        print(f"nf4: {len(todo)} linears converted, weight shapes {shapes}")
    return len(todo)
