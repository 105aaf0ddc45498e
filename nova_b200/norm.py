"""``LeanRMSNorm`` on B200 (drop-in for ``nova.norm``, src/nova/norm.py).

The reference switches between an exact 16-op aten version and a Triton
kernel; here there is a single implementation, the ``nova_rmsnorm`` kernel,
which follows the exact version's operation order (fp32 variance, ``1/sqrt``,
round to fp16, then the fp16 weight multiply).  ``impl`` is accepted for
signature compatibility and ignored.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .kernels import fused_rms_norm


class LeanRMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6, impl: str = "exact", dtype: torch.dtype | None = None,
                 device: torch.device | str | None = None) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim, dtype=dtype or torch.float16, device=device))
        self.eps = float(eps)
        self.impl = impl

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return fused_rms_norm(x, self.weight, self.eps)

    @classmethod
    def from_hf(cls, hf_norm, impl: str = "exact") -> "LeanRMSNorm":
        src = hf_norm.weight.detach()
        dim = int(src.shape[0])
        eps = float(getattr(hf_norm, "variance_epsilon", getattr(hf_norm, "eps", 1e-6)))
        new = cls(dim, eps=eps, impl=impl, dtype=src.dtype, device=src.device)
        with torch.no_grad():
            new.weight.copy_(src)
        return new

    def extra_repr(self) -> str:
        return f"{tuple(self.weight.shape)}, eps={self.eps}"
