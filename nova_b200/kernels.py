"""RMSNorm and NF4 GEMV on B200, keeping the reference entry points of
``nova.kernels`` (src/nova/kernels.py): ``triton_available``,
``fused_rms_norm``, ``build_nf4_lut``, ``fused_nf4_linear``,
``nf4_launch_config`` / ``set_nf4_launch_config``.

The reference implements these as Triton kernels; here they call the sm_100a
kernels of ``libnova_b200.so`` (``nova_rmsnorm``, ``nova_nf4_gemv``).  There is
no fallback: CPU tensors or a missing library raise.
"""

from __future__ import annotations

import torch

from . import _lib

NF4_BLOCK = 64
NF4_BYTES = 32
MAX_GEMV_M = 8

_NF4_DEFAULTS: dict[str, int] = {"block_n": 64, "block_m": 1, "num_warps": 2, "num_stages": 2}
_nf4_launch: dict[str, int] = dict(_NF4_DEFAULTS)

_WORKSPACES: dict[tuple[str, int], torch.Tensor] = {}
_ARGMAX_SLOTS: dict[str, torch.Tensor] = {}


def triton_available() -> bool:
    """Name kept from the reference (src/nova/kernels.py:75-94): True when the
    B200 kernel library is loaded and a CUDA device is present."""
    return _lib.available()


def nf4_launch_config() -> dict[str, int]:
    """The reference's Triton launch knobs; accepted for compatibility, the
    B200 GEMV sizes its persistent grid from the SM count."""
    return dict(_nf4_launch)


def set_nf4_launch_config(**kwargs: int) -> dict[str, int]:
    for key, value in kwargs.items():
        if key not in _NF4_DEFAULTS:
            raise KeyError(f"unknown launch parameter: {key}")
        _nf4_launch[key] = int(value)
    return dict(_nf4_launch)


def fused_rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm over the last dimension, HF order (src/nova/kernels.py:97-115)."""
    _lib.require_cuda(x, weight, names=("x", "weight"))
    n = weight.shape[0]
    if x.shape[-1] != n:
        raise ValueError(f"last dim {x.shape[-1]} does not match weight length {n}")
    if x.dtype != torch.float16 or weight.dtype != torch.float16:
        raise ValueError("fused_rms_norm takes float16 x and weight")
    x = x.contiguous()
    weight = weight.contiguous()
    rows = x.numel() // n
    y = torch.empty_like(x)
    _lib.call("nova_rmsnorm", x.data_ptr(), n, None, 0, None, 0, weight.data_ptr(), y.data_ptr(), n, rows, n,
              float(eps), _lib.stream_of(x.device))
    return y


def residual_rms_norm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float):
    """``h = residual + x`` (fp16) and ``RMSNorm(h)`` in one launch -> (h, y)."""
    _lib.require_cuda(x, residual, weight, names=("x", "residual", "weight"))
    n = weight.shape[0]
    x, residual = x.contiguous(), residual.contiguous()
    rows = x.numel() // n
    h = torch.empty_like(x)
    y = torch.empty_like(x)
    _lib.call("nova_rmsnorm", x.data_ptr(), n, residual.data_ptr(), n, h.data_ptr(), n, weight.data_ptr(),
              y.data_ptr(), n, rows, n, float(eps), _lib.stream_of(x.device))
    return h, y


def build_nf4_lut(code: torch.Tensor) -> torch.Tensor:
    """256-entry int32 table: low 16 bits = fp16(code[a >> 4]), high 16 bits =
    fp16(code[a & 15]) (src/nova/kernels.py:170-182)."""
    c16 = code.detach().to(torch.float16).cpu()
    idx = torch.arange(256, dtype=torch.int64)
    even_bits = c16[idx >> 4].view(torch.int16).to(torch.int64) & 0xFFFF
    odd_bits = c16[idx & 15].view(torch.int16).to(torch.int64) & 0xFFFF
    val = (even_bits | (odd_bits << 16)) & 0xFFFFFFFF
    val = torch.where(val >= 2 ** 31, val - 2 ** 32, val)
    return val.to(torch.int32)


def gemv_workspace(device: torch.device, n: int) -> torch.Tensor:
    """Cached zeroed workspace for ``nova_nf4_gemv`` with N rows (eager path;
    calls on one stream may share it)."""
    out = _lib.ctypes.c_int64(0)
    _lib.call("nova_nf4_workspace_bytes", int(n), _lib.ctypes.byref(out))
    key = (str(device), int(out.value))
    ws = _WORKSPACES.get(key)
    if ws is None:
        ws = torch.zeros(int(out.value), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


def _pack(entry: str, packed: torch.Tensor, absmax: torch.Tensor) -> torch.Tensor:
    _lib.require_cuda(packed, absmax, names=("packed", "absmax"))
    n, k2 = packed.shape
    nbytes = _lib.ctypes.c_int64(0)
    _lib.call("nova_nf4_native_bytes", n, 2 * k2, _lib.ctypes.byref(nbytes))
    out = torch.empty(int(nbytes.value), dtype=torch.uint8, device=packed.device)
    _lib.call(entry, packed.contiguous().data_ptr(), absmax.contiguous().data_ptr(),
              int(absmax.dtype == torch.float32), out.data_ptr(), n, 2 * k2, _lib.stream_of(packed.device))
    return out


def pack_native(packed: torch.Tensor, absmax: torch.Tensor) -> torch.Tensor:
    """Reference NF4 layout (packed ``[N, K/2]``, absmax ``[K/64, N]``) -> the
    B200-native unit stream (uint8, 1088 bytes per 32-row x 64-k unit)."""
    return _pack("nova_nf4_pack_native", packed, absmax)


def pack_tc(packed: torch.Tensor, absmax: torch.Tensor) -> torch.Tensor:
    """Reference NF4 layout -> the unit stream of the tcgen05 GEMM
    (``nova_nf4_gemm`` with layout 2)."""
    return _pack("nova_nf4_pack_tc", packed, absmax)


def nf4_gemv(x: torch.Tensor, packed: torch.Tensor, absmax: torch.Tensor | None, lut: torch.Tensor,
             out: torch.Tensor, *,
             epilogue: int = _lib.NF4_PLAIN, bias: torch.Tensor | None = None, residual: torch.Tensor | None = None,
             norm_weight: torch.Tensor | None = None, eps: float = 1e-6, argmax: torch.Tensor | None = None,
             token_out: torch.Tensor | None = None, pos: torch.Tensor | None = None,
             embed: torch.Tensor | None = None, embed_out: torch.Tensor | None = None,
             workspace: torch.Tensor | None = None, n: int | None = None,
             add_slots: torch.Tensor | None = None, add_k: int = 0,
             resid_out: torch.Tensor | None = None, edge_out: torch.Tensor | None = None,
             edge_in: torch.Tensor | None = None, edge_k: int = 0, attn_part: int | None = None,
             attn_splits: int = 0, attn_heads: int = 0, add_heads: torch.Tensor | None = None) -> torch.Tensor:
    """Launch ``nova_nf4_gemv`` on 2-D views (x ``[M, K]``, out ``[M, N or N/2]``).

    Reference layout: ``packed`` uint8 ``[N, K/2]`` with ``absmax``
    ``[K/64, N]``.  Native layout: ``packed`` is the 1-D unit stream from
    :func:`pack_native`, ``absmax`` is None and ``n`` gives N.
    ``epilogue=NF4_SLOTS``: out is a :func:`slots_buffer` that receives each
    CTA's fp32 sums; a following launch with ``add_slots`` (that buffer) and
    ``add_k`` (the slot launch's K) adds them to its input x (fp16 residual
    add) before its norm prologue and stores the sum to ``resid_out``.
    ``edge_out`` (an :func:`edge_buffer`, with ``NF4_SILU_MUL`` at M = 1): the
    row groups split between CTAs are left there as fp32 sums instead of being
    reduced across CTAs, so ``out`` is incomplete until a following launch with
    ``edge_in`` (that buffer) and ``edge_k`` (this launch's K) completes them
    while it stages x (its K = this launch's N / 2).
    ``attn_part`` (a device address, :func:`nova_b200.kvattn.attn_partials`)
    with ``attn_splits`` / ``attn_heads``: ``NF4_F32`` over the head-major unit
    stream of o_proj (:func:`heads_major`), x merged from the decode
    attention's split partials, ``out`` the fp32 ``[attn_heads, N / attn_heads]``
    per-head sums; ``add_heads`` (those sums) is added to x like ``add_slots``."""
    m, k = x.shape
    native = absmax is None
    if native:
        if n is None or packed.dim() != 1:
            raise ValueError("the native layout needs the 1-D unit stream and n")
    else:
        n = packed.shape[0]
        if packed.shape[1] * 2 != k or absmax.shape != (k // NF4_BLOCK, n):
            raise ValueError(f"weight shapes packed {tuple(packed.shape)} / absmax {tuple(absmax.shape)} "
                             f"do not match K={k}, N={n}")
        if absmax.dtype not in (torch.float32, torch.float16):
            raise ValueError("absmax must be float32 or float16")
    for t, nm in ((x, "x"), (out, "out")):
        if t.stride(1) != 1:
            raise ValueError(f"{nm} must have a contiguous last dimension")
    ws = gemv_workspace(x.device, n) if workspace is None else workspace
    a = _lib.NF4Args()
    a.x, a.x_stride = x.data_ptr(), x.stride(0)
    a.norm_weight, a.eps = _lib.ptr(norm_weight), float(eps)
    a.packed = packed.data_ptr()
    a.absmax = None if native else absmax.data_ptr()
    a.absmax_fp32 = 0 if native else int(absmax.dtype == torch.float32)
    a.layout = 1 if native else 0
    a.lut = lut.data_ptr()
    a.bias = _lib.ptr(bias)
    a.residual, a.res_stride = (_lib.ptr(residual), residual.stride(0) if residual is not None else 0)
    a.out, a.out_stride = out.data_ptr(), out.stride(0)
    a.argmax, a.token_out, a.pos = _lib.ptr(argmax), _lib.ptr(token_out), _lib.ptr(pos)
    a.embed = _lib.ptr(embed)
    a.embed_out = _lib.ptr(embed_out)
    a.embed_out_stride = embed_out.stride(0) if embed_out is not None else 0
    a.embed_dim = embed.shape[1] if embed is not None else 0
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    a.m, a.n, a.k, a.epilogue = m, n, k, int(epilogue)
    if add_slots is not None:
        a.add_slots, a.add_k, a.resid_out = add_slots.data_ptr(), int(add_k), _lib.ptr(resid_out)
    a.edge_out = _lib.ptr(edge_out)
    if attn_part is not None:
        a.attn_part, a.attn_splits, a.attn_heads = int(attn_part), int(attn_splits), int(attn_heads)
    if add_heads is not None:
        a.add_heads, a.add_nheads, a.resid_out = add_heads.data_ptr(), int(add_heads.shape[0]), _lib.ptr(resid_out)
    if edge_in is not None:
        a.edge_in, a.edge_k = edge_in.data_ptr(), int(edge_k)
    _lib.check(_lib.lib().nova_nf4_gemv(_lib.ctypes.byref(a), _lib.stream_of(x.device)), "nova_nf4_gemv")
    return out


def slots_buffer(device: torch.device) -> torch.Tensor:
    """fp32 ``[SMs * 4 * 8, 32]`` buffer for ``NF4_SLOTS`` launches (per
    CTA the sums of the up to four row groups it may touch, up to 8 batch
    rows)."""
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    return torch.zeros(sms * 4 * 8, 32, dtype=torch.float32, device=device)


def heads_major(units: torch.Tensor, n: int, k: int, heads: int) -> torch.Tensor:
    """The native unit stream of an [n, k] matrix reordered head-major: the
    k columns split into ``heads`` blocks, block h's row groups first (the
    layout ``attn_part`` launches read)."""
    rg, kb = n // 32, k // 64
    return units.view(rg, heads, kb // heads, -1).permute(1, 0, 2, 3).contiguous().view(-1)


def edge_buffer(device: torch.device) -> torch.Tensor:
    """fp32 ``[SMs * 2, 32]`` buffer for ``edge_out`` / ``edge_in`` (per CTA
    the sums of its first and last row group, batch row 0)."""
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    return torch.zeros(sms * 2, 32, dtype=torch.float32, device=device)


def gemm_workspace(device: torch.device, n: int, k: int) -> torch.Tensor:
    """Cached zeroed workspace for ``nova_nf4_gemm`` with N rows and K columns."""
    out = _lib.ctypes.c_int64(0)
    _lib.call("nova_nf4_gemm_workspace_bytes", int(n), int(k), _lib.ctypes.byref(out))
    key = (str(device), -int(out.value))
    ws = _WORKSPACES.get(key)
    if ws is None:
        ws = torch.zeros(int(out.value), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


def nf4_gemm(x: torch.Tensor, units: torch.Tensor, lut: torch.Tensor, out: torch.Tensor, *, n: int,
             epilogue: int = _lib.NF4_PLAIN, residual: torch.Tensor | None = None,
             argmax: torch.Tensor | None = None, token_out: torch.Tensor | None = None,
             pos: torch.Tensor | None = None, embed: torch.Tensor | None = None,
             embed_out: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """``nova_nf4_gemm``: x ``[M, K]`` against the tcgen05 unit stream
    (:func:`pack_tc`) of an ``[n, K]`` NF4 weight, on the tensor cores; out
    ``[M, n]`` (``[M, n/2]`` for SiLU*up).  M <= 64: batched decode (every
    epilogue, the step finalize); M > 64: the wide prefill kernel (no argmax)."""
    m, k = x.shape
    if x.stride(1) != 1 or out.stride(1) != 1:
        raise ValueError("x/out must have a contiguous last dimension")
    ws = gemm_workspace(x.device, n, k) if workspace is None else workspace
    a = _lib.NF4Args()
    a.x, a.x_stride = x.data_ptr(), x.stride(0)
    a.norm_weight, a.eps = None, 0.0
    a.packed, a.absmax, a.absmax_fp32, a.layout = units.data_ptr(), None, 0, 2
    a.lut, a.bias = lut.data_ptr(), None
    a.residual, a.res_stride = (_lib.ptr(residual), residual.stride(0) if residual is not None else 0)
    a.out, a.out_stride = out.data_ptr(), out.stride(0)
    a.argmax, a.token_out, a.pos = _lib.ptr(argmax), _lib.ptr(token_out), _lib.ptr(pos)
    a.embed, a.embed_out = _lib.ptr(embed), _lib.ptr(embed_out)
    a.embed_out_stride = embed_out.stride(0) if embed_out is not None else 0
    a.embed_dim = embed.shape[1] if embed is not None else 0
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    a.m, a.n, a.k, a.epilogue = m, n, k, int(epilogue)
    _lib.check(_lib.lib().nova_nf4_gemm(_lib.ctypes.byref(a), _lib.stream_of(x.device)), "nova_nf4_gemm")
    return out


def fused_nf4_linear(x: torch.Tensor, packed: torch.Tensor, absmax: torch.Tensor, lut: torch.Tensor,
                     out_features: int, bias: torch.Tensor | None = None, **launch_overrides: int) -> torch.Tensor:
    """NF4 linear ``x @ dequant(packed, absmax, code).T + bias``
    (src/nova/kernels.py:243-289).  ``x`` fp16 ``[..., K]``; packed uint8
    ``[N, K/2]``; absmax ``[K/64, N]`` fp32 (reference) or fp16 (native).
    Rows are processed 8 at a time by the GEMV kernel."""
    _lib.require_cuda(x, packed, absmax, lut, names=("x", "packed", "absmax", "lut"))
    k = x.shape[-1]
    k2 = packed.shape[-1]
    n_blocks = absmax.shape[0]
    if k2 * 2 != k:
        raise ValueError(f"packed last dim {k2} does not match K={k} (should be K//2)")
    if n_blocks * NF4_BLOCK != k:
        raise ValueError(f"absmax rows {n_blocks} do not match K={k} (should be K//64)")
    if packed.shape[0] != out_features or absmax.shape[1] != out_features:
        raise ValueError(f"weight shapes do not match out_features={out_features}")
    if x.dtype != torch.float16:
        raise ValueError("x must be float16")
    n = out_features
    orig = x.shape
    x2 = x.reshape(-1, k)
    if not x2.is_contiguous() or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    m = x2.shape[0]
    out = torch.empty((m, n), device=x.device, dtype=torch.float16)
    packed = packed.contiguous()
    absmax = absmax.contiguous()
    lut = lut.contiguous()
    for r in range(0, m, MAX_GEMV_M):
        nf4_gemv(x2[r:r + MAX_GEMV_M], packed, absmax, lut, out[r:r + MAX_GEMV_M], bias=bias)
    return out.view(*orig[:-1], n)
