"""int8 KV decode attention and the streaming int8 KV cache on B200.

Drop-in for ``nova.kvattn`` (captain-wangrun-cn/Nova, src/nova/kvattn.py):
same entry points and argument meaning -- ``int8_attn_decode``,
``pack_int8_kv``, ``tail_attend``, ``KVInt8Cache`` -- backed by the sm_100a
kernels in ``libnova_b200.so``:

* ``nova_attn_decode_int8``: one kernel for the int8 prefix, the fp16 tail ring
  and their log-sum-exp merge (the reference runs a Triton partial kernel, a
  Triton combine kernel and ~15 aten ops for the tail and the merge);
* ``nova_kv_append_int8``: ring write + requantization of a completed group +
  device-scalar update in one launch (the reference runs ~20 aten ops);
* ``nova_kv_quant_int8``: the prefill quantizer.

Lengths stay in 1-element int64 device tensors, so one captured CUDA graph
stays valid while the context grows (src/nova/kvattn.py:125-141).

Extensions over the reference: batch > 1 (lengths shared by the batch) and a
sliding ``window`` on both the int8 prefix and the ring.  Limits of the B200
kernels: head_dim 128, group 64, at most 4 query heads per KV head.
"""

from __future__ import annotations

from typing import Any

import torch

from . import _lib
from .kvquant import quantize_int8

GROUP_T = 64
CHUNK = 512
PAD_M = 16       # kept for API compatibility with the reference module
HEAD_DIM = 128
MAX_GQ = 4


def pick_chunk(max_len: int, batch: int, kv_heads: int, q_heads: int, sms: int = 148) -> int:
    """Split size (tokens, a multiple of 64, at least 256) for the decode
    attention at capacity ``max_len``: about two CTAs per SM (splits of at
    most 8192 tokens at large batch), and at most
    ``73728 // (q_heads/kv_heads * 528) - 1`` splits per head, so the last CTA
    of a head merges all split partials from one shared-memory copy."""
    gq = max(1, q_heads // kv_heads)
    per_head = max(1, (2 * sms) // (batch * kv_heads), -(-max_len // 8192))   # and splits of at most 8192 tokens
    per_head = min(per_head, 73728 // (gq * 528) - 1)
    chunk = -(-max_len // per_head)
    return max(GROUP_T * 4, -(-chunk // GROUP_T) * GROUP_T)


def attn_workspace_bytes(batch: int, q_heads: int, kv_heads: int, n_splits: int, has_tail: bool) -> int:
    out = _lib.ctypes.c_int64(0)
    _lib.call("nova_attn_workspace_bytes", int(batch), int(q_heads), int(kv_heads), int(n_splits),
              int(bool(has_tail)), _lib.ctypes.byref(out))
    return int(out.value)


def new_workspace(batch: int, q_heads: int, kv_heads: int, n_splits: int, has_tail: bool,
                  device: torch.device | str = "cuda") -> torch.Tensor:
    """Zeroed workspace for ``nova_attn_decode_int8`` (reusable across calls
    and graph replays; the kernel leaves its counters at zero)."""
    n = attn_workspace_bytes(batch, q_heads, kv_heads, n_splits, has_tail)
    return torch.zeros(n, dtype=torch.uint8, device=device)


# Persistent per-device buffers for the eager path (graph capture must not
# allocate; src/nova/kvattn.py:265-278).  Not thread-safe, like the reference.
_SCALAR_BUFFERS: dict[str, tuple[torch.Tensor, torch.Tensor]] = {}
_WORKSPACES: dict[tuple[str, int], torch.Tensor] = {}


def _scalar_buffers(device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    key = str(device)
    buf = _SCALAR_BUFFERS.get(key)
    if buf is None:
        buf = (torch.zeros(1, dtype=torch.int64, device=device), torch.zeros(1, dtype=torch.int64, device=device))
        _SCALAR_BUFFERS[key] = buf
    return buf


def _cached_workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    key = (str(device), int(nbytes))
    ws = _WORKSPACES.get(key)
    if ws is None:
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


def _check(x: torch.Tensor, name: str, dtype: torch.dtype) -> None:
    if not x.is_cuda:
        raise ValueError(f"{name} must be on CUDA")
    if x.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {x.dtype}")
    if not x.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def attn_partials(workspace: torch.Tensor, batch: int, kv_heads: int) -> int:
    """Device address of the split partials inside an attention workspace
    (``defer_merge``): byte 256 + align_up(batch * kv_heads * 4, 256)."""
    return workspace.data_ptr() + 256 + (batch * kv_heads * 4 + 255) // 256 * 256


def launch_attention(q: torch.Tensor, kv: tuple | None, tail: tuple | None, out: torch.Tensor,
                     lse: torch.Tensor | None, qlen_t: torch.Tensor, pg_t: torch.Tensor,
                     written_t: torch.Tensor | None, first_t: torch.Tensor | None, workspace: torch.Tensor,
                     *, max_len: int, n_splits: int, chunk: int = CHUNK, window: int = 0,
                     qk: "_lib.QKArgs | None" = None, defer_merge: bool = False) -> None:
    """Thin launcher for ``nova_attn_decode_int8``; with ``qk`` (the
    arguments of ``nova_qk_norm_rope_append`` for the same ring and cache) the
    q/k norm + RoPE + ring append runs in the same launch
    (``nova_qk_append_attn_int8``): ``q`` is then not read, and neither are
    ``qlen_t`` / ``pg_t`` / ``written_t``.

    q: fp16 ``[B, Hq, D]`` view (strides are passed through; last dim
    contiguous); kv: ``(kq, kmn, kst, vq, vmn, vst)`` contiguous
    ``[B, Hkv, max_len, D]`` / ``[B, Hkv, G, D]`` or None (tail only); tail:
    ``(tail_k, tail_v)`` fp16 ``[B, Hkv, 64, D]`` or None; out: fp16
    ``[B, Hq, D]`` view; lse: fp32 ``[B, Hq]`` or None.
    """
    B, Hq, D = q.shape
    if q.stride(2) != 1 or out.stride(2) != 1:
        raise ValueError("q/out must have a contiguous last dimension")
    if kv is not None:
        kq, kmn, kst, vq, vmn, vst = kv
        Hkv = kq.shape[1]
        groups = kmn.shape[2]
    else:
        kq = kmn = kst = vq = vmn = vst = None
        Hkv = tail[0].shape[1]
        groups = -(-max_len // GROUP_T)
    a = _lib.AttnArgs()
    a.q, a.q_b_stride, a.q_h_stride = q.data_ptr(), q.stride(0), q.stride(1)
    a.kq, a.vq, a.kmn, a.kst, a.vmn, a.vst = (_lib.ptr(t) for t in (kq, vq, kmn, kst, vmn, vst))
    a.tail_k, a.tail_v = (_lib.ptr(tail[0]), _lib.ptr(tail[1])) if tail is not None else (None, None)
    a.out, a.o_b_stride, a.o_h_stride = out.data_ptr(), out.stride(0), out.stride(1)
    a.lse, a.lse_b_stride = (lse.data_ptr(), lse.stride(0)) if lse is not None else (None, 0)
    a.qlen, a.pg = qlen_t.data_ptr(), pg_t.data_ptr()
    a.written = _lib.ptr(written_t)
    a.first = _lib.ptr(first_t)
    a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    a.batch, a.q_heads, a.kv_heads = B, Hq, Hkv
    a.max_len, a.groups, a.head_dim, a.group = int(max_len), int(groups), D, GROUP_T
    a.chunk, a.n_splits, a.window = int(chunk), int(n_splits), int(window)
    a.defer_merge = int(bool(defer_merge))   # with qk: the split partials stay for the o_proj launch
    if qk is not None:
        _lib.check(_lib.lib().nova_qk_append_attn_int8(_lib.ctypes.byref(qk), _lib.ctypes.byref(a),
                                                       _lib.stream_of(q.device)), "nova_qk_append_attn_int8")
        return
    _lib.check(_lib.lib().nova_attn_decode_int8(_lib.ctypes.byref(a), _lib.stream_of(q.device)),
               "nova_attn_decode_int8")


def int8_attn_decode(
    q: torch.Tensor,
    kq: torch.Tensor,
    kmn: torch.Tensor,
    kst: torch.Tensor,
    vq: torch.Tensor,
    vmn: torch.Tensor,
    vst: torch.Tensor,
    *,
    used: int | None = None,
    group: int = GROUP_T,
    chunk: int = CHUNK,
    num_warps: int = 8,
    num_stages: int = 2,
    scratch: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    lse_out: torch.Tensor | None = None,
    prefix_groups: int | torch.Tensor = -1,
    used_t: torch.Tensor | None = None,
    prefix_groups_t: torch.Tensor | None = None,
    n_splits: int | None = None,
    window: int = 0,
) -> torch.Tensor:
    """One decode step of fused int8-KV attention (src/nova/kvattn.py:281-427).

    - ``q``: fp16 ``[B, H_q, 1, D]`` (RoPE applied); ``kq``/``vq``: uint8
      ``[B, H_kv, L, D]``; ``kmn``/``kst``/``vmn``/``vst``: fp16
      ``[B, H_kv, ceil(L/group), D]``.  The reference accepts B == 1 only;
      here B >= 1 (all rows share the lengths).
    - ``used``: valid prefix length (default L); ``used_t``/``prefix_groups_t``:
      the device-scalar form for CUDA graphs (then ``n_splits`` fixes the grid).
    - ``scratch``: a workspace from :func:`new_workspace` (uint8, zeroed once);
      required under graph capture, like the reference's pre-allocated scratch.
    - ``lse_out``: fp32 ``[B, H_q]`` log-sum-exp of the scaled scores.
    - ``window``: keep positions ``p > used-1-window`` (0 = all).
    - ``num_warps``/``num_stages`` are Triton launch knobs of the reference and
      are accepted and ignored.
    Returns fp16 ``[B, H_q, 1, D]``.
    """
    if q.dim() != 4 or q.shape[2] != 1:
        raise ValueError(f"decode attention takes q of shape [B, H_q, 1, D], got {tuple(q.shape)}")
    _check(q, "q", torch.float16)
    for name, t, dt in (("kq", kq, torch.uint8), ("vq", vq, torch.uint8), ("kmn", kmn, torch.float16),
                        ("kst", kst, torch.float16), ("vmn", vmn, torch.float16), ("vst", vst, torch.float16)):
        _check(t, name, dt)
    b, hq, _, d = q.shape
    h_kv, length = kq.shape[1], kq.shape[2]
    if kq.shape != vq.shape:
        raise ValueError(f"kq {tuple(kq.shape)} and vq {tuple(vq.shape)} differ")
    if kmn.shape != kst.shape or kmn.shape != vmn.shape or kmn.shape != vst.shape:
        raise ValueError("the four scale tensors must have the same shape")
    if kq.shape[0] != b or kmn.shape[0] != b or kmn.shape[1] != h_kv or kmn.shape[3] != d or kq.shape[3] != d:
        raise ValueError(f"scale shape {tuple(kmn.shape)} does not match KV {tuple(kq.shape)} / q {tuple(q.shape)}")
    if hq % h_kv:
        raise ValueError(f"q heads {hq} not divisible by KV heads {h_kv}")
    if hq // h_kv > MAX_GQ:
        raise ValueError(f"{hq // h_kv} query heads per KV head; the B200 kernel supports at most {MAX_GQ}")
    if d != HEAD_DIM:
        raise ValueError(f"head_dim must be {HEAD_DIM}, got {d}")
    if group != GROUP_T:
        raise ValueError(f"group must be {GROUP_T}, got {group}")
    if chunk % group:
        raise ValueError(f"chunk {chunk} must be a multiple of group {group}")
    if kmn.shape[2] != -(-length // group):
        raise ValueError(f"scale groups {kmn.shape[2]} != ceil(L/group) = {-(-length // group)}")
    if isinstance(scratch, (tuple, list)):
        raise ValueError("scratch must be a workspace tensor from nova_b200.kvattn.new_workspace()")

    used = length if used is None else int(used)
    if not 0 <= used <= length:
        raise ValueError(f"used={used} outside [0, {length}]")
    if not isinstance(prefix_groups, torch.Tensor):
        prefix_groups = int(prefix_groups)
        if prefix_groups < 0:
            prefix_groups = -(-used // group)
        elif prefix_groups > kmn.shape[2]:
            raise ValueError(f"prefix_groups={prefix_groups} exceeds the {kmn.shape[2]} scale groups")

    used_is_device = used_t is not None
    if used_is_device:
        for name, t in (("used_t", used_t), ("prefix_groups_t", prefix_groups_t)):
            if t is None or tuple(t.shape) != (1,) or t.dtype != torch.int64 or not t.is_cuda:
                raise ValueError(f"{name} must be a CUDA int64 tensor of shape [1]")
    else:
        used_t, prefix_groups_t = _scalar_buffers(q.device)
        used_t.fill_(used)
        prefix_groups_t.fill_(int(prefix_groups))
    if out is None:
        out = torch.empty((b, hq, 1, d), dtype=torch.float16, device=q.device)
    elif tuple(out.shape) != (b, hq, 1, d) or out.dtype != torch.float16 or not out.is_cuda:
        raise ValueError(f"out has the wrong shape/dtype: {tuple(out.shape)} {out.dtype}")
    if lse_out is not None and (tuple(lse_out.shape) != (b, hq) or lse_out.dtype != torch.float32
                                or not lse_out.is_cuda):
        raise ValueError(f"lse_out has the wrong shape/dtype: {tuple(lse_out.shape)} {lse_out.dtype}")
    if not used_is_device and used == 0:
        out.zero_()
        if lse_out is not None:
            lse_out.fill_(float("-inf"))
        return out

    if n_splits is None:
        span = length if used_is_device else used
        if window:   # the kernel lays the splits over the window when they cover it
            span = min(span, window + group)
        n_splits = -(-span // chunk)
    n_splits = int(n_splits)
    if n_splits < 1:
        raise ValueError(f"n_splits={n_splits} must be >= 1")
    need = attn_workspace_bytes(b, hq, h_kv, n_splits, False)
    if scratch is None:
        scratch = _cached_workspace(q.device, need)
    elif scratch.dtype != torch.uint8 or not scratch.is_cuda or scratch.numel() < need:
        raise ValueError(f"scratch must be a CUDA uint8 workspace of >= {need} bytes")
    launch_attention(q[:, :, 0], (kq, kmn, kst, vq, vmn, vst), None, out[:, :, 0], lse_out, used_t,
                     prefix_groups_t, None, None, scratch, max_len=length, n_splits=n_splits, chunk=chunk,
                     window=window)
    return out


def prefill_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, prefix: int,
                      int8: tuple | None = None, int8_len: int = 0, window: int = 0,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """Causal attention of a prefill chunk (``nova_attn_prefill_int8``).

    q fp16 ``[B, Hq, n, D]``: the chunk's queries at positions [prefix,
    prefix + n), RoPE applied.  k / v fp16 ``[B, Hkv, rows, D]``: positions
    [int8_len, prefix + n).  ``int8`` = (kq, kmn, kst, vq, vmn, vst) of one
    layer's cache holding positions [0, int8_len) (int8_len a multiple of 64).
    Returns fp16 ``[B, n, Hq * D]`` (row = token: the o_proj input)."""
    b, hq, n, d = q.shape
    hkv = k.shape[1]
    for name, t in (("q", q), ("k", k), ("v", v)):
        _check_any(t, name, torch.float16)
    if d != HEAD_DIM or k.shape[3] != d or v.shape != k.shape or k.shape[0] != b or hq % hkv:
        raise ValueError(f"shapes q {tuple(q.shape)} k {tuple(k.shape)} v {tuple(v.shape)} do not match")
    if k.shape[2] < prefix + n - int8_len:
        raise ValueError(f"k holds {k.shape[2]} rows, positions [{int8_len}, {prefix + n}) are needed")
    if q.stride(3) != 1 or k.stride(3) != 1 or v.stride()[:3] != k.stride()[:3] or v.stride(3) != 1:
        raise ValueError("q / k / v need a contiguous last dimension (and k, v the same strides)")
    if out is None:
        out = torch.empty(b, n, hq * d, dtype=torch.float16, device=q.device)
    a = _lib.PrefillAttnArgs()
    a.q, a.q_b_stride, a.q_h_stride, a.q_t_stride = q.data_ptr(), q.stride(0), q.stride(1), q.stride(2)
    a.k, a.v = k.data_ptr(), v.data_ptr()
    a.kv_b_stride, a.kv_h_stride, a.kv_t_stride = k.stride(0), k.stride(1), k.stride(2)
    a.max_len, a.groups = 0, 0
    if int8 is not None and int8_len:
        kq, kmn, kst, vq, vmn, vst = int8
        a.kq, a.vq = kq.data_ptr(), vq.data_ptr()
        a.kmn, a.kst, a.vmn, a.vst = kmn.data_ptr(), kst.data_ptr(), vmn.data_ptr(), vst.data_ptr()
        a.max_len, a.groups = kq.shape[2], kmn.shape[2]
    a.out, a.o_b_stride, a.o_t_stride = out.data_ptr(), out.stride(0), out.stride(1)
    a.batch, a.q_heads, a.kv_heads, a.head_dim = b, hq, hkv, d
    a.n, a.prefix, a.int8_len, a.window = n, int(prefix), int(int8_len), int(window)
    _lib.check(_lib.lib().nova_attn_prefill_int8(_lib.ctypes.byref(a), _lib.stream_of(q.device)),
               "nova_attn_prefill_int8")
    return out


def _check_any(x: torch.Tensor, name: str, dtype: torch.dtype) -> None:
    if not x.is_cuda:
        raise ValueError(f"{name} must be on CUDA")
    if x.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {x.dtype}")


def pack_int8_kv(k: torch.Tensor, v: torch.Tensor, group: int = GROUP_T):
    """fp16 K/V ``[B, H, L, D]`` -> the fused kernel's layout, with the same
    quantizer the cache uses (src/nova/kvattn.py:430-441)."""
    kq, kmn, kst = quantize_int8(k, group, "token")
    vq, vmn, vst = quantize_int8(v, group, "token")
    return kq, kmn, kst, vq, vmn, vst


def tail_attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, written: torch.Tensor, qlen: torch.Tensor,
                first: torch.Tensor | None = None):
    """Attention over the fp16 ring alone, with its log-sum-exp
    (src/nova/kvattn.py:447-482).  The reference takes a boolean slot mask; here
    the validity comes from the device scalars that produce that mask
    (``written``, ``qlen``, ``first``; src/nova/kvattn.py:819-833).
    q fp16 ``[B, H_q, 1, D]``, k/v fp16 ``[B, H_kv, 64, D]``.
    Returns ``(out [B, H_q, 1, D] fp16, lse [B, H_q] fp32)``."""
    _check(q, "q", torch.float16)
    _check(k, "k", torch.float16)
    _check(v, "v", torch.float16)
    b, hq, _, d = q.shape
    out = torch.empty_like(q)
    lse = torch.empty((b, hq), dtype=torch.float32, device=q.device)
    ws = _cached_workspace(q.device, attn_workspace_bytes(b, hq, k.shape[1], 0, True))
    launch_attention(q[:, :, 0], None, (k, v), out[:, :, 0], lse, qlen, torch.zeros_like(qlen), written, first,
                     ws, max_len=GROUP_T, n_splits=0)
    return out, lse


class _Staging:
    """fp16 prefill staging area sized to the prompt (the reference uses
    ``StaticKVCache``, src/nova/cache.py:117-175, for the same purpose)."""

    def __init__(self, num_slots, num_kv_heads, head_dim, max_len, batch, dtype, device) -> None:
        shape = (batch, num_kv_heads, max_len, head_dim)
        self.key_cache = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(num_slots)]
        self.value_cache = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(num_slots)]
        self.pos = torch.zeros(1, dtype=torch.long, device=device)

    def reset(self) -> None:
        self.pos.zero_()

    def update(self, key, value, layer_idx):
        n = key.shape[2]
        start = int(self.pos.item())
        self.key_cache[layer_idx][:, :, start:start + n] = key
        self.value_cache[layer_idx][:, :, start:start + n] = value
        return self.key_cache[layer_idx], self.value_cache[layer_idx]

    append_prefill = update


class KVInt8Cache:
    r"""Streaming int8 KV cache (src/nova/kvattn.py:488-880), B200 kernels.

    Storage: each tensor family is one allocation over all layers --
    ``codes`` uint8 ``[2, slots, B, H_kv, max_len, D]`` (K then V), ``scales``
    fp16 ``[4, slots, B, H_kv, ceil(max_len/64), D]`` (K min, K step, V min,
    V step), ``ring`` fp16 ``[2, slots, B, H_kv, 64, D]`` (the <= 63 newest
    tokens whose group is not complete, at slot ``pos % 64``) -- and the
    reference's per-layer attributes (``kq``, ``vq``, ``kmn``, ``kst``, ``vmn``,
    ``vst``, ``tail_k``, ``tail_v``: lists indexed by layer) are views into
    them.  The five lengths live in one int64 device vector; ``pos``,
    ``first``, ``_written``, ``_qlen`` and ``_pg`` are 1-element views of it,
    so saving or restoring the cache state is a copy of a few tensors.

    ``update`` (decode) is one ``nova_kv_append_int8`` launch; ``attend`` is one
    ``nova_attn_decode_int8`` launch that reads prefix and ring and merges them
    in the same kernel.  Prefill writes an fp16 staging area sized to the
    prompt and ``finish_prefill`` quantizes its complete groups with
    ``nova_kv_quant_int8`` (bit-identical to ``quantize_int8(..., "token")``).
    """

    _LENGTHS = ("pos", "first", "_written", "_qlen", "_pg")

    def __init__(
        self,
        num_slots: int,
        num_kv_heads: int,
        head_dim: int,
        max_len: int,
        num_q_heads: int,
        batch: int = 1,
        dtype: torch.dtype = torch.float16,
        device: str | torch.device = "cuda",
        group: int = GROUP_T,
        chunk: int = CHUNK,
        num_warps: int = 8,
        num_stages: int = 2,
        window: int = 0,
    ) -> None:
        for ok, msg in ((head_dim == HEAD_DIM, f"head_dim must be {HEAD_DIM}, got {head_dim}"),
                        (num_q_heads % num_kv_heads == 0,
                         f"q heads {num_q_heads} not divisible by KV heads {num_kv_heads}"),
                        (num_q_heads // max(num_kv_heads, 1) <= MAX_GQ,
                         f"{num_q_heads // max(num_kv_heads, 1)} q heads per KV head exceeds {MAX_GQ}"),
                        (group == GROUP_T, f"group must be {GROUP_T}"),
                        (chunk % group == 0, f"chunk {chunk} must be a multiple of group {group}"),
                        (dtype == torch.float16, "dtype must be float16")):
            if not ok:
                raise ValueError(msg)
        self.num_slots, self.num_kv_heads, self.num_q_heads = int(num_slots), int(num_kv_heads), int(num_q_heads)
        self.head_dim, self.max_len, self.batch = int(head_dim), int(max_len), int(batch)
        self.group, self.chunk, self.window = int(group), int(chunk), int(window)
        self.num_warps, self.num_stages = int(num_warps), int(num_stages)   # Triton knobs, accepted and unused
        self.dtype, self.device = dtype, torch.device(device)
        self._alloc()
        # grid fixed by the capacity (one captured graph serves every length); with a window the splits
        # are laid over the window only
        span = min(self.max_len, self.window + self.group) if self.window else self.max_len
        self.n_splits = -(-span // self.chunk)
        self.workspace = new_workspace(self.batch, self.num_q_heads, self.num_kv_heads, self.n_splits, True,
                                       self.device)
        self.out = torch.zeros((self.batch, self.num_q_heads, 1, self.head_dim), dtype=dtype, device=self.device)
        self.lse = torch.zeros((self.batch, self.num_q_heads), dtype=torch.float32, device=self.device)
        self.merged = self.out  # prefix and ring are merged inside the kernel
        self.staging: Any = None

    def _alloc(self) -> None:
        L, B, H, D, dev = self.num_slots, self.batch, self.num_kv_heads, self.head_dim, self.device
        self.codes = torch.zeros((2, L, B, H, self.max_len, D), dtype=torch.uint8, device=dev)
        self.scales = torch.zeros((4, L, B, H, -(-self.max_len // self.group), D), dtype=self.dtype, device=dev)
        self.ring = torch.zeros((2, L, B, H, self.group, D), dtype=self.dtype, device=dev)
        self.lengths = torch.zeros(len(self._LENGTHS), dtype=torch.long, device=dev)
        self.kq, self.vq = list(self.codes[0]), list(self.codes[1])
        self.kmn, self.kst, self.vmn, self.vst = (list(self.scales[i]) for i in range(4))
        self.tail_k, self.tail_v = list(self.ring[0]), list(self.ring[1])
        for i, name in enumerate(self._LENGTHS):
            setattr(self, name, self.lengths[i:i + 1])

    # ---- StaticKVCache-compatible surface ----

    def get_seq_length(self, layer_idx: int = 0) -> int:
        return int(self.pos.item())

    def reset(self) -> None:
        self.lengths.zero_()
        if self.staging is not None:
            self.staging.reset()

    def set_lengths(self, total: int) -> None:
        """Lengths after ``total`` tokens are in the cache: pos = written =
        total, the int8 prefix the complete groups, no position dropped."""
        q = total - total % self.group
        self.lengths.copy_(torch.tensor([total, 0, total, q, q // self.group], dtype=torch.long))

    # ---- prefill: fp16 staging ----

    def begin_prefill(self, total_len: int) -> None:
        total_len = int(total_len)
        if total_len <= 0 or total_len > self.max_len:
            raise ValueError(f"prefill length {total_len} outside (0, {self.max_len}]")
        self.staging = _Staging(self.num_slots, self.num_kv_heads, self.head_dim, total_len, self.batch,
                                self.dtype, self.device)

    def set_prefill_pos(self, off: int) -> None:
        self.pos.fill_(int(off))
        self._ensure_staging()
        self.staging.pos.fill_(int(off))

    def _ensure_staging(self) -> None:
        if self.staging is None:
            raise RuntimeError("no fp16 staging area: call begin_prefill(total_len) before prefill")

    def update(self, key: torch.Tensor, value: torch.Tensor, layer_idx: int):
        """Write K/V; returns ``(None, None)`` (attention goes through
        ``attend`` / ``attend_prefill``), src/nova/kvattn.py:668-691."""
        if self.staging is not None:
            self.staging.update(key, value, layer_idx)
            return None, None
        if key.shape[2] != 1:
            raise RuntimeError("without a staging area only single-token decode updates are allowed; "
                               "call begin_prefill() for prefill")
        if key.stride(3) != 1 or value.stride(3) != 1 or key.stride()[:2] != value.stride()[:2]:
            key, value = key.contiguous(), value.contiguous()
        _lib.call("nova_kv_append_int8", key.data_ptr(), value.data_ptr(), key.stride(0), key.stride(1),
                  self.tail_k[layer_idx].data_ptr(), self.tail_v[layer_idx].data_ptr(),
                  self.kq[layer_idx].data_ptr(), self.vq[layer_idx].data_ptr(),
                  self.kmn[layer_idx].data_ptr(), self.kst[layer_idx].data_ptr(),
                  self.vmn[layer_idx].data_ptr(), self.vst[layer_idx].data_ptr(),
                  self.pos.data_ptr(), self._written.data_ptr(), self._qlen.data_ptr(), self._pg.data_ptr(),
                  self.batch, self.num_kv_heads, self.max_len, self.head_dim, self.group,
                  _lib.stream_of(self.device))
        return None, None

    append_prefill = update

    def refresh_scalars(self) -> None:
        """Recompute written / qlen / pg from ``pos`` as a decode update at
        ``pos`` leaves them (written = pos + 1); reads ``pos`` on the host, so
        call it outside a graph (src/nova/kvattn.py:699-714)."""
        w = int(self.pos.item()) + 1
        q = w - w % self.group
        self.lengths[2:].copy_(torch.tensor([w, q, q // self.group], dtype=torch.long))

    def write_ring(self, layer_idx: int, k: torch.Tensor, v: torch.Tensor, end: int) -> None:
        """Put the last min(end, 64) positions of fp16 K/V ``[B, H_kv, n, D]``
        (whose last position is ``end - 1``) into the layer's ring: position p
        goes to slot p % 64, i.e. at most two contiguous slot ranges."""
        take = min(int(end), self.group, k.shape[2])
        p0 = end - take
        s0 = p0 % self.group
        first = min(take, self.group - s0)
        for ring, src in ((self.tail_k[layer_idx], k), (self.tail_v[layer_idx], v)):
            seg = src[:, :, src.shape[2] - take:]
            ring[:, :, s0:s0 + first].copy_(seg[:, :, :first])
            if take > first:
                ring[:, :, :take - first].copy_(seg[:, :, first:])

    def finish_prefill(self, total: int) -> None:
        """Quantize the complete groups of the staging area, fill the ring with
        the last <= 64 tokens, set the lengths, free the staging area
        (src/nova/kvattn.py:745-783)."""
        self._ensure_staging()
        total = int(total)
        full = total - total % self.group
        stream = _lib.stream_of(self.device)
        g_cap = self.scales.shape[4]
        for layer in range(self.num_slots):
            staged = (self.staging.key_cache[layer], self.staging.value_cache[layer])
            if full:
                for j, src in enumerate(staged):   # j = 0: K, 1: V
                    _lib.call("nova_kv_quant_int8", src.data_ptr(), src.shape[2] * self.head_dim,
                              self.codes[j, layer].data_ptr(), self.max_len * self.head_dim,
                              self.scales[2 * j, layer].data_ptr(), self.scales[2 * j + 1, layer].data_ptr(),
                              g_cap * self.head_dim, self.batch * self.num_kv_heads, full, self.head_dim,
                              self.group, stream)
            if total:
                self.write_ring(layer, staged[0][:, :, :total], staged[1][:, :, :total], total)
        self.set_lengths(total)
        self.staging = None

    def release_staging(self) -> None:
        self.staging = None

    def attend_prefill(self, query: torch.Tensor, layer_idx: int) -> torch.Tensor:
        """Causal attention of a prefill chunk (queries at positions off ..
        off+n-1, ``[B, H_q, n, D]``) over the fp16 staging area up to the
        chunk's end (src/nova/kvattn.py:791-815), in one
        ``nova_attn_prefill_int8`` launch; with ``window`` a query at q sees
        only positions p > q - window.  Returns ``[B, H_q, n, D]`` (a view of
        the kernel's token-major output)."""
        self._ensure_staging()
        b, hq, n, d = query.shape
        off = int(self.staging.pos.item())
        keys = self.staging.key_cache[layer_idx]
        vals = self.staging.value_cache[layer_idx]
        out = prefill_attention(query.contiguous(), keys, vals, prefix=off, window=self.window)
        return out.view(b, n, hq, d).transpose(1, 2)

    def ring_mask(self) -> torch.Tensor:
        """Which ring slots the next attention reads, ``[1, 1, 1, 64]`` bool
        (src/nova/kvattn.py:819-833): slot i holds the position u - age with
        u = written - 1 and age = (u - i) mod 64; it is read when that position
        is at or after qlen and first (and, with a window, age < window).  The
        kernel evaluates the same predicate itself; this is for callers."""
        u = self._written - 1
        age = torch.remainder(u - torch.arange(self.group, device=self.device), self.group)
        newest_allowed = u - torch.maximum(self._qlen, self.first)   # largest age still valid
        valid = age <= newest_allowed
        if self.window:
            valid &= age < self.window
        return valid.view(1, 1, 1, self.group)

    def attend(self, query: torch.Tensor, layer_idx: int) -> torch.Tensor:
        """Decode-step attention: int8 prefix + fp16 ring, merged in-kernel
        (src/nova/kvattn.py:835-862).  No host sync, no allocation."""
        if query.shape[2] != 1:
            raise ValueError("attend() handles one decode token (q_len == 1); use attend_prefill()")
        launch_attention(query[:, :, 0], (self.kq[layer_idx], self.kmn[layer_idx], self.kst[layer_idx],
                                          self.vq[layer_idx], self.vmn[layer_idx], self.vst[layer_idx]),
                         (self.tail_k[layer_idx], self.tail_v[layer_idx]), self.out[:, :, 0], self.lse,
                         self._qlen, self._pg, self._written, self.first, self.workspace,
                         max_len=self.max_len, n_splits=self.n_splits, chunk=self.chunk, window=self.window)
        return self.out

    # ---- capacity-bucket migration ----

    def grow(self, new_max_len: int) -> "KVInt8Cache":
        """A cache of capacity ``new_max_len`` holding this cache's contents:
        the int8 codes and min/step scales of every written group, the fp16
        ring and the lengths, copied on the device (the reference moves fp16
        caches across buckets in ``GraphDecoder.grow``, src/nova/decode.py:
        444-500, and raises NotImplementedError for the int8 cache).  The split
        size is kept, so the added splits are empty and decoding continues
        bit-identically; a captured decode graph must be captured again.  The
        staging area is not carried over."""
        new_max_len = int(new_max_len)
        if new_max_len < self.max_len:
            raise ValueError(f"new capacity {new_max_len} is below the current {self.max_len}")
        new = KVInt8Cache(self.num_slots, self.num_kv_heads, self.head_dim, new_max_len, self.num_q_heads,
                          batch=self.batch, dtype=self.dtype, device=self.device, group=self.group, chunk=self.chunk,
                          num_warps=self.num_warps, num_stages=self.num_stages, window=self.window)
        new.codes[..., :self.max_len, :].copy_(self.codes)
        new.scales[..., :self.scales.shape[4], :].copy_(self.scales)
        new.ring.copy_(self.ring)
        new.lengths.copy_(self.lengths)
        return new

    # ---- memory ----

    def nbytes(self) -> int:
        """Resident bytes of the int8 codes, the scales and the fp16 ring."""
        return sum(t.numel() * t.element_size() for t in (self.codes, self.scales, self.ring))

    def fp16_nbytes(self) -> int:
        """Bytes an fp16 cache of the same capacity would hold."""
        return self.codes.numel() * 2

    def extra_repr(self) -> str:
        mib = 1 << 20
        return (f"int8 KV, {self.num_slots} layers x {self.batch} x {self.num_kv_heads} heads x {self.max_len} "
                f"tokens: {self.nbytes() / mib:.0f} MiB ({self.nbytes() / self.fp16_nbytes():.2f} of fp16)")
