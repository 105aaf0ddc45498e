"""ctypes binding of ``libnova_b200.so`` (declared in ``include/nova_b200.h``).

The library is loaded from the package directory (built in-tree by
``python -m nova_b200.build``).  There is no fallback: if the shared object is
missing, or the tensors are not on a CUDA device, the calls raise.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().with_name("libnova_b200.so")

NOVA_OK, NOVA_ERR_INVALID, NOVA_ERR_ALIGN, NOVA_ERR_UNSUPPORTED, NOVA_ERR_CUDA = range(5)
NF4_PLAIN, NF4_RESIDUAL, NF4_SILU_MUL, NF4_ARGMAX, NF4_F32, NF4_SLOTS = range(6)
NOVA_ATTN_NOALLOC_SCRATCH_BYTES = 4 << 20   # built-in scratch of nova_attn_decode_int8_noalloc

_P = ctypes.c_void_p
_I = ctypes.c_int64
_i = ctypes.c_int


class AttnArgs(ctypes.Structure):
    """Mirror of ``nova_attn_int8_args``."""

    _fields_ = [
        ("q", _P), ("q_b_stride", _I), ("q_h_stride", _I),
        ("kq", _P), ("vq", _P), ("kmn", _P), ("kst", _P), ("vmn", _P), ("vst", _P),
        ("tail_k", _P), ("tail_v", _P),
        ("out", _P), ("o_b_stride", _I), ("o_h_stride", _I),
        ("lse", _P), ("lse_b_stride", _I),
        ("qlen", _P), ("pg", _P), ("written", _P), ("first", _P),
        ("workspace", _P), ("workspace_bytes", _I),
        ("batch", _I), ("q_heads", _I), ("kv_heads", _I), ("max_len", _I), ("groups", _I),
        ("head_dim", _I), ("group", _I), ("chunk", _I), ("n_splits", _I), ("window", _I),
        ("defer_merge", _I),
    ]


class NF4Args(ctypes.Structure):
    """Mirror of ``nova_nf4_args``."""

    _fields_ = [
        ("x", _P), ("x_stride", _I), ("norm_weight", _P), ("eps", ctypes.c_double),
        ("packed", _P), ("absmax", _P), ("absmax_fp32", _I), ("lut", _P), ("bias", _P),
        ("residual", _P), ("res_stride", _I), ("out", _P), ("out_stride", _I), ("argmax", _P),
        ("token_out", _P), ("pos", _P), ("embed", _P), ("embed_out", _P), ("embed_out_stride", _I),
        ("embed_dim", _I), ("workspace", _P), ("workspace_bytes", _I),
        ("m", _I), ("n", _I), ("k", _I), ("epilogue", _I), ("layout", _I),
        ("add_slots", _P), ("add_k", _I), ("resid_out", _P),
        ("edge_out", _P), ("edge_in", _P), ("edge_k", _I),
        ("attn_part", _P), ("attn_splits", _I), ("attn_heads", _I), ("add_heads", _P), ("add_nheads", _I),
    ]


class QKArgs(ctypes.Structure):
    """Mirror of ``nova_qk_args``."""

    _fields_ = [
        ("qkv", _P), ("qkv_stride", _I), ("q_norm_weight", _P), ("k_norm_weight", _P), ("eps", ctypes.c_double),
        ("cos", _P), ("sin", _P), ("rope_len", _I), ("q_out", _P), ("q_out_stride", _I),
        ("tail_k", _P), ("tail_v", _P), ("kq", _P), ("vq", _P), ("kmn", _P), ("kst", _P), ("vmn", _P), ("vst", _P),
        ("pos", _P), ("written", _P), ("qlen", _P), ("pg", _P),
        ("batch", _I), ("q_heads", _I), ("kv_heads", _I), ("head_dim", _I), ("max_len", _I), ("group", _I),
    ]


class PrefillAttnArgs(ctypes.Structure):
    """Mirror of ``nova_prefill_attn_args``."""

    _fields_ = [
        ("q", _P), ("q_b_stride", _I), ("q_h_stride", _I), ("q_t_stride", _I),
        ("k", _P), ("v", _P), ("kv_b_stride", _I), ("kv_h_stride", _I), ("kv_t_stride", _I),
        ("kq", _P), ("vq", _P), ("kmn", _P), ("kst", _P), ("vmn", _P), ("vst", _P), ("max_len", _I), ("groups", _I),
        ("out", _P), ("o_b_stride", _I), ("o_t_stride", _I),
        ("batch", _I), ("q_heads", _I), ("kv_heads", _I), ("head_dim", _I), ("n", _I), ("prefix", _I),
        ("int8_len", _I), ("window", _I),
    ]


class QKPrefillArgs(ctypes.Structure):
    """Mirror of ``nova_qk_prefill_args``."""

    _fields_ = [
        ("qkv", _P), ("qkv_b_stride", _I), ("qkv_t_stride", _I), ("q_norm_weight", _P), ("k_norm_weight", _P),
        ("eps", ctypes.c_double), ("cos", _P), ("sin", _P), ("rope_len", _I),
        ("q_out", _P), ("k_out", _P), ("k_pre", _P), ("v_out", _P),
        ("q_b_stride", _I), ("q_h_stride", _I), ("kv_b_stride", _I), ("kv_h_stride", _I),
        ("batch", _I), ("q_heads", _I), ("kv_heads", _I), ("head_dim", _I), ("n", _I), ("pos0", _I),
    ]


class SampleArgs(ctypes.Structure):
    """Mirror of ``nova_sample_args``."""

    _fields_ = [
        ("logits", _P), ("logits_stride", _I), ("seen", _P), ("seen_stride", _I), ("uniform", _P),
        ("token_out", _P), ("embed", _P), ("embed_out", _P), ("embed_out_stride", _I), ("embed_dim", _I),
        ("probs_out", _P), ("idx_out", _P), ("seen_mark", _P), ("seen_mark_stride", _I),
        ("rows", _I), ("vocab", _I), ("top_k", _I),
        ("temperature", ctypes.c_double), ("top_p", ctypes.c_double), ("repetition_penalty", ctypes.c_double),
    ]


class TPAllReduceArgs(ctypes.Structure):
    """Mirror of ``nova_tp_allreduce_args``."""

    _fields_ = [
        ("partial", _P), ("residual", _P), ("res_stride", _I), ("recv", _P * 8), ("epoch", _P), ("counter", _P),
        ("err", _P), ("rows", _I), ("n", _I), ("rank", _I), ("world", _I), ("timeout_ns", _I),
    ]


# name -> argtypes (every entry point returns int status unless noted)
_SIGNATURES: dict[str, list] = {
    "nova_abi_sizes": [_P, _i],
    "nova_kv_quant_int8": [_P, _I, _P, _I, _P, _P, _I, _I, _I, _I, _I, _P],
    "nova_kv_dequant_int8": [_P, _I, _P, _P, _I, _P, _I, _I, _I, _I, _I, _P],
    "nova_kv_append_int8": [_P, _P, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                            _I, _I, _I, _I, _I, _P],
    "nova_attn_workspace_bytes": [_I, _I, _I, _I, _i, ctypes.POINTER(_I)],
    "nova_attn_decode_int8": [ctypes.POINTER(AttnArgs), _P],
    "nova_attn_read_error": [_P, _I, _I, ctypes.POINTER(_i)],
    "nova_attn_decode_int8_noalloc": [ctypes.POINTER(AttnArgs), _P],
    "nova_attn_noalloc_read_error": [ctypes.POINTER(_i)],
    "nova_nf4_workspace_bytes": [_I, ctypes.POINTER(_I)],
    "nova_nf4_gemv": [ctypes.POINTER(NF4Args), _P],
    "nova_nf4_gemv_read_error": [_P, ctypes.POINTER(_i)],
    "nova_nf4_quantize": [_P, _I, _I, _P, _P, _P, _i, _P],
    "nova_nf4_dequant": [_P, _P, _i, _P, _P, _I, _I, _P],
    "nova_nf4_native_bytes": [_I, _I, ctypes.POINTER(_I)],
    "nova_nf4_pack_native": [_P, _P, _i, _P, _I, _I, _P],
    "nova_nf4_pack_tc": [_P, _P, _i, _P, _I, _I, _P],
    "nova_set_launch_flags": [_i],
    "nova_rmsnorm": [_P, _I, _P, _I, _P, _I, _P, _P, _I, _I, _I, ctypes.c_double, _P],
    "nova_residual_add_f32": [_P, _I, _P, _I, _I, _I, _P],
    "nova_tp_recv_bytes": [_I, _I, _I, ctypes.POINTER(_I)],
    "nova_tp_allreduce_add": [ctypes.POINTER(TPAllReduceArgs), _P],
    "nova_ipc_handle": [_P, _P, ctypes.POINTER(_I)],
    "nova_ipc_open": [_P, _I, ctypes.POINTER(_P), ctypes.POINTER(_P)],
    "nova_ipc_close": [_P],
    "nova_nf4_gemm_workspace_bytes": [_I, _I, ctypes.POINTER(_I)],
    "nova_nf4_gemm": [ctypes.POINTER(NF4Args), _P],
    "nova_nf4_gemm_read_error": [_P, ctypes.POINTER(_i)],
    "nova_qk_norm_rope_append": [ctypes.POINTER(QKArgs), _P],
    "nova_qk_append_attn_int8": [ctypes.POINTER(QKArgs), ctypes.POINTER(AttnArgs), _P],
    "nova_sample_topk": [ctypes.POINTER(SampleArgs), _P],
    "nova_attn_prefill_int8": [ctypes.POINTER(PrefillAttnArgs), _P],
    "nova_qk_prefill": [ctypes.POINTER(QKPrefillArgs), _P],
}
_STRING_FNS = ("nova_version", "nova_last_error")
_INT_FNS = ("nova_get_launch_flags",)
ABI_STRUCTS = ("AttnArgs", "NF4Args", "QKArgs", "PrefillAttnArgs", "QKPrefillArgs", "SampleArgs", "TPAllReduceArgs")

_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Load (once) and return the CUDA library.  Raises RuntimeError when the
    shared object has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH.name} is not built; run `python -m nova_b200.build`")
        h = ctypes.CDLL(str(LIB_PATH))
        for name, argtypes in _SIGNATURES.items():
            fn = getattr(h, name)
            fn.argtypes = argtypes
            fn.restype = ctypes.c_int
        for name in _STRING_FNS:
            fn = getattr(h, name)
            fn.argtypes = []
            fn.restype = ctypes.c_char_p
        for name in _INT_FNS:
            fn = getattr(h, name)
            fn.argtypes = []
            fn.restype = ctypes.c_int
        _lib = h
    return _lib


def exported_names() -> list[str]:
    return list(_SIGNATURES) + list(_STRING_FNS) + list(_INT_FNS)


LAUNCH_PDL = 1          # programmatic dependent launch
LAUNCH_WARP_SPLITK = 2  # native-layout GEMV: warp-level instead of CTA-level split-K


def set_pdl(enabled: bool) -> None:
    """Programmatic dependent launch for every kernel launched afterwards
    (other launch flags are kept)."""
    flags = lib().nova_get_launch_flags()
    call("nova_set_launch_flags", (flags | LAUNCH_PDL) if enabled else (flags & ~LAUNCH_PDL))


def set_launch_flags(flags: int) -> None:
    call("nova_set_launch_flags", int(flags))


def pdl_enabled() -> bool:
    return bool(lib().nova_get_launch_flags() & 1)


def version() -> str:
    return lib().nova_version().decode()


def last_error() -> str:
    return lib().nova_last_error().decode()


def check(rc: int, what: str) -> None:
    if rc == NOVA_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc in (NOVA_ERR_INVALID, NOVA_ERR_ALIGN, NOVA_ERR_UNSUPPORTED):
        raise ValueError(msg)
    raise RuntimeError(msg)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)


def ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def stream_of(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def available() -> bool:
    """True when the library loads and a CUDA device is visible."""
    try:
        lib()
    except (RuntimeError, OSError):
        return False
    return torch.cuda.is_available()


def require_cuda(*tensors: torch.Tensor, names: tuple[str, ...] = ()) -> None:
    for i, t in enumerate(tensors):
        if t is not None and not t.is_cuda:
            name = names[i] if i < len(names) else f"arg{i}"
            raise ValueError(f"{name} must be a CUDA tensor (the B200 path has no CPU fallback)")
