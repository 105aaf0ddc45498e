"""CPU: the C-ABI library loads without a GPU and exports every entry point
that include/nova_b200.h declares (no compute calls here)."""

from __future__ import annotations

import ctypes
import re

import pytest

from conftest import REPO
from nova_b200 import _lib


def _declared() -> list[str]:
    names = []
    for hdr in (REPO / "include").glob("*.h"):
        text = hdr.read_text()
        names += re.findall(r"^NOVA_API\s+[\w\s\*]+?\b(nova_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = _declared()
    assert "nova_attn_decode_int8" in names and "nova_version" in names
    assert len(names) >= 8


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    for name in _declared():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"


def test_python_binding_covers_every_declared_symbol():
    assert sorted(_declared()) == sorted(_lib.exported_names())


def test_version_string_without_gpu():
    assert "sm_100a" in _lib.version()


def test_host_side_argument_checks_need_no_gpu():
    """Invalid arguments are rejected on the host before any launch."""
    lib = _lib.lib()
    rc = lib.nova_kv_quant_int8(None, 0, None, 0, None, None, 0, 1, 10, 0, 64, None)
    assert rc == _lib.NOVA_ERR_INVALID
    assert "dim" in _lib.last_error()
    out = ctypes.c_int64(0)
    rc = lib.nova_attn_workspace_bytes(1, 32, 8, 16, 1, ctypes.byref(out))
    assert rc == _lib.NOVA_OK and out.value > 0
    with pytest.raises(ValueError):
        _lib.check(lib.nova_attn_workspace_bytes(1, 30, 8, 16, 1, ctypes.byref(out)), "ws")


def test_fused_append_attention_checks_need_no_gpu():
    """nova_qk_append_attn_int8 rejects NULL arguments and q/k and attention
    arguments that disagree, on the host (the pointers below are never read)."""
    lib = _lib.lib()
    assert lib.nova_qk_append_attn_int8(None, None, None) == _lib.NOVA_ERR_INVALID
    qk, at = _lib.QKArgs(), _lib.AttnArgs()
    for s in (qk, at):
        s.batch, s.q_heads, s.kv_heads, s.max_len = 1, 32, 8, 256
    qk.head_dim, qk.group = 128, 64
    at.n_splits = 4
    fake = [0x10000 * (i + 1) for i in range(8)]
    qk.tail_k, qk.tail_v, qk.kq, qk.vq, qk.kmn, qk.kst, qk.vmn, qk.vst = fake
    at.tail_k, at.tail_v, at.kq, at.vq, at.kmn, at.kst, at.vmn, at.vst = fake
    at.batch = 2
    rc = lib.nova_qk_append_attn_int8(ctypes.byref(qk), ctypes.byref(at), None)
    assert rc == _lib.NOVA_ERR_INVALID and "disagree" in _lib.last_error()
    at.batch = 1
    at.vst = fake[0]
    rc = lib.nova_qk_append_attn_int8(ctypes.byref(qk), ctypes.byref(at), None)
    assert rc == _lib.NOVA_ERR_INVALID and "same ring" in _lib.last_error()
    at.vst = fake[7]
    at.tail_k = at.tail_v = None
    rc = lib.nova_qk_append_attn_int8(ctypes.byref(qk), ctypes.byref(at), None)
    assert rc == _lib.NOVA_ERR_INVALID and "tail ring" in _lib.last_error()
    qk.head_dim = 64
    assert lib.nova_qk_append_attn_int8(ctypes.byref(qk), ctypes.byref(at), None) == _lib.NOVA_ERR_UNSUPPORTED


def test_ctypes_mirrors_match_the_header_structs():
    """Every ctypes mirror in nova_b200/_lib.py has the size of the C struct it
    stands for (nova_abi_sizes), so a field added on one side only is caught
    without a GPU."""
    import ctypes

    from nova_b200 import _lib

    n = len(_lib.ABI_STRUCTS)
    out = (ctypes.c_int64 * n)()
    assert _lib.lib().nova_abi_sizes(out, n) == n
    for i, name in enumerate(_lib.ABI_STRUCTS):
        assert ctypes.sizeof(getattr(_lib, name)) == out[i], f"{name}: {ctypes.sizeof(getattr(_lib, name))} != {out[i]}"
