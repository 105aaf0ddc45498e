"""GPU: nova_attn_decode_int8_noalloc (built-in scratch array, no workspace
argument) against nova_attn_decode_int8 with a caller-allocated workspace.

The same inputs go through both entry points; outputs and log-sum-exp must
agree within the attention tolerance of the reference's tests (2 fp16 ULP or
1e-5 absolute).  Two calls in a row with different shapes check that the
shared array's leftover contents do not leak into the next call.  This file
is named to be collected last, so it also runs after every other GPU test has
used the library in the same process."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import assert_ulp_or_abs

pytestmark = pytest.mark.gpu

D = 128
GROUP = 64


def _case(b, hq, hkv, max_len, qlen, written, seed):
    from nova_b200.kvattn import pack_int8_kv

    g = torch.Generator().manual_seed(seed)
    k = torch.randn(b, hkv, max_len, D, generator=g).half().cuda()
    v = torch.randn(b, hkv, max_len, D, generator=g).half().cuda()
    kv = pack_int8_kv(k, v)
    tail_k = torch.randn(b, hkv, GROUP, D, generator=g).half().cuda()
    tail_v = torch.randn(b, hkv, GROUP, D, generator=g).half().cuda()
    q = torch.randn(b, hq, D, generator=g).half().cuda()
    scal = {name: torch.tensor([val], dtype=torch.int64, device="cuda")
            for name, val in (("qlen", qlen), ("pg", qlen // GROUP), ("written", written))}
    return q, kv, (tail_k, tail_v), scal


def _args(q, kv, tail, scal, out, lse, *, max_len, chunk, n_splits, window, workspace=None):
    from nova_b200 import _lib

    kq, kmn, kst, vq, vmn, vst = kv
    a = _lib.AttnArgs()
    a.q, a.q_b_stride, a.q_h_stride = q.data_ptr(), q.stride(0), q.stride(1)
    a.kq, a.vq, a.kmn, a.kst, a.vmn, a.vst = (t.data_ptr() for t in (kq, vq, kmn, kst, vmn, vst))
    a.tail_k, a.tail_v = tail[0].data_ptr(), tail[1].data_ptr()
    a.out, a.o_b_stride, a.o_h_stride = out.data_ptr(), out.stride(0), out.stride(1)
    a.lse, a.lse_b_stride = lse.data_ptr(), lse.stride(0)
    a.qlen, a.pg, a.written = scal["qlen"].data_ptr(), scal["pg"].data_ptr(), scal["written"].data_ptr()
    a.first = None
    if workspace is not None:
        a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel()
    a.batch, a.q_heads, a.kv_heads = q.shape[0], q.shape[1], kq.shape[1]
    a.max_len, a.groups, a.head_dim, a.group = max_len, kmn.shape[2], D, GROUP
    a.chunk, a.n_splits, a.window = chunk, n_splits, window
    return a


def _noalloc_error() -> int:
    """The no-allocation entry point's error word on the current device (read and cleared)."""
    from nova_b200 import _lib

    val = ctypes.c_int(-1)
    _lib.check(_lib.lib().nova_attn_noalloc_read_error(ctypes.byref(val)), "nova_attn_noalloc_read_error")
    return int(val.value)


def _both(b, hq, hkv, max_len, qlen, written, chunk, window, seed):
    from nova_b200 import _lib
    from nova_b200.kvattn import new_workspace

    lib = _lib.lib()
    q, kv, tail, scal = _case(b, hq, hkv, max_len, qlen, written, seed)
    n_splits = -(-max_len // chunk)
    outs = []
    for noalloc in (False, True):
        out = torch.full((b, hq, D), float("nan"), dtype=torch.float16, device="cuda")
        lse = torch.full((b, hq), float("nan"), dtype=torch.float32, device="cuda")
        ws = None if noalloc else new_workspace(b, hq, hkv, n_splits, True, q.device)
        a = _args(q, kv, tail, scal, out, lse, max_len=max_len, chunk=chunk, n_splits=n_splits, window=window,
                  workspace=ws)
        fn = lib.nova_attn_decode_int8_noalloc if noalloc else lib.nova_attn_decode_int8
        _lib.check(fn(ctypes.byref(a), _lib.stream_of(q.device)), fn.__name__)
        torch.cuda.synchronize()
        outs.append((out.float().cpu().numpy(), lse.cpu().numpy()))
    (o_ref, l_ref), (o_new, l_new) = outs
    assert np.isfinite(o_new).all() and np.isfinite(l_new).all()
    assert_ulp_or_abs(o_new, o_ref.astype(np.float16), 2.0, 1e-5, f"noalloc out b={b} hq={hq}")
    np.testing.assert_allclose(l_new, l_ref, rtol=1e-6, atol=1e-6)
    assert _noalloc_error() == 0, "a bounded wait of the no-allocation call gave up"


def test_noalloc_matches_workspace_entry_two_calls(cuda_lib):
    # first call: batch 2, GQA 4, many splits + the fp16 ring
    _both(b=2, hq=32, hkv=8, max_len=3072, qlen=2944, written=2990, chunk=256, window=0, seed=1)
    # second call right after: another shape and a sliding window, over the same scratch array
    _both(b=1, hq=8, hkv=4, max_len=1536, qlen=1408, written=1450, chunk=128, window=700, seed=2)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs in one process")
def test_noalloc_on_a_second_device(cuda_lib):
    """The scratch address and the kernel attributes are per device: the same
    comparison with device 1 current, after calls on device 0."""
    _both(b=1, hq=32, hkv=8, max_len=1024, qlen=960, written=1000, chunk=256, window=0, seed=4)
    with torch.cuda.device(1):
        _both(b=1, hq=32, hkv=8, max_len=1024, qlen=960, written=1000, chunk=256, window=0, seed=5)


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda_lib):
    from nova_b200 import _lib

    need = ctypes.c_int64(0)
    _lib.call("nova_attn_workspace_bytes", 8, 32, 8, 255, 1, ctypes.byref(need))
    assert need.value > _lib.NOVA_ATTN_NOALLOC_SCRATCH_BYTES
    q, kv, tail, scal = _case(1, 8, 2, 256, 192, 200, 3)
    out = torch.empty(1, 8, D, dtype=torch.float16, device="cuda")
    lse = torch.empty(1, 8, dtype=torch.float32, device="cuda")
    a = _args(q, kv, tail, scal, out, lse, max_len=256, chunk=64, n_splits=4, window=0)
    a.batch, a.q_heads, a.kv_heads, a.n_splits = 8, 32, 8, 255   # sized past the array; rejected before launch
    rc = _lib.lib().nova_attn_decode_int8_noalloc(ctypes.byref(a), _lib.stream_of(q.device))
    assert rc == _lib.NOVA_ERR_UNSUPPORTED
    assert b"scratch" in _lib.lib().nova_last_error()
