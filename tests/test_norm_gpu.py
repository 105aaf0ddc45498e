"""GPU: RMSNorm (nova_rmsnorm) and the fused q/k-norm + RoPE + KV append
(nova_qk_norm_rope_append) against the oracle and the reference fixtures."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import assert_ulp_or_abs, golden
from oracle import kvquant as okv
from oracle import norm as onorm

pytestmark = pytest.mark.gpu


def _close_fp16(got, want, tag, min_exact=0.99, max_ulp=1.0):
    """RMSNorm: a different fp32 summation order can move 1/sqrt(var) by an
    ulp, which flips an fp16 rounding now and then: <= 1 ULP everywhere and
    bit-exact almost everywhere.  After RoPE (two more fp16-rounded products
    and a sum, as in the reference) such a flip can reach 2 ULP."""
    st = assert_ulp_or_abs(got, want, max_ulp, 0.0, tag)
    assert st["exact"] >= min_exact, f"{tag}: only {st['exact']:.4f} bit-exact"


@pytest.mark.parametrize("dim", [2560, 128])
def test_rmsnorm_matches_reference_fixture(cuda_lib, dim):
    from nova_b200.kernels import fused_rms_norm

    g = golden("norm_rope.npz")
    y = fused_rms_norm(torch.from_numpy(g[f"norm{dim}_x"]).cuda(), torch.from_numpy(g[f"norm{dim}_w"]).cuda(), 1e-6)
    _close_fp16(y.cpu().numpy(), g[f"norm{dim}_y"], f"norm{dim}")


def test_lean_rmsnorm_module(cuda_lib):
    from nova_b200.norm import LeanRMSNorm

    x = (torch.randn(2, 3, 2560, generator=torch.Generator().manual_seed(0)) * 2).half()
    norm = LeanRMSNorm(2560, eps=1e-6, dtype=torch.float16, device="cuda")
    with torch.no_grad():
        norm.weight.copy_((1 + 0.05 * torch.randn(2560, generator=torch.Generator().manual_seed(1))).half())
    y = norm(x.cuda())
    want = onorm.rms_norm(x.numpy(), norm.weight.detach().cpu().numpy(), 1e-6)
    _close_fp16(y.cpu().numpy(), want, "LeanRMSNorm")


def test_residual_rmsnorm(cuda_lib):
    from nova_b200.kernels import residual_rms_norm

    g = torch.Generator().manual_seed(2)
    x = torch.randn(4, 2560, generator=g).half()
    r = torch.randn(4, 2560, generator=g).half()
    w = (1 + 0.1 * torch.randn(2560, generator=g)).half()
    h, y = residual_rms_norm(x.cuda(), r.cuda(), w.cuda(), 1e-6)
    hw = (r.numpy().astype(np.float32) + x.numpy().astype(np.float32)).astype(np.float16)
    np.testing.assert_array_equal(h.cpu().numpy().view(np.uint16), hw.view(np.uint16))
    _close_fp16(y.cpu().numpy(), onorm.rms_norm(hw, w.numpy(), 1e-6), "residual+norm")


def _rope_tables(max_pos):
    cos, sin = onorm.rope_cos_sin(np.arange(max_pos))
    return torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()


def test_qk_norm_rope_append(cuda_lib):
    """q/k per-head norm + RoPE + ring append with a group completing at
    position 127, against the oracle, for batch 2."""
    from nova_b200 import _lib
    from nova_b200.kvattn import KVInt8Cache

    b, hq, hkv, d, max_len = 2, 32, 8, 128, 256
    g = torch.Generator().manual_seed(3)
    cos, sin = _rope_tables(max_len)
    qn = (1 + 0.1 * torch.randn(d, generator=g)).half()
    kn = (1 + 0.1 * torch.randn(d, generator=g)).half()
    cache = KVInt8Cache(num_slots=1, num_kv_heads=hkv, head_dim=d, max_len=max_len, num_q_heads=hq, batch=b)
    ring_k = np.zeros((b, hkv, 64, d), np.float16)
    ring_v = np.zeros_like(ring_k)
    q_out = torch.empty(b, hq * d, dtype=torch.float16, device="cuda")
    qn_d, kn_d = qn.cuda(), kn.cuda()
    for pos in range(64, 128):
        qkv = (torch.randn(b, (hq + 2 * hkv) * d, generator=g) * 2).half()
        qkv_dev = qkv.cuda()
        cache.pos.fill_(pos)
        a = _lib.QKArgs()
        a.qkv, a.qkv_stride = qkv_dev.data_ptr(), qkv_dev.stride(0)
        a.q_norm_weight, a.k_norm_weight, a.eps = qn_d.data_ptr(), kn_d.data_ptr(), 1e-6
        a.cos, a.sin, a.rope_len = cos.data_ptr(), sin.data_ptr(), max_len
        a.q_out, a.q_out_stride = q_out.data_ptr(), q_out.stride(0)
        a.tail_k, a.tail_v = cache.tail_k[0].data_ptr(), cache.tail_v[0].data_ptr()
        a.kq, a.vq = cache.kq[0].data_ptr(), cache.vq[0].data_ptr()
        a.kmn, a.kst, a.vmn, a.vst = (cache.kmn[0].data_ptr(), cache.kst[0].data_ptr(), cache.vmn[0].data_ptr(),
                                      cache.vst[0].data_ptr())
        a.pos, a.written, a.qlen, a.pg = (cache.pos.data_ptr(), cache._written.data_ptr(), cache._qlen.data_ptr(),
                                          cache._pg.data_ptr())
        a.batch, a.q_heads, a.kv_heads, a.head_dim, a.max_len, a.group = b, hq, hkv, d, max_len, 64
        _lib.check(_lib.lib().nova_qk_norm_rope_append(_lib.ctypes.byref(a), _lib.stream_of()), "qk")
        torch.cuda.synchronize()
        # oracle
        x = qkv.numpy().reshape(b, hq + 2 * hkv, d)
        c, s = cos[pos].cpu().numpy(), sin[pos].cpu().numpy()
        q_want = onorm.apply_rope(onorm.rms_norm(x[:, :hq], qn.numpy(), 1e-6), c, s)
        k_want = onorm.apply_rope(onorm.rms_norm(x[:, hq:hq + hkv], kn.numpy(), 1e-6), c, s)
        _close_fp16(q_out.cpu().numpy().reshape(b, hq, d), q_want, f"q pos={pos}", min_exact=0.98, max_ulp=2.0)
        ring_k[:, :, pos % 64] = cache.tail_k[0][:, :, pos % 64].cpu().numpy()
        ring_v[:, :, pos % 64] = x[:, hq + hkv:]
        _close_fp16(ring_k[:, :, pos % 64], k_want, f"k pos={pos}", min_exact=0.98, max_ulp=2.0)
        np.testing.assert_array_equal(cache.tail_v[0][:, :, pos % 64].cpu().numpy(), x[:, hq + hkv:])
    assert int(cache._qlen.item()) == 128 and int(cache._written.item()) == 128 and int(cache._pg.item()) == 2
    # group 1 (positions 64..127) was requantized from the ring at position 127
    oq, omn, ost = okv.quantize_ring(cache.tail_k[0].cpu().numpy())
    np.testing.assert_array_equal(cache.kq[0][:, :, 64:128].cpu().numpy(), oq)
    np.testing.assert_array_equal(cache.kmn[0][:, :, 1].cpu().numpy().view(np.uint16), omn.view(np.uint16))
    np.testing.assert_array_equal(cache.kst[0][:, :, 1].cpu().numpy().view(np.uint16), ost.view(np.uint16))
    vq_, vmn_, vst_ = okv.quantize_ring(ring_v)
    np.testing.assert_array_equal(cache.vq[0][:, :, 64:128].cpu().numpy(), vq_)
