"""GPU: the prefill kernels against the CPU oracle.

nova_attn_prefill_int8 -- causal attention of a chunk of queries over int8
cache positions read in place (dequantized as src/nova/kvquant.py:166-176)
and fp16 keys, each query against the oracle's fp32 softmax attention over
exactly the positions it may see (src/nova/kvattn.py:791-815 semantics, the
window of src/nova/decode.py:207-220); criterion: 4 fp16 ULP or 1e-3, the
reference's streaming-cache bound (tests/test_kvattn_stream.py:38-41).
nova_qk_prefill -- q/k norm + RoPE of a chunk against the oracle's RMSNorm
and fp16 op-by-op RoPE (src/nova/norm.py:37-42, src/nova/layers.py:30-36),
within 2 fp16 ULP."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import assert_ulp_or_abs
from oracle import attention as oatt
from oracle import kvquant as okv
from oracle import norm as onorm

pytestmark = pytest.mark.gpu

D = 128


@pytest.mark.parametrize("b,hq,hkv,n,prefix,int8_len,window", [
    (1, 32, 8, 150, 0, 0, 0),        # a whole prompt over its own fp16 K/V
    (2, 32, 8, 100, 128, 128, 0),    # a chunk after two int8 groups
    (1, 8, 2, 70, 200, 192, 0),      # int8 groups, then staged fp16 positions, then the chunk
    (1, 8, 2, 130, 64, 64, 100),     # sliding window across the int8 / fp16 boundary
    (1, 32, 8, 1, 511, 448, 0),      # a single query
])
def test_prefill_attention_matches_oracle(cuda_lib, b, hq, hkv, n, prefix, int8_len, window):
    from nova_b200.kvattn import pack_int8_kv, prefill_attention

    g = torch.Generator().manual_seed(n + prefix)
    total = prefix + n
    k = (torch.randn(b, hkv, total, D, generator=g) * 0.7).half()
    v = (torch.randn(b, hkv, total, D, generator=g) * 0.7).half()
    q = (torch.randn(b, hq, n, D, generator=g) * 0.7).half()
    int8 = None
    keys, vals = k.numpy(), v.numpy()
    if int8_len:
        max_len = int8_len + 64
        kc = torch.zeros(b, hkv, max_len, D, dtype=torch.float16)
        vc = torch.zeros_like(kc)
        kc[:, :, :int8_len], vc[:, :, :int8_len] = k[:, :, :int8_len], v[:, :, :int8_len]
        int8 = pack_int8_kv(kc.cuda(), vc.cuda())
        kq, kmn, kst, vq, vmn, vst = (t.cpu().numpy() for t in int8)
        kd = okv.dequantize_int8_token(kq[:, :, :int8_len], kmn, kst, 64)
        vd = okv.dequantize_int8_token(vq[:, :, :int8_len], vmn, vst, 64)
        keys = np.concatenate([kd, keys[:, :, int8_len:]], axis=2)
        vals = np.concatenate([vd, vals[:, :, int8_len:]], axis=2)
    got = prefill_attention(q.cuda(), k[:, :, int8_len:].cuda().contiguous(), v[:, :, int8_len:].cuda().contiguous(),
                            prefix=prefix, int8=int8, int8_len=int8_len, window=window)
    got = got.view(b, n, hq, D).cpu().numpy()
    qn = q.numpy()
    for i in range(n):
        p = prefix + i
        valid = np.arange(p + 1) > p - window if window else np.ones(p + 1, bool)
        want, _ = oatt.attend(qn[:, :, i], keys[:, :, :p + 1], vals[:, :, :p + 1], np.broadcast_to(valid, (b, p + 1)))
        assert_ulp_or_abs(got[:, i], want, 4.0, 1e-3, f"query {i}")


def test_qk_prefill_matches_oracle(cuda_lib):
    from nova_b200 import _lib
    from nova_b200.decoder import rope_tables

    b, hq, hkv, n, pos0 = 2, 8, 2, 37, 1000
    g = torch.Generator().manual_seed(3)
    qkv = (torch.randn(b, n, (hq + 2 * hkv) * D, generator=g) * 2).half()
    qw = (1 + 0.1 * torch.randn(D, generator=g)).half()
    kw = (1 + 0.1 * torch.randn(D, generator=g)).half()
    cos, sin = rope_tables(2048)
    dev = {"dtype": torch.float16, "device": "cuda"}
    q_out, k_out = torch.empty(b, hq, n, D, **dev), torch.empty(b, hkv, n, D, **dev)
    k_pre, v_out = torch.empty(b, hkv, n, D, **dev), torch.empty(b, hkv, n, D, **dev)
    qc, qwc, kwc = qkv.cuda(), qw.cuda(), kw.cuda()
    a = _lib.QKPrefillArgs()
    a.qkv, a.qkv_b_stride, a.qkv_t_stride = qc.data_ptr(), qc.stride(0), qc.stride(1)
    a.q_norm_weight, a.k_norm_weight, a.eps = qwc.data_ptr(), kwc.data_ptr(), 1e-6
    a.cos, a.sin, a.rope_len = cos.data_ptr(), sin.data_ptr(), cos.shape[0]
    a.q_out, a.k_out, a.k_pre, a.v_out = q_out.data_ptr(), k_out.data_ptr(), k_pre.data_ptr(), v_out.data_ptr()
    a.q_b_stride, a.q_h_stride, a.kv_b_stride, a.kv_h_stride = q_out.stride(0), q_out.stride(1), k_out.stride(0), \
        k_out.stride(1)
    a.batch, a.q_heads, a.kv_heads, a.head_dim, a.n, a.pos0 = b, hq, hkv, D, n, pos0
    _lib.check(_lib.lib().nova_qk_prefill(_lib.ctypes.byref(a), _lib.stream_of()), "nova_qk_prefill")
    x = qkv.numpy()
    oc, os_ = onorm.rope_cos_sin(np.arange(pos0, pos0 + n))
    qn = onorm.rms_norm(x[..., :hq * D].reshape(b, n, hq, D), qw.numpy())
    kn = onorm.rms_norm(x[..., hq * D:(hq + hkv) * D].reshape(b, n, hkv, D), kw.numpy())
    qe = onorm.apply_rope(qn, oc[None, :, None], os_[None, :, None]).transpose(0, 2, 1, 3)
    ke = onorm.apply_rope(kn, oc[None, :, None], os_[None, :, None]).transpose(0, 2, 1, 3)
    # the fp32 sum of squares is ordered differently: an fp16 rounding of the normed value moves now and then,
    # and RoPE adds two such values
    assert_ulp_or_abs(q_out.cpu().numpy(), qe, 2.0, 0.0, "q")
    assert_ulp_or_abs(k_out.cpu().numpy(), ke, 2.0, 0.0, "k")
    assert_ulp_or_abs(k_pre.cpu().numpy(), kn.transpose(0, 2, 1, 3), 1.0, 0.0, "k before RoPE")
    assert np.array_equal(v_out.cpu().numpy(), x[..., (hq + hkv) * D:].reshape(b, n, hkv, D).transpose(0, 2, 1, 3))


def test_cache_attend_prefill_in_chunks(cuda_lib):
    """KVInt8Cache.attend_prefill (the reference's prefill attention entry,
    src/nova/kvattn.py:791-815) in two chunks over the fp16 staging area,
    against the oracle, in the [B, H_q, n, D] shape LeanAttention expects."""
    from nova_b200.kvattn import KVInt8Cache

    b, hq, hkv, total = 1, 32, 8, 200
    g = torch.Generator().manual_seed(11)
    k = (torch.randn(b, hkv, total, D, generator=g) * 0.7).half()
    v = (torch.randn(b, hkv, total, D, generator=g) * 0.7).half()
    q = (torch.randn(b, hq, total, D, generator=g) * 0.7).half()
    cache = KVInt8Cache(num_slots=1, num_kv_heads=hkv, head_dim=D, max_len=256, num_q_heads=hq)
    cache.begin_prefill(total)
    outs = []
    for c0, c1 in ((0, 120), (120, 200)):
        cache.set_prefill_pos(c0)
        cache.update(k[:, :, c0:c1].cuda(), v[:, :, c0:c1].cuda(), 0)
        o = cache.attend_prefill(q[:, :, c0:c1].cuda(), 0)
        assert o.shape == (b, hq, c1 - c0, D)
        outs.append(o.float().cpu().numpy())
    got = np.concatenate(outs, axis=2)
    for i in range(total):
        want, _ = oatt.attend(q[:, :, i].numpy(), k[:, :, :i + 1].numpy(), v[:, :, :i + 1].numpy())
        assert_ulp_or_abs(got[:, :, i], want, 4.0, 1e-3, f"position {i}")
