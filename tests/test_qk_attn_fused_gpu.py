"""GPU: the decode step's q/k norm + RoPE + ring append fused into the
attention launch (nova_qk_append_attn_int8) against the two separate launches
(nova_qk_norm_rope_append, then nova_attn_decode_int8) on the same state.
The ring, the int8 cache and the lengths must come out bit-identical; the
attention output within the attention criterion of tests/test_attn_gpu.py
(2 fp16 ULP or 1e-5): when a token completes a group, the fused launch attends
that group in its int8 form from the ring CTA instead of a prefix split, so
the split partials are merged in another order.  With a capacity far above
the prefix the fused launch also lays its splits over the prefix (256-token
splits instead of the host's chunk), so the partials differ and only the
elementwise criterion applies."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import assert_ulp_or_abs
from oracle import norm as onorm

pytestmark = pytest.mark.gpu

D = 128


def _qk_args(qkv, qn, kn, cos, sin, q_out, cache):
    from nova_b200 import _lib

    a = _lib.QKArgs()
    a.qkv, a.qkv_stride = qkv.data_ptr(), qkv.stride(0)
    a.q_norm_weight, a.k_norm_weight, a.eps = qn.data_ptr(), kn.data_ptr(), 1e-6
    a.cos, a.sin, a.rope_len = cos.data_ptr(), sin.data_ptr(), cos.shape[0]
    a.q_out, a.q_out_stride = q_out.data_ptr(), q_out.stride(0)
    a.tail_k, a.tail_v = cache.tail_k[0].data_ptr(), cache.tail_v[0].data_ptr()
    a.kq, a.vq = cache.kq[0].data_ptr(), cache.vq[0].data_ptr()
    a.kmn, a.kst, a.vmn, a.vst = (cache.kmn[0].data_ptr(), cache.kst[0].data_ptr(), cache.vmn[0].data_ptr(),
                                  cache.vst[0].data_ptr())
    a.pos, a.written, a.qlen, a.pg = (cache.pos.data_ptr(), cache._written.data_ptr(), cache._qlen.data_ptr(),
                                      cache._pg.data_ptr())
    a.batch, a.q_heads, a.kv_heads = cache.batch, cache.num_q_heads, cache.num_kv_heads
    a.head_dim, a.max_len, a.group = D, cache.max_len, 64
    return a


def _attend(cache, q3, out3, qk=None):
    from nova_b200.kvattn import launch_attention

    launch_attention(q3, (cache.kq[0], cache.kmn[0], cache.kst[0], cache.vq[0], cache.vmn[0], cache.vst[0]),
                     (cache.tail_k[0], cache.tail_v[0]), out3, None, cache._qlen, cache._pg, cache._written,
                     cache.first, cache.workspace, max_len=cache.max_len, n_splits=cache.n_splits,
                     chunk=cache.chunk, window=cache.window, qk=qk)


def _state(cache):
    return [t.cpu().numpy() for t in (cache.tail_k[0], cache.tail_v[0], cache.kq[0], cache.vq[0], cache.kmn[0],
                                      cache.kst[0], cache.vmn[0], cache.vst[0], cache._written, cache._qlen,
                                      cache._pg)]


@pytest.mark.parametrize("b,hq,hkv,window,chunk,start,steps,max_len", [
    (2, 32, 8, 0, 64, 0, 140, 512),       # two group completions (positions 63 and 127), small splits
    (1, 32, 8, 100, 128, 180, 90, 512),   # sliding window across the completion at 255
    (3, 16, 8, 0, 256, 250, 20, 512),     # gq = 2, completion at 255 inside a larger split
    # capacity far above the prefix: the fused launch splits the prefix into 256-token splits
    # (not the host's 1024), across the completions at 703 and 767
    (1, 32, 8, 0, 1024, 690, 90, 4096),
])
def test_fused_append_attention_matches_two_launches(cuda_lib, b, hq, hkv, window, chunk, start, steps, max_len):
    from nova_b200.kvattn import KVInt8Cache

    g = torch.Generator().manual_seed(11 + b)
    cos_np, sin_np = onorm.rope_cos_sin(np.arange(max_len + 1))
    cos, sin = torch.from_numpy(cos_np).cuda(), torch.from_numpy(sin_np).cuda()
    qn = (1 + 0.1 * torch.randn(D, generator=g)).half().cuda()
    kn = (1 + 0.1 * torch.randn(D, generator=g)).half().cuda()
    caches = [KVInt8Cache(num_slots=1, num_kv_heads=hkv, head_dim=D, max_len=max_len, num_q_heads=hq, batch=b,
                          chunk=chunk, window=window) for _ in range(2)]
    # a random history: int8 codes, scales and ring contents identical in both caches
    gd = torch.Generator(device="cuda").manual_seed(5)
    for t in ("kq", "vq"):
        src = torch.randint(0, 256, getattr(caches[0], t)[0].shape, generator=gd, device="cuda", dtype=torch.uint8)
        for c in caches:
            getattr(c, t)[0].copy_(src)
    for t in ("kst", "vst", "kmn", "vmn", "tail_k", "tail_v"):
        ref = getattr(caches[0], t)[0]
        src = (torch.rand(ref.shape, generator=gd, device="cuda") * (0.02 if t in ("kst", "vst") else 1.0)).half()
        if t in ("kmn", "vmn"):
            src = src - 2.5
        for c in caches:
            getattr(c, t)[0].copy_(src)
    q_out = torch.zeros(b, hq * D, dtype=torch.float16, device="cuda")
    q3 = q_out.view(b, hq, D)
    outs = [torch.zeros(b, hq, D, dtype=torch.float16, device="cuda") for _ in range(2)]
    completions = 0
    for pos in range(start, start + steps):
        qkv = (torch.randn(b, (hq + 2 * hkv) * D, generator=g) * 2).half().cuda()
        for c in caches:
            c.pos.fill_(pos)
        sep, fus = caches
        from nova_b200 import _lib

        qa = _qk_args(qkv, qn, kn, cos, sin, q_out, sep)
        _lib.check(_lib.lib().nova_qk_norm_rope_append(_lib.ctypes.byref(qa), _lib.stream_of()), "qk")
        _attend(sep, q3, outs[0].view(b, hq, D))
        _attend(fus, q3, outs[1].view(b, hq, D), qk=_qk_args(qkv, qn, kn, cos, sin, q_out, fus))
        torch.cuda.synchronize()
        for i, (x, y) in enumerate(zip(_state(sep), _state(fus))):
            np.testing.assert_array_equal(x, y, err_msg=f"state {i} at pos {pos}")
        st = assert_ulp_or_abs(outs[1].cpu().numpy(), outs[0].cpu().numpy(), 2.0, 1e-5, f"out pos={pos}")
        if max_len == 512:   # same split layout on both paths: every element within 2 ULP, or all within 1e-5
            assert st["max_ulp"] <= 2.0 or st["max_abs"] <= 1e-5
        completions += pos % 64 == 63
    assert completions >= 1


def test_fused_append_rejects_mismatched_cache(cuda_lib):
    from nova_b200 import _lib
    from nova_b200.kvattn import KVInt8Cache

    a = KVInt8Cache(num_slots=1, num_kv_heads=8, head_dim=D, max_len=256, num_q_heads=32, batch=1, chunk=64)
    other = KVInt8Cache(num_slots=1, num_kv_heads=8, head_dim=D, max_len=256, num_q_heads=32, batch=1, chunk=64)
    cos = torch.zeros(257, D, dtype=torch.float16, device="cuda")
    w = torch.ones(D, dtype=torch.float16, device="cuda")
    qkv = torch.zeros(1, 48 * D, dtype=torch.float16, device="cuda")
    q_out = torch.zeros(1, 32 * D, dtype=torch.float16, device="cuda")
    out = torch.zeros(1, 32, D, dtype=torch.float16, device="cuda")
    with pytest.raises(ValueError, match="same ring"):
        _attend(a, out, out, qk=_qk_args(qkv, w, w, cos, cos, q_out, other))
    qa = _qk_args(qkv, w, w, cos, cos, q_out, a)
    qa.qkv_stride = 16
    with pytest.raises(ValueError, match="qkv_stride"):
        _attend(a, out, out, qk=qa)
