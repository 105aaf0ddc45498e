"""GPU: fused int8-KV decode attention (nova_attn_decode_int8) against the CPU
oracle and the reference fixtures.  Criterion = the reference's own
(tests/test_kvattn.py:83-94): each element within 2 fp16 ULP or 1e-5 absolute
of "dequantize then fp32 attention"; the streaming cache within 4 ULP or 1e-3
(tests/test_kvattn_stream.py:38-41)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import assert_ulp_or_abs, golden
from oracle import attention as oatt
from oracle import kvquant as okv

pytestmark = pytest.mark.gpu

HQ, H_KV, D = 32, 8, 128


def _make(used, seed=0, outliers=False, b=1, hq=HQ, hkv=H_KV):
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(b, hkv, used, D, generator=g) * 0.7
    if outliers:
        k[..., [3, 71, 120]] *= 65.0
    v = torch.randn(b, hkv, used, D, generator=g) * 0.7
    q = torch.randn(b, hq, 1, D, generator=g) * 0.7
    return q.half(), k.half(), v.half()


def _oracle_fused(q, k, v, used, window=0):
    kq, kmn, kst = okv.quantize_int8_token(k.numpy(), 64)
    vq, vmn, vst = okv.quantize_int8_token(v.numpy(), 64)
    out, lse = oatt.fused_prefix_attend(q[:, :, 0].numpy(), kq, kmn, kst, vq, vmn, vst, used, window=window)
    return out, lse


@pytest.mark.parametrize("used", [7, 63, 64, 65, 511, 512, 513, 1024, 2049, 4096])
def test_fused_matches_oracle(cuda_lib, used):
    from nova_b200.kvattn import int8_attn_decode, pack_int8_kv

    q, k, v = _make(used)
    packed = pack_int8_kv(k.cuda(), v.cuda())
    lse = torch.empty(1, HQ, dtype=torch.float32, device="cuda")
    got = int8_attn_decode(q.cuda(), *packed, used=used, lse_out=lse)
    want, want_lse = _oracle_fused(q, k, v, used)
    st = assert_ulp_or_abs(got[:, :, 0].cpu().numpy(), want, 2.0, 1e-5, f"used={used}")
    assert st["max_ulp"] <= 2.0 or st["max_abs"] <= 1e-5
    np.testing.assert_allclose(lse.cpu().numpy(), want_lse, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("used", [7, 64, 65, 513, 1000])
def test_fused_matches_reference_fixture(cuda_lib, used):
    from nova_b200.kvattn import int8_attn_decode, pack_int8_kv

    g = golden("attention.npz")
    q = torch.from_numpy(g[f"fused{used}_q"]).cuda()
    packed = pack_int8_kv(torch.from_numpy(g[f"fused{used}_k"]).cuda(), torch.from_numpy(g[f"fused{used}_v"]).cuda())
    got = int8_attn_decode(q, *packed, used=used)
    assert_ulp_or_abs(got.cpu().numpy(), g[f"fused{used}_out"], 2.0, 1e-5, f"fixture used={used}")


@pytest.mark.parametrize("used", [300, 2049])
def test_channel_outliers(cuda_lib, used):
    from nova_b200.kvattn import int8_attn_decode, pack_int8_kv

    q, k, v = _make(used, seed=1, outliers=True)
    got = int8_attn_decode(q.cuda(), *pack_int8_kv(k.cuda(), v.cuda()), used=used)
    want, _ = _oracle_fused(q, k, v, used)
    assert_ulp_or_abs(got[:, :, 0].cpu().numpy(), want, 2.0, 1e-5, f"outliers used={used}")


@pytest.mark.parametrize("chunk", [64, 512, 4096])
def test_split_sizes_agree(cuda_lib, chunk):
    from nova_b200.kvattn import int8_attn_decode, pack_int8_kv

    used = 3000
    q, k, v = _make(used, seed=2)
    got = int8_attn_decode(q.cuda(), *pack_int8_kv(k.cuda(), v.cuda()), used=used, chunk=chunk)
    want, _ = _oracle_fused(q, k, v, used)
    assert_ulp_or_abs(got[:, :, 0].cpu().numpy(), want, 2.0, 1e-5, f"chunk={chunk}")


def test_gqa_head_mapping(cuda_lib):
    """V constant per KV head: query head h must return the constant of KV head h // 4."""
    from nova_b200.kvattn import int8_attn_decode, pack_int8_kv

    used = 256
    q, k, _ = _make(used, seed=3)
    v = torch.arange(H_KV, dtype=torch.float16).view(1, H_KV, 1, 1).expand(1, H_KV, used, D).contiguous()
    got = int8_attn_decode(q.cuda(), *pack_int8_kv(k.cuda(), v.cuda()), used=used)
    want = (torch.arange(HQ) // (HQ // H_KV)).half().view(1, HQ, 1, 1).expand(1, HQ, 1, D)
    assert torch.equal(got.cpu(), want)


def test_garbage_after_used_is_ignored(cuda_lib):
    from nova_b200.kvattn import int8_attn_decode, pack_int8_kv

    used, length = 333, 512
    q, k, v = _make(length, seed=4)
    kq, kmn, kst, vq, vmn, vst = pack_int8_kv(k.cuda(), v.cuda())
    a = int8_attn_decode(q.cuda(), kq, kmn, kst, vq, vmn, vst, used=used)
    kq2, vq2 = kq.clone(), vq.clone()
    kq2[:, :, used:] = 255
    vq2[:, :, used:] = 7
    kst2 = kst.clone()
    kst2[:, :, used // 64 + 1:] = float("nan")
    b = int8_attn_decode(q.cuda(), kq2, kmn, kst2, vq2, vmn, vst, used=used)
    assert torch.equal(a, b)


def test_used_zero_gives_zeros(cuda_lib):
    from nova_b200.kvattn import int8_attn_decode, pack_int8_kv

    q, k, v = _make(64)
    lse = torch.empty(1, HQ, dtype=torch.float32, device="cuda")
    out = int8_attn_decode(q.cuda(), *pack_int8_kv(k.cuda(), v.cuda()), used=0, lse_out=lse)
    assert torch.count_nonzero(out).item() == 0
    assert torch.isinf(lse).all() and (lse < 0).all()


def test_device_scalars_match_python_ints_and_extra_splits(cuda_lib):
    from nova_b200.kvattn import int8_attn_decode, new_workspace, pack_int8_kv

    used, length = 320, 1024
    q, k, v = _make(length, seed=5)
    packed = pack_int8_kv(k.cuda(), v.cuda())
    a = int8_attn_decode(q.cuda(), *packed, used=used, prefix_groups=used // 64)
    used_t = torch.tensor([used], dtype=torch.int64, device="cuda")
    pg_t = torch.tensor([used // 64], dtype=torch.int64, device="cuda")
    n_splits = 8   # grid sized for the full 1024-token capacity; most splits are empty
    ws = new_workspace(1, HQ, H_KV, n_splits, False)
    out = torch.zeros(1, HQ, 1, D, dtype=torch.float16, device="cuda")
    b = int8_attn_decode(q.cuda(), *packed, used_t=used_t, prefix_groups_t=pg_t, n_splits=n_splits, scratch=ws,
                         out=out)
    assert torch.isfinite(b).all()
    want, _ = _oracle_fused(q[:, :, :, :], k[:, :, :used], v[:, :, :used], used)
    assert_ulp_or_abs(b[:, :, 0].cpu().numpy(), want, 2.0, 1e-5, "device scalars")
    # only the order of the fp32 merge differs: tiny, and bit-identical here for equal split counts
    c = int8_attn_decode(q.cuda(), *packed, used=used, prefix_groups=used // 64, n_splits=n_splits)
    assert torch.equal(b, c)
    assert_ulp_or_abs(a.cpu().numpy(), b.cpu().numpy(), 1.0, 1e-5, "python vs device scalars")


def test_cuda_graph_replay_is_bit_identical(cuda_lib):
    from nova_b200.kvattn import int8_attn_decode, new_workspace, pack_int8_kv

    used, length = 1500, 2048
    q, k, v = _make(length, seed=6)
    packed = pack_int8_kv(k.cuda(), v.cuda())
    qd = q.cuda()
    used_t = torch.tensor([used], dtype=torch.int64, device="cuda")
    pg_t = torch.tensor([-(-used // 64)], dtype=torch.int64, device="cuda")
    n_splits = 4
    ws = new_workspace(1, HQ, H_KV, n_splits, False)
    out = torch.zeros(1, HQ, 1, D, dtype=torch.float16, device="cuda")
    eager = int8_attn_decode(qd, *packed, used_t=used_t, prefix_groups_t=pg_t, n_splits=n_splits, scratch=ws,
                             out=out).clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        int8_attn_decode(qd, *packed, used_t=used_t, prefix_groups_t=pg_t, n_splits=n_splits, scratch=ws, out=out)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        int8_attn_decode(qd, *packed, used_t=used_t, prefix_groups_t=pg_t, n_splits=n_splits, scratch=ws, out=out)
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    # the graph reads the length on the device: grow it and replay again
    used_t.fill_(2000)
    pg_t.fill_(-(-2000 // 64))
    graph.replay()
    torch.cuda.synchronize()
    want, _ = _oracle_fused(q, k, v, 2000)   # quantized over the full 2048, attend [0, 2000)
    assert_ulp_or_abs(out[:, :, 0].cpu().numpy(), want, 2.0, 1e-5, "graph after growth")
    del graph


def test_rejects_bad_inputs(cuda_lib):
    from nova_b200.kvattn import int8_attn_decode, pack_int8_kv

    q, k, v = _make(128)
    packed = pack_int8_kv(k.cuda(), v.cuda())
    with pytest.raises(ValueError):
        int8_attn_decode(q.cuda().float(), *packed)                      # dtype
    with pytest.raises(ValueError):
        int8_attn_decode(q.cuda()[:, :30], *packed)                      # heads not divisible
    with pytest.raises(ValueError):
        int8_attn_decode(q.cuda(), *packed, used=129)                    # used > L
    with pytest.raises(ValueError):
        int8_attn_decode(q.cuda(), *packed, chunk=100)                   # chunk % group
    with pytest.raises(ValueError):
        int8_attn_decode(q.cuda(), *packed, group=32)                    # group != 64
    with pytest.raises(ValueError):
        int8_attn_decode(q.cuda()[:, :16], *[t[:, :2] for t in packed])  # 8 q heads per KV head > 4
    with pytest.raises(ValueError):
        int8_attn_decode(q, *packed)                                     # CPU tensor


@pytest.mark.parametrize("window,used", [(100, 1000), (4096, 6000), (64, 64)])
def test_sliding_window_matches_oracle(cuda_lib, window, used):
    from nova_b200.kvattn import int8_attn_decode, pack_int8_kv

    q, k, v = _make(used, seed=7)
    got = int8_attn_decode(q.cuda(), *pack_int8_kv(k.cuda(), v.cuda()), used=used, window=window)
    want, _ = _oracle_fused(q, k, v, used, window=window)
    assert_ulp_or_abs(got[:, :, 0].cpu().numpy(), want, 2.0, 1e-5, f"window={window}")


def test_batch_rows_are_independent(cuda_lib):
    from nova_b200.kvattn import int8_attn_decode, pack_int8_kv

    used, b = 777, 4
    q, k, v = _make(used, seed=8, b=b)
    got = int8_attn_decode(q.cuda(), *pack_int8_kv(k.cuda(), v.cuda()), used=used)
    want, _ = _oracle_fused(q, k, v, used)
    assert_ulp_or_abs(got[:, :, 0].cpu().numpy(), want, 2.0, 1e-5, "batch")


def test_long_context_32k(cuda_lib):
    from nova_b200.kvattn import int8_attn_decode, pack_int8_kv

    used = 32768
    q, k, v = _make(used, seed=9, hq=8, hkv=2)
    got = int8_attn_decode(q.cuda(), *pack_int8_kv(k.cuda(), v.cuda()), used=used, chunk=1024)
    want, _ = _oracle_fused(q, k, v, used)
    assert_ulp_or_abs(got[:, :, 0].cpu().numpy(), want, 2.0, 1e-5, "32k")


# ---------------------------------------------------------------- streaming cache (prefix + ring)


def _cache_step(k, v, q, chunk_prefill=0, window=0):
    """Prefill L-1 tokens, decode the L-th (tests/test_kvattn_stream.py:61-83)."""
    from nova_b200.kvattn import KVInt8Cache

    b, hkv, L, _ = k.shape
    cache = KVInt8Cache(num_slots=1, num_kv_heads=hkv, head_dim=D, max_len=max(512, L + 64), num_q_heads=q.shape[1],
                        batch=b, window=window)
    kd, vd = k.cuda(), v.cuda()
    n0 = L - 1
    if n0 == 0:   # nothing to prefill: decode straight into an empty cache
        cache.pos.fill_(0)
        cache.update(kd[:, :, :1], vd[:, :, :1], 0)
        return cache, cache.attend(q.cuda(), 0)
    cache.begin_prefill(n0)
    if chunk_prefill:
        for c0 in range(0, n0, chunk_prefill):
            nc = min(chunk_prefill, n0 - c0)
            cache.set_prefill_pos(c0)
            cache.update(kd[:, :, c0:c0 + nc], vd[:, :, c0:c0 + nc], 0)
    else:
        cache.set_prefill_pos(0)
        cache.update(kd[:, :, :n0], vd[:, :, :n0], 0)
    cache.finish_prefill(n0)
    cache.pos.fill_(L - 1)
    cache.update(kd[:, :, L - 1:], vd[:, :, L - 1:], 0)
    return cache, cache.attend(q.cuda(), 0)


def _oracle_stream(cache, q, window=0):
    written = int(cache._written.item())
    qlen = int(cache._qlen.item())
    arr = lambda t: t.cpu().numpy()  # noqa: E731
    return oatt.streaming_attend(q[:, :, 0].numpy(), arr(cache.kq[0]), arr(cache.kmn[0]), arr(cache.kst[0]),
                                 arr(cache.vq[0]), arr(cache.vmn[0]), arr(cache.vst[0]), arr(cache.tail_k[0]),
                                 arr(cache.tail_v[0]), written=written, qlen=qlen, window=window)


@pytest.mark.parametrize("used", [1, 33, 40, 64, 100, 128, 192, 320, 4100])
def test_streaming_cache_matches_oracle(cuda_lib, used):
    q, k, v = _make(used, seed=10)
    cache, got = _cache_step(k, v, q)
    assert int(cache._qlen.item()) == used // 64 * 64
    want, _ = _oracle_stream(cache, q)
    assert torch.isfinite(got).all()
    assert_ulp_or_abs(got[:, :, 0].cpu().numpy(), want, 2.0, 1e-5, f"stream used={used}")


@pytest.mark.parametrize("used", [40, 100, 320])
def test_streaming_cache_matches_reference_fixture(cuda_lib, used):
    g = golden("attention.npz")
    q = torch.from_numpy(g[f"stream{used}_q"])
    k, v = torch.from_numpy(g[f"stream{used}_k"]), torch.from_numpy(g[f"stream{used}_v"])
    _, got = _cache_step(k, v, q)
    assert_ulp_or_abs(got.cpu().numpy(), g[f"stream{used}_out"], 4.0, 1e-3, f"fixture stream used={used}")


@pytest.mark.parametrize("chunk", [64, 96, 128])
def test_chunked_prefill_equals_single(cuda_lib, chunk):
    q, k, v = _make(300, seed=11)
    _, one = _cache_step(k, v, q)
    _, many = _cache_step(k, v, q, chunk_prefill=chunk)
    assert torch.equal(one, many)


def test_streaming_window_and_batch(cuda_lib):
    q, k, v = _make(1000, seed=12, b=2)
    cache, got = _cache_step(k, v, q, window=300)
    want, _ = _oracle_stream(cache, q, window=300)
    assert_ulp_or_abs(got[:, :, 0].cpu().numpy(), want, 2.0, 1e-5, "stream window batch")


def test_tail_attend_alone(cuda_lib):
    """Ring-only attention with its LSE (the reference's tail_attend)."""
    from nova_b200.kvattn import tail_attend

    q, k, v = _make(64, seed=13)
    written, qlen = torch.tensor([200], device="cuda"), torch.tensor([192], device="cuda")
    out, lse = tail_attend(q.cuda(), k.cuda(), v.cuda(), written, qlen)
    pos = oatt.ring_positions(200)
    valid = (pos >= 192) & (pos <= 199)
    want, want_lse = oatt.attend(q[:, :, 0].numpy(), k.numpy(), v.numpy(), valid)
    assert_ulp_or_abs(out[:, :, 0].cpu().numpy(), want, 2.0, 1e-5, "tail")
    np.testing.assert_allclose(lse.cpu().numpy(), want_lse, rtol=1e-5, atol=1e-5)


def test_streaming_graph_capture_bit_identical(cuda_lib):
    q, k, v = _make(700, seed=14)
    cache, eager = _cache_step(k, v, q)
    eager = eager.clone()
    qd = q.cuda()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        cache.attend(qd, 0)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = cache.attend(qd, 0)
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    del graph


# ---------------------------------------------------------------- BASELINE configs 1 and 3 at full size


@pytest.mark.parametrize("ctx,batch,window", [(131072, 1, 0), (32768, 16, 0), (32768, 4, 4096)])
def test_config3_full_size_matches_oracle(cuda_lib, ctx, batch, window):
    """BASELINE config 3 shapes (32 q / 8 KV heads, the decoder's split size for
    that capacity): full-causal decode at ctx 131072 (batch 1) and 32768
    (batch 16), and the sliding window of 4096 at ctx 32768 (batch 4).  K/V are
    N(0, 0.7) fp16 quantized on the GPU (nova_kv_quant_int8, bit-exact with the
    reference quantizer); the oracle dequantizes the same codes and attends in
    fp32, one batch row at a time."""
    from nova_b200.kvattn import int8_attn_decode, pack_int8_kv, pick_chunk

    g = torch.Generator(device="cuda").manual_seed(ctx + batch + window)
    k = (torch.randn(batch, H_KV, ctx, D, generator=g, device="cuda") * 0.7).half()
    v = (torch.randn(batch, H_KV, ctx, D, generator=g, device="cuda") * 0.7).half()
    q = (torch.randn(batch, HQ, 1, D, generator=g, device="cuda") * 0.7).half()
    packed = pack_int8_kv(k, v)
    del k, v
    chunk = pick_chunk(ctx, batch, H_KV, HQ, torch.cuda.get_device_properties(0).multi_processor_count)
    got = int8_attn_decode(q, *packed, used=ctx, chunk=chunk, window=window)[:, :, 0].cpu().numpy()
    qh = q[:, :, 0].cpu().numpy()
    for b in range(batch):
        host = [t[b:b + 1].cpu().numpy() for t in packed]
        want, _ = oatt.fused_prefix_attend(qh[b:b + 1], *host, ctx, window=window)
        assert_ulp_or_abs(got[b:b + 1], want, 2.0, 1e-5, f"ctx={ctx} batch row {b} window={window}")


def test_config1_append_and_attend_through_the_cache(cuda_lib):
    """BASELINE config 1 exactly: one layer, batch 1, 32 q / 8 KV heads,
    ctx 4096, q/K/V N(0, 1) fp16, through KVInt8Cache (prefill of 4095 tokens,
    then the decode append of token 4096, which completes group 63 and
    requantizes it, then attend).  The appended group's codes and scales are
    bit-exact with the token-axis quantizer over those 64 tokens, and the
    output is within the reference's attention criterion."""
    g = torch.Generator().manual_seed(4096)
    k = torch.randn(1, H_KV, 4096, D, generator=g).half()
    v = torch.randn(1, H_KV, 4096, D, generator=g).half()
    q = torch.randn(1, HQ, 1, D, generator=g).half()
    cache, got = _cache_step(k, v, q)
    assert int(cache._qlen.item()) == 4096 and int(cache._written.item()) == 4096
    kq, kmn, kst = okv.quantize_int8_token(k[:, :, 4032:].numpy(), 64)
    vq, vmn, vst = okv.quantize_int8_token(v[:, :, 4032:].numpy(), 64)
    np.testing.assert_array_equal(cache.kq[0][:, :, 4032:4096].cpu().numpy(), kq)
    np.testing.assert_array_equal(cache.vq[0][:, :, 4032:4096].cpu().numpy(), vq)
    for have, want in ((cache.kmn[0][:, :, 63:64], kmn), (cache.kst[0][:, :, 63:64], kst),
                       (cache.vmn[0][:, :, 63:64], vmn), (cache.vst[0][:, :, 63:64], vst)):
        np.testing.assert_array_equal(have.cpu().numpy().view(np.uint16), want.view(np.uint16))
    want, _ = _oracle_stream(cache, q)
    assert_ulp_or_abs(got[:, :, 0].cpu().numpy(), want, 2.0, 1e-5, "config 1")
