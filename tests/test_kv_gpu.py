"""GPU: int8 KV quantizer and the streaming-cache append path against the
oracle and the reference fixtures -- bit-exact (codes, fp16 scales, ring)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import kvquant as okv

pytestmark = pytest.mark.gpu

D = 128


def _t(a, dev="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.mark.parametrize("case", ["rand", "outlier", "const"])
def test_quantize_matches_reference_fixture(cuda_lib, case):
    from nova_b200.kvquant import dequantize_int8, quantize_int8

    g = golden("kvquant_token.npz")
    q, mn, st = quantize_int8(_t(g[f"{case}_x"]), 64, "token")
    np.testing.assert_array_equal(q.cpu().numpy(), g[f"{case}_q"])
    np.testing.assert_array_equal(mn.cpu().numpy().view(np.uint16), g[f"{case}_mn"].view(np.uint16))
    np.testing.assert_array_equal(st.cpu().numpy().view(np.uint16), g[f"{case}_st"].view(np.uint16))
    deq = dequantize_int8(q, mn, st, 64, "token")
    np.testing.assert_array_equal(deq.cpu().numpy().view(np.uint16), g[f"{case}_deq"].view(np.uint16))


@pytest.mark.parametrize("n", [1, 63, 64, 65, 200, 4097])
def test_quantize_ragged_lengths_match_oracle(cuda_lib, n):
    torch.manual_seed(n)
    x = (torch.randn(2, 3, n, D) * 2.5).to(torch.float16)
    from nova_b200.kvquant import quantize_int8

    q, mn, st = quantize_int8(x.cuda(), 64, "token")
    oq, omn, ost = okv.quantize_int8_token(x.numpy(), 64)
    np.testing.assert_array_equal(q.cpu().numpy(), oq)
    np.testing.assert_array_equal(mn.cpu().numpy().view(np.uint16), omn.view(np.uint16))
    np.testing.assert_array_equal(st.cpu().numpy().view(np.uint16), ost.view(np.uint16))


def test_quantize_rejects_channel_axis_and_cpu(cuda_lib):
    from nova_b200.kvquant import quantize_int8

    x = torch.zeros(1, 1, 64, D, dtype=torch.float16)
    with pytest.raises(ValueError):
        quantize_int8(x.cuda(), 32, "channel")
    with pytest.raises(ValueError):
        quantize_int8(x, 64, "token")


def test_cache_prefill_and_decode_match_reference_cache(cuda_lib):
    """Same inputs as the reference KVInt8Cache fixture (100 prefill tokens +
    100 decode updates, 2 layers): finalized codes/scales, ring and scalars are
    bit-identical."""
    from nova_b200.kvattn import KVInt8Cache

    g = golden("kv_ring.npz")
    n0, steps, max_len = int(g["n0"]), int(g["steps"]), int(g["max_len"])
    cache = KVInt8Cache(num_slots=2, num_kv_heads=2, head_dim=D, max_len=max_len, num_q_heads=8)
    k, v = _t(g["k"]), _t(g["v"])
    cache.begin_prefill(n0)
    cache.set_prefill_pos(0)
    for layer in range(2):
        cache.update(k[layer, :, :, :n0], v[layer, :, :, :n0], layer)
    cache.finish_prefill(n0)
    for p in range(n0, n0 + steps):
        cache.pos.fill_(p)
        for layer in range(2):
            cache.update(k[layer, :, :, p:p + 1], v[layer, :, :, p:p + 1], layer)
    qlen = int(g["qlen"])
    assert int(cache._qlen.item()) == qlen
    assert int(cache._written.item()) == int(g["written"])
    assert int(cache._pg.item()) == int(g["pg"])
    for layer in range(2):
        np.testing.assert_array_equal(cache.kq[layer][:, :, :qlen].cpu().numpy(), g[f"kq{layer}"])
        np.testing.assert_array_equal(cache.vq[layer][:, :, :qlen].cpu().numpy(), g[f"vq{layer}"])
        for nm in ("kmn", "kst", "vmn", "vst"):
            got = getattr(cache, nm)[layer][:, :, :qlen // 64].cpu().numpy()
            np.testing.assert_array_equal(got.view(np.uint16), g[f"{nm}{layer}"].view(np.uint16))
        np.testing.assert_array_equal(cache.tail_k[layer].cpu().numpy().view(np.uint16),
                                      g[f"tail_k{layer}"].view(np.uint16))
        np.testing.assert_array_equal(cache.tail_v[layer].cpu().numpy().view(np.uint16),
                                      g[f"tail_v{layer}"].view(np.uint16))
    np.testing.assert_array_equal(cache.ring_mask().view(-1).cpu().numpy(), g["ring_mask"])


def test_prefix_grows_only_at_group_boundaries(cuda_lib):
    from nova_b200.kvattn import KVInt8Cache

    torch.manual_seed(0)
    k = (torch.randn(1, 8, 200, D) * 0.7).to(torch.float16).cuda()
    v = (torch.randn(1, 8, 200, D) * 0.7).to(torch.float16).cuda()
    cache = KVInt8Cache(num_slots=1, num_kv_heads=8, head_dim=D, max_len=256, num_q_heads=32)
    cache.begin_prefill(63)
    cache.set_prefill_pos(0)
    cache.update(k[:, :, :63], v[:, :, :63], 0)
    cache.finish_prefill(63)
    assert int(cache._qlen.item()) == 0
    for p in range(63, 200):
        cache.pos.fill_(p)
        cache.update(k[:, :, p:p + 1], v[:, :, p:p + 1], 0)
        assert int(cache._qlen.item()) == (p + 1) // 64 * 64
        assert int(cache._written.item()) == p + 1
    q = (200 // 64) * 64
    oq, _, _ = okv.quantize_int8_token(k[:, :, :q].cpu().numpy(), 64)
    np.testing.assert_array_equal(cache.kq[0][:, :, :q].cpu().numpy(), oq)


def test_append_ignores_positions_past_capacity(cuda_lib):
    from nova_b200.kvattn import KVInt8Cache

    cache = KVInt8Cache(num_slots=1, num_kv_heads=2, head_dim=D, max_len=128, num_q_heads=8)
    before = [t.clone() for t in (cache.kq[0], cache.tail_k[0])]
    cache.pos.fill_(128)
    k = torch.ones(1, 2, 1, D, dtype=torch.float16, device="cuda")
    cache.update(k, k, 0)
    torch.cuda.synchronize()
    assert torch.equal(before[0], cache.kq[0]) and torch.equal(before[1], cache.tail_k[0])
    assert int(cache._written.item()) == 129
