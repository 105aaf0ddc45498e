"""CPU: the oracle against the golden fixtures generated from the reference's
own code (tests/golden/make_golden.py).  Integer / byte outputs must match
bit for bit; attention uses the reference's own ULP criterion."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_ulp_or_abs, golden
from oracle import attention as oatt
from oracle import kvquant as okv
from oracle import nf4 as onf4
from oracle import norm as onorm


@pytest.mark.parametrize("case", ["rand", "outlier", "const"])
def test_quantize_int8_token_bit_exact(case):
    g = golden("kvquant_token.npz")
    q, mn, st = okv.quantize_int8_token(g[f"{case}_x"], 64)
    np.testing.assert_array_equal(q, g[f"{case}_q"])
    np.testing.assert_array_equal(mn.view(np.uint16), g[f"{case}_mn"].view(np.uint16))
    np.testing.assert_array_equal(st.view(np.uint16), g[f"{case}_st"].view(np.uint16))
    deq = okv.dequantize_int8_token(q, mn, st, 64)
    np.testing.assert_array_equal(deq.view(np.uint16), g[f"{case}_deq"].view(np.uint16))


def test_ring_requantization_matches_reference_cache():
    """Prefill of 100 tokens + 100 decode updates through the reference
    KVInt8Cache: the oracle's group/ring arithmetic reproduces every finalized
    byte, the ring contents and the scalars."""
    g = golden("kv_ring.npz")
    n0, steps = int(g["n0"]), int(g["steps"])
    total = n0 + steps
    qlen = total // 64 * 64
    assert int(g["qlen"]) == qlen and int(g["written"]) == total and int(g["pg"]) == qlen // 64
    for layer in range(2):
        k, v = g["k"][layer], g["v"][layer]
        # every finalized group equals the token-axis quantizer over those tokens
        kq, kmn, kst = okv.quantize_int8_token(k[:, :, :qlen], 64)
        vq, vmn, vst = okv.quantize_int8_token(v[:, :, :qlen], 64)
        np.testing.assert_array_equal(kq, g[f"kq{layer}"])
        np.testing.assert_array_equal(vq, g[f"vq{layer}"])
        for a, nm in ((kmn, "kmn"), (kst, "kst"), (vmn, "vmn"), (vst, "vst")):
            np.testing.assert_array_equal(a.view(np.uint16), g[f"{nm}{layer}"].view(np.uint16))
        # the last group completed during decode also equals quantize_ring of its 64 tokens
        last = qlen - 64
        rq, rmn, rst = okv.quantize_ring(k[:, :, last:qlen])
        np.testing.assert_array_equal(rq, g[f"kq{layer}"][:, :, last:qlen])
        np.testing.assert_array_equal(rmn.view(np.uint16), g[f"kmn{layer}"][:, :, -1].view(np.uint16))
        # ring: slot p % 64 holds the newest token at position p
        pos = oatt.ring_positions(total)
        valid = pos >= 0
        np.testing.assert_array_equal(g[f"tail_k{layer}"][:, :, valid], k[:, :, pos[valid]])
    mask = (oatt.ring_positions(total) >= qlen) & (oatt.ring_positions(total) <= total - 1)
    np.testing.assert_array_equal(mask, g["ring_mask"])


@pytest.mark.parametrize("used", [7, 64, 65, 513, 1000])
def test_fused_prefix_attention_matches_reference(used):
    g = golden("attention.npz")
    q, k, v = g[f"fused{used}_q"], g[f"fused{used}_k"], g[f"fused{used}_v"]
    kq, kmn, kst = okv.quantize_int8_token(k, 64)
    vq, vmn, vst = okv.quantize_int8_token(v, 64)
    out, lse = oatt.fused_prefix_attend(q[:, :, 0], kq, kmn, kst, vq, vmn, vst, used)
    assert_ulp_or_abs(out, g[f"fused{used}_out"][:, :, 0], 2.0, 1e-5, f"used={used}")


@pytest.mark.parametrize("used", [40, 100, 320])
def test_streaming_attention_matches_reference(used):
    """int8 prefix + fp16 ring through the oracle's cache-state form equals the
    reference's single-SDPA ground truth (tests/test_kvattn_stream.py:68-83)."""
    g = golden("attention.npz")
    q, k, v = g[f"stream{used}_q"], g[f"stream{used}_k"], g[f"stream{used}_v"]
    prefix = used // 64 * 64
    max_len = 384
    b, h, _, d = k.shape
    kq = np.zeros((b, h, max_len, d), np.uint8)
    vq = np.zeros_like(kq)
    ng = max_len // 64
    kmn, kst, vmn, vst = (np.zeros((b, h, ng, d), np.float16) for _ in range(4))
    if prefix:
        a = okv.quantize_int8_token(k[:, :, :prefix], 64)
        c = okv.quantize_int8_token(v[:, :, :prefix], 64)
        kq[:, :, :prefix], kmn[:, :, :prefix // 64], kst[:, :, :prefix // 64] = a
        vq[:, :, :prefix], vmn[:, :, :prefix // 64], vst[:, :, :prefix // 64] = c
    tail_k = np.zeros((b, h, 64, d), np.float16)
    tail_v = np.zeros_like(tail_k)
    for p in range(max(0, used - 64), used):
        tail_k[:, :, p % 64] = k[:, :, p]
        tail_v[:, :, p % 64] = v[:, :, p]
    out, _ = oatt.streaming_attend(q[:, :, 0], kq, kmn, kst, vq, vmn, vst, tail_k, tail_v, written=used,
                                   qlen=prefix)
    assert_ulp_or_abs(out, g[f"stream{used}_out"][:, :, 0], 2.0, 1e-5, f"used={used}")


def test_nf4_lut_and_layout_match_reference():
    g = golden("nf4.npz")
    code = onf4.nf4_codebook()
    np.testing.assert_array_equal(code, g["code"])
    np.testing.assert_array_equal(onf4.build_nf4_lut(code), g["lut"])
    packed, absmax = onf4.quantize_nf4(g["w"], code, absmax_dtype=np.float32)
    np.testing.assert_array_equal(packed, g["packed"])
    np.testing.assert_array_equal(absmax, g["absmax"])
    deq16 = onf4.dequantize_nf4(packed, absmax, code, round_fp16=True, code_fp16=False)
    np.testing.assert_array_equal(deq16.view(np.uint16), g["deq16"].view(np.uint16))


def test_nf4_codebook_matches_published_levels():
    """The QLoRA paper's NF4 levels (Dettmers et al. 2023, Appendix E)."""
    published = np.array([-1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
                          -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
                          0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
                          0.44070982933044556, 0.5626170039176941, 0.7229568362236023, 1.0], np.float32)
    code = onf4.nf4_codebook()
    np.testing.assert_allclose(code, published, rtol=0, atol=2e-7)
    np.testing.assert_array_equal(code.astype(np.float16), published.astype(np.float16))


def test_nf4_quantizer_roundtrip_properties():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((64, 512)) * 0.02).astype(np.float16)
    code = onf4.nf4_codebook()
    packed, absmax = onf4.quantize_nf4(w, code)
    deq = onf4.dequantize_nf4(packed, absmax, code)
    # nearest level: error at most half the widest gap between levels, times absmax
    gap = np.diff(code).max() / 2
    am = np.repeat(absmax.astype(np.float32).T, 64, axis=1)
    assert np.all(np.abs(deq - w.astype(np.float32)) <= gap * am * 1.001 + 1e-6)
    # the absmax element of every block is reproduced up to the fp16 absmax rounding
    wb = np.abs(w.astype(np.float32)).reshape(64, 8, 64)
    i = wb.argmax(-1)
    got = np.abs(deq.reshape(64, 8, 64))[np.arange(64)[:, None], np.arange(8)[None, :], i]
    np.testing.assert_allclose(got, wb.max(-1), rtol=2 ** -10)


@pytest.mark.parametrize("dim", [2560, 128])
def test_rmsnorm_matches_reference_exact(dim):
    g = golden("norm_rope.npz")
    y = onorm.rms_norm(g[f"norm{dim}_x"], g[f"norm{dim}_w"], 1e-6)
    np.testing.assert_array_equal(y.view(np.uint16), g[f"norm{dim}_y"].view(np.uint16))


def test_rope_matches_reference():
    g = golden("norm_rope.npz")
    cos, sin = onorm.rope_cos_sin(g["rope_pos"])
    np.testing.assert_array_equal(cos.view(np.uint16), g["rope_cos"].view(np.uint16))
    np.testing.assert_array_equal(sin.view(np.uint16), g["rope_sin"].view(np.uint16))
    qe = onorm.apply_rope(g["rope_q"], cos[None, None], sin[None, None])
    ke = onorm.apply_rope(g["rope_k"], cos[None, None], sin[None, None])
    np.testing.assert_array_equal(qe.view(np.uint16), g["rope_qe"].view(np.uint16))
    np.testing.assert_array_equal(ke.view(np.uint16), g["rope_ke"].view(np.uint16))
