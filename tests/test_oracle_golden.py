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


# ---------------------------------------------------------------- decoder

def _decoder_fixture():
    """The fixture, the seeded weights it was made with and an oracle decoder."""
    from oracle.decoder import OracleDecoder, random_weights

    g = golden("decoder.npz")
    vocab, hidden, layers, hq, hkv, inter = (int(x) for x in g["dims"])
    W = random_weights(vocab=vocab, hidden=hidden, layers=layers, q_heads=hq, kv_heads=hkv, inter=inter,
                       seed=int(g["seed"]))
    return g, lambda: OracleDecoder(W, hidden=hidden, q_heads=hq, kv_heads=hkv, max_len=int(g["max_len"]))


def _load_reference_state(orc, g) -> None:
    """Seed the oracle with the reference cache as its prefill left it."""
    T, L = len(g["prompt"]), orc.max_len
    q = T // 64 * 64
    st = {"pos": T}
    for name in ("kq", "vq", "kmn", "kst", "vmn", "vst", "tail_k", "tail_v"):
        st[name] = []
        for li in range(len(orc.W["layers"])):
            a = g[f"state_{name}{li}"]
            if name in ("kq", "vq"):
                full = np.zeros(a.shape[:2] + (L, a.shape[3]), a.dtype)
                full[:, :, :q] = a
            elif name in ("kmn", "kst", "vmn", "vst"):
                full = np.zeros(a.shape[:2] + (-(-L // 64), a.shape[3]), a.dtype)
                full[:, :, :q // 64] = a
            else:
                full = a.copy()
            st[name].append(full)
    orc.load_state(st)


def _check_steps(got_logits, want_logits, got_tokens, want_tokens, max_frac, mean_frac, what):
    """Per step: logits within max_frac (max) / mean_frac (mean) of the
    logit range; tokens equal unless the reference's own top-2 margin is
    within twice the observed logit error (a genuine near-tie)."""
    for i in range(len(want_tokens)):
        want = want_logits[i].astype(np.float32)
        got = got_logits[i].astype(np.float32)
        scale = float(np.abs(want).max())
        d = np.abs(got - want)
        assert d.max() <= max_frac * scale and d.mean() <= mean_frac * scale, \
            f"{what} step {i}: logits differ by max {d.max():.3e} mean {d.mean():.3e} (range {scale:.3f})"
        if got_tokens[i] != want_tokens[i]:
            top2 = np.sort(want)[-2:]
            assert top2[1] - top2[0] <= 2 * d.max(), f"{what} step {i}: token differs without a near-tie"


def test_decoder_matches_reference_graph_decoder():
    """The oracle decoder (oracle/decoder.py) against the reference's own int8
    greedy decode (GraphDecoder prefill + _body steps over NovaTextModel on a
    random-init Qwen3-VL text model at real widths, 2 layers; fixture from
    tests/golden/make_golden.py).  (1) prefill: last-position logits and first
    token; (2) 72 decode steps from the reference's own post-prefill cache,
    fed the reference's tokens: per-step logits and greedy tokens; (3) the
    same steps after the oracle's own prefill."""
    g, make = _decoder_fixture()
    tokens = g["tokens"]
    orc = make()
    plog, ptok = orc.prefill(g["prompt"][None])
    want = g["prefill_logits"].astype(np.float32)
    assert np.abs(plog[0].astype(np.float32) - want).max() <= 4e-3 * np.abs(want).max()
    assert int(ptok[0]) == int(tokens[0])
    lg, tk = orc.decode_teacher_forced(tokens[:-1, None])
    _check_steps(lg[:, 0], g["logits"], tk[:, 0], tokens[1:], 3e-3, 5e-4, "after the oracle's prefill")
    orc = make()
    _load_reference_state(orc, g)
    lg, tk = orc.decode_teacher_forced(tokens[:-1, None])
    _check_steps(lg[:, 0], g["logits"], tk[:, 0], tokens[1:], 2.5e-3, 4e-4, "from the reference's cache")
    assert np.array_equal(tk[:, 0], tokens[1:]), "greedy tokens differ from the reference's"


def test_decoder_batched_steps_equal_single_steps():
    """decode_teacher_forced (all steps per layer at once) against step() called
    once per token, on a small model across two group boundaries."""
    import copy

    from oracle.decoder import OracleDecoder, random_weights

    W = random_weights(vocab=512, hidden=256, layers=2, q_heads=8, kv_heads=2, inter=512, seed=3)
    a = OracleDecoder(W, hidden=256, q_heads=8, kv_heads=2, max_len=320, batch=2)
    _, first = a.prefill(np.random.default_rng(1).integers(0, 512, (2, 100)))
    b = copy.deepcopy(a)
    toks, logs = [first], []
    for _ in range(90):
        lg, t = a.step(toks[-1])
        logs.append(lg)
        toks.append(t)
    lb, tb = b.decode_teacher_forced(np.stack(toks[:-1]))
    la = np.stack(logs).astype(np.float32)
    assert np.abs(la - lb.astype(np.float32)).max() <= 2e-3 * np.abs(la).max()
    assert np.array_equal(np.stack(toks[1:]), tb)
    assert a.pos == b.pos == 190
    for li in range(2):   # the groups completed during the steps agree to within one code
        d = np.abs(a.kq[li][:, :, :128].astype(int) - b.kq[li][:, :, :128].astype(int))
        assert d.max() <= 1
