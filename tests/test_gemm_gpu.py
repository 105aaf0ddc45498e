"""GPU: batched NF4 GEMM (nova_nf4_gemm on the tcgen05 tensor cores, M up to
64, units from pack_tc) against the CPU oracle.

The GEMM computes x @ dequant(W)^T as the reference kernel does: fp16
codebook values times x summed in fp32 per 64-element block, times the block's
absmax, accumulated in fp32.  Each fp16 output must be within 1 fp16 ULP of the
oracle's fp32 result or within 1e-5 * max|y| absolute (the sums are ordered
differently), and within the north-star bound of 1e-2 relative."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import assert_ulp_or_abs, fp16_ulp
from oracle import nf4 as onf4
from oracle import norm as onorm

pytestmark = pytest.mark.gpu


def _weights(n, k, seed):
    from nova_b200.quant import nf4_codebook, quantize_nf4

    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(n, k, generator=g) * 0.02).half()
    return quantize_nf4(w.cuda(), nf4_codebook(), torch.float16)


def _lut():
    from nova_b200.kernels import build_nf4_lut
    from nova_b200.quant import nf4_codebook

    return build_nf4_lut(nf4_codebook()).cuda()


def _oracle(x, packed, absmax):
    """The reference kernel's arithmetic (src/nova/kernels.py:213-232): fp16
    codebook values times x, fp32 per 64-element block, times the block's
    absmax -- the same oracle as the batch-1 GEMV's."""
    return onf4.nf4_linear(x.float().cpu().numpy(), packed.cpu().numpy(), absmax.cpu().numpy(), onf4.nf4_codebook())


@pytest.mark.parametrize("m", [9, 16, 37, 64])
@pytest.mark.parametrize("n,k", [(1024, 2560), (2560, 9728), (6144, 2560), (96, 192), (3072, 2560), (2560, 2048),
                                 (2560, 4864), (2560, 1216)])
def test_gemm_plain_matches_dequant_matmul(cuda_lib, m, n, k):
    from nova_b200.kernels import nf4_gemm, pack_tc

    packed, absmax = _weights(n, k, n + k + m)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(m)).half()
    out = torch.full((m, n), float("nan"), dtype=torch.float16, device="cuda")
    nf4_gemm(x.cuda(), pack_tc(packed, absmax), _lut(), out, n=n)
    want = _oracle(x, packed, absmax)
    got = out.float().cpu().numpy()
    scale = float(np.abs(want).max())
    assert_ulp_or_abs(got, want.astype(np.float16), 1.0, 1e-5 * scale, f"gemm m={m} {n}x{k}")
    assert np.abs(got - want).max() <= 1e-2 * scale


@pytest.mark.parametrize("m", [65, 128, 300, 512])
@pytest.mark.parametrize("n,k", [(6144, 2560), (2560, 4096), (2560, 9728), (96, 192), (3072, 2560)])
def test_gemm_wide_matches_reference_kernel(cuda_lib, m, n, k):
    """M > 64 (prefill chunks): the 128 x 256-tile kernel with hi + lo weight
    terms, against the same oracle and bounds as the narrow path; ragged token
    tiles (65, 300) and a partial weight tile (96 rows) included."""
    from nova_b200.kernels import nf4_gemm, pack_tc

    packed, absmax = _weights(n, k, n + k + m)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(m)).half()
    out = torch.full((m, n), float("nan"), dtype=torch.float16, device="cuda")
    nf4_gemm(x.cuda(), pack_tc(packed, absmax), _lut(), out, n=n)
    want = _oracle(x, packed, absmax)
    got = out.float().cpu().numpy()
    scale = float(np.abs(want).max())
    w16 = want.astype(np.float16)
    # one fp16 ULP (the larger spacing around the value: at a power of two a sum that lands on the other
    # side of the rounding midpoint is one upper spacing away) or 1e-5 * max|y|
    ulp = np.maximum(fp16_ulp(w16), fp16_ulp(-w16))
    bad = np.argwhere(np.abs(got - w16.astype(np.float32)) > np.maximum(ulp, 1e-5 * scale))
    assert bad.size == 0, (f"wide gemm m={m} {n}x{k}: {len(bad)} outputs off, first {bad[:6].tolist()}, got "
                           f"{[float(got[tuple(b)]) for b in bad[:6]]}, want {[float(want[tuple(b)]) for b in bad[:6]]}")


def test_gemm_wide_epilogues(cuda_lib):
    """Residual (in place), fp32 and SiLU*up epilogues of the wide kernel at
    M = 300, every launch twice."""
    from nova_b200 import _lib
    from nova_b200.decoder import interleave_gate_up
    from nova_b200.kernels import nf4_gemm, pack_tc

    m, k = 300, 2560
    lut = _lut()
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(11)).half()
    xc = x.cuda()
    packed, absmax = _weights(2560, k, 12)
    units = pack_tc(packed, absmax)
    y = _oracle(x, packed, absmax)
    res = (torch.randn(m, 2560, generator=torch.Generator().manual_seed(13)) * 0.5).half()
    for _ in range(2):
        out = res.cuda()
        nf4_gemm(xc, units, lut, out, n=2560, epilogue=_lib.NF4_RESIDUAL, residual=out)
        want = (res.float().numpy() + y.astype(np.float16).astype(np.float32)).astype(np.float16)
        bound = fp16_ulp(y) + np.maximum(fp16_ulp(want), fp16_ulp(-want)) + 1e-5 * np.abs(y).max()
        assert np.all(np.abs(out.float().cpu().numpy() - want.astype(np.float32)) <= bound)
    out32 = torch.empty(m, 2560, dtype=torch.float32, device="cuda")
    nf4_gemm(xc, units, lut, out32, n=2560, epilogue=_lib.NF4_F32)
    np.testing.assert_allclose(out32.cpu().numpy(), y, rtol=1e-4, atol=1e-4 * np.abs(y).max())
    gp, ga = _weights(1024, k, 14)
    up, ua = _weights(1024, k, 15)
    ip, ia = interleave_gate_up(gp, ga, up, ua)
    act = torch.empty(m, 1024, dtype=torch.float16, device="cuda")
    nf4_gemm(xc, pack_tc(ip, ia), lut, act, n=2048, epilogue=_lib.NF4_SILU_MUL)
    g32, u32 = _oracle(x, gp, ga), _oracle(x, up, ua)
    g16, u16 = g32.astype(np.float16), u32.astype(np.float16)
    want = onorm.silu_mul(g16, u16).astype(np.float32)
    eg = np.maximum(fp16_ulp(g16), 1e-5 * np.abs(g32).max())
    eu = np.maximum(fp16_ulp(u16), 1e-5 * np.abs(u32).max())
    dev = np.zeros_like(want)
    for dg in (-1, 0, 1):
        for du in (-1, 0, 1):
            gg, uu = g16.astype(np.float32) + dg * eg, u16.astype(np.float32) + du * eu
            dev = np.maximum(dev, np.abs(gg / (1.0 + np.exp(-gg)) * uu - want))
    assert np.all(np.abs(act.float().cpu().numpy() - want) <= dev + 2 * fp16_ulp(want))


@pytest.mark.parametrize("m", [64, 33])
def test_gemm_lm_head_shape_sampled_rows(cuda_lib, m):
    """The 4-bit lm_head of config 5 (N = 151936, K = 2560) at batch 64 and a
    ragged 33: every row is computed; 3000 sampled rows (the first and last
    tiles included) are checked against the oracle's dequant-matmul."""
    from nova_b200.kernels import nf4_gemm, pack_tc

    n, k = 151936, 2560
    packed, absmax = _weights(n, k, 151936 + m)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(m)).half()
    out = torch.full((m, n), float("nan"), dtype=torch.float16, device="cuda")
    nf4_gemm(x.cuda(), pack_tc(packed, absmax), _lut(), out, n=n)
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    rows = np.unique(np.concatenate([np.arange(128), np.arange(n - 128, n),
                                     np.random.default_rng(m).choice(n, 2744, replace=False)]))
    want = _oracle(x, packed[rows], absmax[:, rows])
    scale = float(np.abs(want).max())
    assert_ulp_or_abs(got[:, rows], want.astype(np.float16), 1.0, 1e-5 * scale, f"lm_head m={m}")


def test_gemm_epilogues_and_repeat(cuda_lib):
    """Residual, fp32 partial, SiLU*up (gate/up interleaved) and argmax with the
    step finalize at M = 64; every launch twice to check the split-K counters
    re-arm."""
    from nova_b200 import _lib
    from nova_b200.decoder import interleave_gate_up
    from nova_b200.kernels import nf4_gemm, pack_tc

    m, k = 64, 2560
    lut = _lut()
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(1)).half()
    xc = x.cuda()
    # residual
    packed, absmax = _weights(2560, k, 2)
    units = pack_tc(packed, absmax)
    y = _oracle(x, packed, absmax)
    res = (torch.randn(m, 2560, generator=torch.Generator().manual_seed(3)) * 0.5).half()
    for _ in range(2):
        out = res.cuda()
        nf4_gemm(xc, units, lut, out, n=2560, epilogue=_lib.NF4_RESIDUAL, residual=out)
        want = (res.float().numpy() + y.astype(np.float16).astype(np.float32)).astype(np.float16)
        # y16 may round either way at a midpoint, and res + y16 then lands a whole
        # spacing away: the larger of the two spacings around want
        bound = fp16_ulp(y) + np.maximum(fp16_ulp(want), fp16_ulp(-want)) + 1e-5 * np.abs(y).max()
        diff = np.abs(out.float().cpu().numpy() - want.astype(np.float32))
        bad = np.argwhere(diff > bound)
        assert bad.size == 0, (f"{len(bad)} outputs beyond the bound, first {bad[:4].tolist()}: got "
                               f"{out.float().cpu().numpy()[tuple(bad[0])]}, want {want[tuple(bad[0])]}, "
                               f"y {y[tuple(bad[0])]}, res {res.float().numpy()[tuple(bad[0])]}")
    # fp32 partial
    out32 = torch.empty(m, 2560, dtype=torch.float32, device="cuda")
    nf4_gemm(xc, units, lut, out32, n=2560, epilogue=_lib.NF4_F32)
    np.testing.assert_allclose(out32.cpu().numpy(), y, rtol=1e-4, atol=1e-4 * np.abs(y).max())
    # SiLU * up
    gp, ga = _weights(1024, k, 4)
    up, ua = _weights(1024, k, 5)
    ip, ia = interleave_gate_up(gp, ga, up, ua)
    act = torch.empty(m, 1024, dtype=torch.float16, device="cuda")
    nf4_gemm(xc, pack_tc(ip, ia), lut, act, n=2048, epilogue=_lib.NF4_SILU_MUL)
    g32, u32 = _oracle(x, gp, ga), _oracle(x, up, ua)
    g16, u16 = g32.astype(np.float16), u32.astype(np.float16)
    want = onorm.silu_mul(g16, u16).astype(np.float32)
    eg = np.maximum(fp16_ulp(g16), 1e-5 * np.abs(g32).max())
    eu = np.maximum(fp16_ulp(u16), 1e-5 * np.abs(u32).max())
    dev = np.zeros_like(want)
    for dg in (-1, 0, 1):
        for du in (-1, 0, 1):
            gg, uu = g16.astype(np.float32) + dg * eg, u16.astype(np.float32) + du * eu
            dev = np.maximum(dev, np.abs(gg / (1.0 + np.exp(-gg)) * uu - want))
    assert np.all(np.abs(act.float().cpu().numpy() - want) <= dev + 2 * fp16_ulp(want))
    # argmax + finalize (token, re-armed slots, embedding gather, pos += 1)
    vocab = 4096
    lp, la = _weights(vocab, k, 6)
    embed = (torch.randn(vocab, k, generator=torch.Generator().manual_seed(7)) * 0.02).half().cuda()
    logits = torch.empty(m, vocab, dtype=torch.float16, device="cuda")
    slot = torch.zeros(m, dtype=torch.int64, device="cuda")
    tok = torch.zeros(m, dtype=torch.int64, device="cuda")
    pos = torch.tensor([10], dtype=torch.int64, device="cuda")
    nxt = torch.empty(m, k, dtype=torch.float16, device="cuda")
    lu = pack_tc(lp, la)
    for step in range(2):
        nf4_gemm(xc, lu, lut, logits, n=vocab, epilogue=_lib.NF4_ARGMAX, argmax=slot, token_out=tok, pos=pos,
                 embed=embed, embed_out=nxt)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(tok.cpu().numpy(), logits.float().argmax(dim=1).cpu().numpy())
        assert int(pos.item()) == 11 + step
        assert torch.equal(slot, torch.zeros_like(slot))
        assert torch.equal(nxt, embed[tok])


def test_gemm_rejects(cuda_lib):
    from nova_b200 import _lib
    from nova_b200.kernels import nf4_gemm, pack_tc

    packed, absmax = _weights(64, 128, 9)
    units = pack_tc(packed, absmax)
    out = torch.empty(65, 64, dtype=torch.float16, device="cuda")
    slot = torch.zeros(65, dtype=torch.int64, device="cuda")
    with pytest.raises(ValueError):   # argmax + step finalize only up to 64 rows
        nf4_gemm(torch.zeros(65, 128, dtype=torch.float16, device="cuda"), units, _lut(), out, n=64,
                 epilogue=_lib.NF4_ARGMAX, argmax=slot)
