"""GPU: NF4 quantizer / dequant / GEMV (nova_nf4_*) against the CPU oracle.

Tolerances: the GEMV accumulates exact fp16 products in fp32 like the
reference kernel, so each fp16 output must be within 1 fp16 ULP of the
oracle's fp32 result or within 1e-5 * max|y| absolute
(1e-2 relative to the dequant-matmul) is asserted as well.  The quantizer
and dequant are bit-exact."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import assert_ulp_or_abs, fp16_ulp
from oracle import nf4 as onf4
from oracle import norm as onorm

pytestmark = pytest.mark.gpu

SHAPES = {  # name: (N, K) -- Qwen3-4B decode projections
    "q_proj": (4096, 2560), "k_proj": (1024, 2560), "v_proj": (1024, 2560), "o_proj": (2560, 4096),
    "gate_proj": (9728, 2560), "up_proj": (9728, 2560), "down_proj": (2560, 9728),
}


def _weights(n, k, seed, absmax_dtype=torch.float16):
    from nova_b200.quant import nf4_codebook, quantize_nf4

    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(n, k, generator=g) * 0.02).half()
    packed, absmax = quantize_nf4(w.cuda(), nf4_codebook(), absmax_dtype)
    return w, packed, absmax


def _lut(device="cuda"):
    from nova_b200.kernels import build_nf4_lut
    from nova_b200.quant import nf4_codebook

    return build_nf4_lut(nf4_codebook()).to(device)


def _oracle_y(x, packed, absmax, rows=None):
    p, a = packed.cpu().numpy(), absmax.cpu().numpy()
    if rows is not None:
        p, a = p[rows], a[:, rows]
    return onf4.nf4_linear(x.float().cpu().numpy(), p, a, onf4.nf4_codebook())


LAYOUTS = ["ref", "native"]


def _gemv(layout, x, packed, absmax, out, **kw):
    """Run the GEMV on the reference layout or on the packed native unit stream."""
    from nova_b200.kernels import nf4_gemv, pack_native

    if layout == "native":
        return nf4_gemv(x, pack_native(packed, absmax), None, _lut(), out, n=packed.shape[0], **kw)
    return nf4_gemv(x, packed, absmax, _lut(), out, **kw)


def _check(got, want32, tag):
    got = got.float().cpu().numpy()
    scale = float(np.abs(want32).max())
    assert_ulp_or_abs(got, want32.astype(np.float16), 1.0, 1e-5 * scale, tag)
    assert np.abs(got - want32).max() <= 1e-2 * scale, f"{tag}: beyond 1e-2 relative"


def _assert_silu(got, g32, u32, tag):
    """SiLU·mul outputs against the oracle.  gate and up are rounded to fp16
    before SiLU*up, and each may sit one ulp (or, where the dot product cancels,
    1e-5 * max|y|: the GEMV criterion) away from the oracle's; SiLU amplifies
    that by up to |g| where it is flat.  Bound: the oracle evaluated at gate/up
    moved by that much either way, plus 2 ulp; over 99 % exact."""
    g16, u16 = g32.astype(np.float16), u32.astype(np.float16)
    want = onorm.silu_mul(g16, u16).astype(np.float32)
    eg = np.maximum(fp16_ulp(g16), 1e-5 * np.abs(g32).max())
    eu = np.maximum(fp16_ulp(u16), 1e-5 * np.abs(u32).max())
    dev = np.zeros_like(want)
    for dg in (-1, 0, 1):
        for du in (-1, 0, 1):
            gg = g16.astype(np.float32) + dg * eg
            uu = u16.astype(np.float32) + du * eu
            alt = gg / (1.0 + np.exp(-gg)) * uu
            dev = np.maximum(dev, np.abs(alt - want))
    assert np.all(np.abs(got - want) <= dev + 2 * fp16_ulp(want)), tag
    assert (got == want).mean() > 0.99, f"{tag}: too few exact"
    return want


def test_codebook_matches_oracle(cuda_lib):
    from nova_b200.quant import nf4_codebook

    np.testing.assert_array_equal(nf4_codebook().numpy(), onf4.nf4_codebook())
    from nova_b200.kernels import build_nf4_lut

    np.testing.assert_array_equal(build_nf4_lut(nf4_codebook()).numpy(), onf4.build_nf4_lut(onf4.nf4_codebook()))


@pytest.mark.parametrize("absmax_dtype", [torch.float16, torch.float32])
def test_quantizer_bit_exact(cuda_lib, absmax_dtype):
    w, packed, absmax = _weights(320, 1024, 1, absmax_dtype)
    w[5, :64] = 0   # an all-zero block
    from nova_b200.quant import nf4_codebook, quantize_nf4

    packed, absmax = quantize_nf4(w.cuda(), nf4_codebook(), absmax_dtype)
    op, oa = onf4.quantize_nf4(w.numpy(), onf4.nf4_codebook(),
                               np.float16 if absmax_dtype == torch.float16 else np.float32)
    np.testing.assert_array_equal(packed.cpu().numpy(), op)
    np.testing.assert_array_equal(absmax.cpu().numpy(), oa)


def test_dequant_bit_exact(cuda_lib):
    from nova_b200.quant import dequantize_nf4

    _, packed, absmax = _weights(256, 512, 2)
    got = dequantize_nf4(packed, absmax, _lut())
    want = onf4.dequantize_nf4(packed.cpu().numpy(), absmax.cpu().numpy(), onf4.nf4_codebook(), round_fp16=True)
    np.testing.assert_array_equal(got.cpu().numpy().view(np.uint16), want.view(np.uint16))


@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("name", list(SHAPES))
def test_gemv_qwen_shapes_m1(cuda_lib, name, layout):
    n, k = SHAPES[name]
    _, packed, absmax = _weights(n, k, sum(map(ord, name)))
    x = (torch.randn(1, k, generator=torch.Generator().manual_seed(3))).half()
    out = torch.empty(1, n, dtype=torch.float16, device="cuda")
    _gemv(layout, x.cuda(), packed, absmax, out)
    _check(out, _oracle_y(x, packed, absmax), f"{name} {layout}")


@pytest.mark.parametrize("layout", LAYOUTS)
def test_gemv_lm_head_shape_sampled_rows(cuda_lib, layout):
    """151936 x 2560 (the 4-bit lm_head): all rows computed on the GPU, 4096
    random rows checked against the oracle."""
    n, k = 151936, 2560
    _, packed, absmax = _weights(n, k, 11)
    x = torch.randn(1, k, generator=torch.Generator().manual_seed(4)).half()
    out = torch.empty(1, n, dtype=torch.float16, device="cuda")
    _gemv(layout, x.cuda(), packed, absmax, out)
    rows = np.sort(np.random.default_rng(0).choice(n, 4096, replace=False))
    _check(out[:, rows], _oracle_y(x, packed, absmax, rows), "lm_head")


@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("m", [2, 5, 8])
def test_gemv_small_batch(cuda_lib, m, layout):
    _, packed, absmax = _weights(1024, 2560, 5)
    x = torch.randn(m, 2560, generator=torch.Generator().manual_seed(m)).half()
    out = torch.empty(m, 1024, dtype=torch.float16, device="cuda")
    _gemv(layout, x.cuda(), packed, absmax, out)
    _check(out, _oracle_y(x, packed, absmax), f"m={m} {layout}")


@pytest.mark.parametrize("layout", LAYOUTS)
def test_gemv_is_deterministic(cuda_lib, layout):
    """The split-K reduction adds partials in a fixed order: repeated launches
    are bit-identical, with and without programmatic dependent launch."""
    from nova_b200 import _lib

    _, packed, absmax = _weights(2560, 4096, 6)
    x = torch.randn(1, 4096, generator=torch.Generator().manual_seed(7)).half().cuda()
    a = _gemv(layout, x, packed, absmax, torch.empty(1, 2560, dtype=torch.float16, device="cuda"))
    b = _gemv(layout, x, packed, absmax, torch.empty(1, 2560, dtype=torch.float16, device="cuda"))
    _lib.set_pdl(True)
    try:
        c = _gemv(layout, x, packed, absmax, torch.empty(1, 2560, dtype=torch.float16, device="cuda"))
    finally:
        _lib.set_pdl(False)
    assert torch.equal(a, b) and torch.equal(a, c)


@pytest.mark.parametrize("layout", LAYOUTS)
def test_residual_epilogue(cuda_lib, layout):
    from nova_b200 import _lib

    _, packed, absmax = _weights(2560, 4096, 8)
    x = torch.randn(1, 4096, generator=torch.Generator().manual_seed(8)).half()
    res = torch.randn(1, 2560, generator=torch.Generator().manual_seed(9)).half()
    out = res.clone().cuda()
    _gemv(layout, x.cuda(), packed, absmax, out, epilogue=_lib.NF4_RESIDUAL, residual=out)   # in place
    y16 = _oracle_y(x, packed, absmax).astype(np.float16)
    want = (res.numpy().astype(np.float32) + y16.astype(np.float32)).astype(np.float16)
    got = out.cpu().numpy().astype(np.float32)
    # the projection may round to the neighbouring fp16 value (fp32 summation order); after the
    # residual add that ULP of y can dominate a small result, so the bound is ulp(y) + ulp(result)
    from conftest import fp16_ulp

    tol = fp16_ulp(y16) + fp16_ulp(want)
    assert np.all(np.abs(got - want.astype(np.float32)) <= tol), "residual add beyond one ULP of each operand"
    assert (got == want.astype(np.float32)).mean() > 0.99


@pytest.mark.parametrize("layout", LAYOUTS)
def test_silu_mul_epilogue_interleaved(cuda_lib, layout):
    from nova_b200 import _lib
    from nova_b200.decoder import interleave_gate_up

    n, k = 1024, 2560
    _, gp, ga = _weights(n, k, 12)
    _, up, ua = _weights(n, k, 13)
    packed, absmax = interleave_gate_up(gp, ga, up, ua)
    x = torch.randn(1, k, generator=torch.Generator().manual_seed(14)).half()
    out = torch.empty(1, n, dtype=torch.float16, device="cuda")
    _gemv(layout, x.cuda(), packed, absmax, out, epilogue=_lib.NF4_SILU_MUL)
    g16 = _oracle_y(x, gp, ga).astype(np.float16)
    u16 = _oracle_y(x, up, ua).astype(np.float16)
    want = onorm.silu_mul(g16, u16)
    assert_ulp_or_abs(out.cpu().numpy(), want, 1.0, 1e-6, "silu_mul")


@pytest.mark.parametrize("layout", LAYOUTS)
def test_norm_prologue(cuda_lib, layout):
    _, packed, absmax = _weights(6144, 2560, 15)
    h = (torch.randn(3, 2560, generator=torch.Generator().manual_seed(16)) * 3).half()
    w = (1 + 0.1 * torch.randn(2560, generator=torch.Generator().manual_seed(17))).half()
    out = torch.empty(3, 6144, dtype=torch.float16, device="cuda")
    _gemv(layout, h.cuda(), packed, absmax, out, norm_weight=w.cuda(), eps=1e-6)
    xn = onorm.rms_norm(h.numpy(), w.numpy(), 1e-6)
    _check(out, _oracle_y(torch.from_numpy(xn), packed, absmax), "norm prologue")


@pytest.mark.parametrize("layout", LAYOUTS)
def test_argmax_epilogue_and_step_finalize(cuda_lib, layout):
    from nova_b200 import _lib

    n, k, vocab_embed = 8192, 2560, 8192
    _, packed, absmax = _weights(n, k, 18)
    x = torch.randn(2, k, generator=torch.Generator().manual_seed(19)).half()
    embed = (torch.randn(vocab_embed, k, generator=torch.Generator().manual_seed(20)) * 0.02).half().cuda()
    logits = torch.empty(2, n, dtype=torch.float16, device="cuda")
    slot = torch.zeros(2, dtype=torch.int64, device="cuda")
    tokens = torch.full((2,), -1, dtype=torch.int64, device="cuda")
    pos = torch.tensor([41], dtype=torch.int64, device="cuda")
    hidden = torch.empty(2, k, dtype=torch.float16, device="cuda")
    _gemv(layout, x.cuda(), packed, absmax, logits, epilogue=_lib.NF4_ARGMAX, argmax=slot, token_out=tokens,
          pos=pos, embed=embed, embed_out=hidden)
    torch.cuda.synchronize()
    # greedy token = first index of the maximal fp16 logit (torch.argmax semantics)
    want_tok = torch.argmax(logits, dim=-1)
    assert torch.equal(tokens, want_tok)
    assert int(pos.item()) == 42
    assert torch.count_nonzero(slot).item() == 0
    assert torch.equal(hidden, embed[want_tok])
    _check(logits, _oracle_y(x, packed, absmax), "logits")


@pytest.mark.parametrize("layout", LAYOUTS)
def test_shared_workspace_across_shapes(cuda_lib, layout):
    """GEMVs with different N on one workspace (as the decoder launches them)
    give the same results as with private workspaces, including the argmax
    finalize."""
    from nova_b200 import _lib
    from nova_b200.kernels import gemv_workspace

    shapes = [(512, 1024, _lib.NF4_RESIDUAL), (2048, 512, _lib.NF4_SILU_MUL), (1536, 512, _lib.NF4_PLAIN),
              (4096, 512, _lib.NF4_ARGMAX)]
    ws_shared = gemv_workspace(torch.device("cuda"), 4096).clone()
    for n, k, epi in shapes * 2:
        _, packed, absmax = _weights(n, k, n + k)
        x = torch.randn(1, k, generator=torch.Generator().manual_seed(k)).half().cuda()
        outs = []
        for ws in (ws_shared, gemv_workspace(torch.device("cuda"), n).clone()):
            nout = n // 2 if epi == _lib.NF4_SILU_MUL else n
            out = torch.zeros(1, nout, dtype=torch.float16, device="cuda")
            kw = {}
            if epi == _lib.NF4_RESIDUAL:
                kw["residual"] = out
            if epi == _lib.NF4_ARGMAX:
                kw.update(argmax=torch.zeros(1, dtype=torch.int64, device="cuda"),
                          token_out=torch.full((1,), -1, dtype=torch.int64, device="cuda"),
                          pos=torch.zeros(1, dtype=torch.int64, device="cuda"))
            _gemv(layout, x, packed, absmax, out, epilogue=epi, workspace=ws, **kw)
            outs.append((out, kw))
        assert torch.equal(outs[0][0], outs[1][0]), f"N={n} epilogue {epi}"
        if epi == _lib.NF4_ARGMAX:
            for o, kw in outs:
                assert int(kw["pos"].item()) == 1 and int(kw["token_out"].item()) == int(torch.argmax(o).item())


def test_native_packer_layout(cuda_lib):
    """Unit record = two lane-major halves of code bytes (rows g, g+8 then rows
    g+16, g+24; 16 bytes per lane in each), then absmax in lane-group order."""
    from nova_b200.kernels import pack_native

    _, packed, absmax = _weights(64, 128, 31)
    u = pack_native(packed, absmax).cpu().numpy()
    p, a = packed.cpu().numpy(), absmax.cpu().numpy()
    assert u.size == 2 * 2 * 1088
    for unit in range(4):
        rg, b = divmod(unit, 2)
        rec = u[unit * 1088:(unit + 1) * 1088]
        for lane in range(32):
            g, t = divmod(lane, 4)
            for r in range(4):
                row = 32 * rg + g + 8 * r
                off = 512 * (r // 2) + 16 * lane + 8 * (r % 2)
                np.testing.assert_array_equal(rec[off: off + 8],
                                              p[row, 32 * b + 8 * t: 32 * b + 8 * t + 8])
        am = rec[1024:].view(np.float16)
        for g in range(8):
            for r in range(4):
                assert am[4 * g + r] == a[b, 32 * rg + g + 8 * r]


def test_fused_nf4_linear_reference_layout(cuda_lib):
    """Reference calling convention: fp32 absmax [K/64, N], bias, M = 7 and 20."""
    from nova_b200.kernels import build_nf4_lut, fused_nf4_linear
    from nova_b200.quant import nf4_codebook

    _, packed, absmax = _weights(512, 256, 21, torch.float32)
    lut = build_nf4_lut(nf4_codebook()).cuda()
    bias = (torch.randn(512, generator=torch.Generator().manual_seed(22)) * 0.01).half()
    for m in (7, 20):
        x = (torch.randn(1, m, 256, generator=torch.Generator().manual_seed(m)) * 0.5).half()
        got = fused_nf4_linear(x.cuda(), packed, absmax, lut, 512, bias.cuda())
        assert got.shape == (1, m, 512)
        want = onf4.nf4_linear(x[0].float().numpy(), packed.cpu().numpy(), absmax.cpu().numpy(),
                               onf4.nf4_codebook(), bias.float().numpy())
        _check(got[0], want, f"fused_nf4_linear m={m}")


def test_nf4linear_module_and_rejects_bad_inputs(cuda_lib):
    from nova_b200.kernels import fused_nf4_linear
    from nova_b200.quant import NF4Linear

    w = (torch.randn(256, 512, generator=torch.Generator().manual_seed(23)) * 0.02).half().cuda()
    lin = NF4Linear.from_float(w)
    x = torch.randn(1, 1, 512, generator=torch.Generator().manual_seed(24)).half().cuda()
    y = lin(x)
    want = _oracle_y(x[0].cpu(), lin.packed, lin.absmax)
    _check(y[0], want, "NF4Linear")
    with pytest.raises(ValueError):
        fused_nf4_linear(x[..., :256], lin.packed, lin.absmax, lin.lut, 256)
    with pytest.raises(ValueError):
        fused_nf4_linear(x, lin.packed, lin.absmax, lin.lut, 128)
    with pytest.raises(ValueError):
        fused_nf4_linear(x.cpu(), lin.packed, lin.absmax, lin.lut, 256)


@pytest.mark.parametrize("variant", ["cta", "warp"])
@pytest.mark.parametrize("n,k,epi", [(1024, 2560, "plain"), (2560, 9728, "residual"), (96, 192, "plain"),
                                     (19456, 2560, "silu")])
def test_native_split_k_variants(cuda_lib, variant, n, k, epi):
    """Both native split-K schedules (CTA-level on whole row groups, warp-level
    stream-K) match the oracle on shapes that select each by default; M = 2."""
    from nova_b200 import _lib
    from nova_b200.decoder import interleave_gate_up
    from nova_b200.kernels import nf4_gemv, pack_native

    x = (torch.randn(2, k, generator=torch.Generator().manual_seed(5))).half()
    if epi == "silu":
        _, gp, ga = _weights(n // 2, k, 31)
        _, up, ua = _weights(n // 2, k, 32)
        packed, absmax = interleave_gate_up(gp, ga, up, ua)
    else:
        _, packed, absmax = _weights(n, k, n + k)
    nout = n // 2 if epi == "silu" else n
    res = (torch.randn(2, nout, generator=torch.Generator().manual_seed(6)) * 0.1).half().cuda()
    out = res.clone() if epi == "residual" else torch.empty(2, nout, dtype=torch.float16, device="cuda")
    kw = {}
    if epi == "residual":
        kw = {"epilogue": _lib.NF4_RESIDUAL, "residual": out}
    elif epi == "silu":
        kw = {"epilogue": _lib.NF4_SILU_MUL}
    flags = _lib.lib().nova_get_launch_flags()
    try:
        _lib.set_launch_flags((flags & _lib.LAUNCH_PDL) | (_lib.LAUNCH_WARP_SPLITK if variant == "warp" else 0))
        nf4_gemv(x.cuda(), pack_native(packed, absmax), None, _lut(), out, n=n, **kw)
    finally:
        _lib.set_launch_flags(flags)
    got = out.float().cpu().numpy()
    if epi == "plain":
        _check(out, _oracle_y(x, packed, absmax), f"{variant} {n}x{k}")
    elif epi == "residual":
        y = _oracle_y(x, packed, absmax)
        want = (res.float().cpu().numpy() + y.astype(np.float16).astype(np.float32)).astype(np.float16)
        # fp16(y) may land one ulp(y) away, then the add rounds again: ulp(y) + ulp(result)
        bound = fp16_ulp(y) + fp16_ulp(want) + 1e-5 * np.abs(y).max()
        assert np.all(np.abs(got - want.astype(np.float32)) <= bound), variant
    else:
        _assert_silu(got, _oracle_y(x, gp, ga), _oracle_y(x, up, ua), f"silu {variant}")


@pytest.mark.parametrize("n_prev,k_prev", [(2560, 4096), (2560, 9728)])
def test_slot_epilogue_and_deferred_residual_add(cuda_lib, n_prev, k_prev):
    """o_proj / down_proj as NF4_SLOTS (every SM takes an equal share of the
    k-blocks, fp32 sums per CTA) and the next GEMV adding them to the residual
    while it stages its normed input: the stored residual equals
    fp16(res + fp16(x @ W^T)) within one fp16 ULP of the oracle, and the next
    projection matches the oracle on it; run twice (no state left behind)."""
    from nova_b200 import _lib
    from nova_b200.kernels import gemv_workspace, nf4_gemv, pack_native, slots_buffer

    _, pp, pa = _weights(n_prev, k_prev, 21)
    _, qp, qa = _weights(6144, n_prev, 22)
    a = torch.randn(1, k_prev, generator=torch.Generator().manual_seed(23)).half()
    res = (torch.randn(1, n_prev, generator=torch.Generator().manual_seed(24)) * 2).half()
    w = (1 + 0.1 * torch.randn(n_prev, generator=torch.Generator().manual_seed(25))).half()
    up, uq = pack_native(pp, pa), pack_native(qp, qa)
    slots = slots_buffer(torch.device("cuda"))
    ws = gemv_workspace(torch.device("cuda"), 6144)
    lut = _lut()
    o16 = _oracle_y(a, pp, pa).astype(np.float16)
    want_res = (res.float().numpy() + o16.astype(np.float32)).astype(np.float16)
    for _ in range(2):
        resid_out = torch.full((1, n_prev), float("nan"), dtype=torch.float16, device="cuda")
        out = torch.empty(1, 6144, dtype=torch.float16, device="cuda")
        nf4_gemv(a.cuda(), up, None, lut, slots, epilogue=_lib.NF4_SLOTS, workspace=ws, n=n_prev)
        nf4_gemv(res.cuda(), uq, None, lut, out, norm_weight=w.cuda(), eps=1e-6, workspace=ws, n=6144,
                 add_slots=slots, add_k=k_prev, resid_out=resid_out)
        got_res = resid_out.float().cpu().numpy()
        w16 = want_res
        ulp = np.maximum(fp16_ulp(w16), fp16_ulp(-w16)) + fp16_ulp(o16)
        assert np.all(np.abs(got_res - w16.astype(np.float32)) <= ulp), "deferred residual add"
        xn = onorm.rms_norm(resid_out.cpu().numpy(), w.numpy(), 1e-6)
        _check(out, _oracle_y(torch.from_numpy(xn), qp, qa), "projection after the deferred add")


def test_gate_up_edges_completed_by_down(cuda_lib):
    """gate|up (19456 x 2560, SiLU·mul) with edge_out: the row groups split
    between its CTAs stay fp32 sums, and down_proj (2560 x 9728) with edge_in
    completes them while staging its input.  The edge sums plus the written
    outputs give the activation within the SiLU·mul bound of the oracle (the
    edges are added in CTA order on the host the way the consumer does), and the
    down projection matches the oracle over that completed activation; run
    twice (no state left behind)."""
    from nova_b200 import _lib
    from nova_b200.decoder import interleave_gate_up
    from nova_b200.kernels import edge_buffer, gemv_workspace, nf4_gemv, pack_native

    hidden, inter = 2560, 9728
    _, gp, ga = _weights(inter, hidden, 31)
    _, upk, ua = _weights(inter, hidden, 32)
    _, dp, da = _weights(hidden, inter, 33)
    packed, absmax = interleave_gate_up(gp, ga, upk, ua)
    gu, dn = pack_native(packed, absmax), pack_native(dp, da)
    x = torch.randn(1, hidden, generator=torch.Generator().manual_seed(34)).half()
    lut = _lut()
    ws = gemv_workspace(torch.device("cuda"), 2 * inter)
    edges = edge_buffer(torch.device("cuda"))
    g32, u32 = _oracle_y(x, gp, ga), _oracle_y(x, upk, ua)

    sms = torch.cuda.get_device_properties(0).multi_processor_count
    kb = hidden // 64
    units = (2 * inter // 32) * kb
    gate_ix = [0, 1, 2, 3, 4, 5, 6, 7, 16, 17, 18, 19, 20, 21, 22, 23]
    up_ix = [8, 9, 10, 11, 12, 13, 14, 15, 24, 25, 26, 27, 28, 29, 30, 31]
    for _ in range(2):
        edges.fill_(float("nan"))
        h = torch.full((1, inter), float("nan"), dtype=torch.float16, device="cuda")
        nf4_gemv(x.cuda(), gu, None, lut, h, epilogue=_lib.NF4_SILU_MUL, workspace=ws, n=2 * inter, edge_out=edges)
        y = torch.empty(1, hidden, dtype=torch.float16, device="cuda")
        nf4_gemv(h, dn, None, lut, y, workspace=ws, n=hidden, edge_in=edges, edge_k=hidden)
        got_h = h.float().cpu().numpy()[0].copy()
        e = edges.cpu().numpy()
        split = np.zeros(inter, dtype=bool)
        for bnd in range(1, sms):
            u = units * bnd // sms
            if u % kb == 0:
                continue
            rg = u // kb
            a, b = e[2 * (bnd - 1) + 1], e[2 * bnd]
            gs, us = a[gate_ix] + b[gate_ix], a[up_ix] + b[up_ix]
            got_h[16 * rg:16 * rg + 16] = onorm.silu_mul(gs.astype(np.float16), us.astype(np.float16))
            split[16 * rg:16 * rg + 16] = True
        assert split.sum() > 100 * 16, "expected row groups split between CTAs"
        assert not np.isnan(got_h).any(), "an activation was neither written nor left as an edge"
        _assert_silu(got_h, g32[0], u32[0], "silu_mul with edges")
        # down over the activation the launches produced (completed by the consumer as on the host)
        _check(y, _oracle_y(torch.from_numpy(got_h[None].astype(np.float32)), dp, da), "down_proj completing the edges")


def test_edges_rejected_outside_their_shapes(cuda_lib):
    from nova_b200 import _lib
    from nova_b200.kernels import edge_buffer, gemv_workspace, nf4_gemv, pack_native

    _, p, a = _weights(4096, 2560, 41)
    units = pack_native(p, a)
    x = torch.zeros(1, 2560, dtype=torch.float16, device="cuda")
    out = torch.empty(1, 4096, dtype=torch.float16, device="cuda")
    edges = edge_buffer(torch.device("cuda"))
    ws = gemv_workspace(torch.device("cuda"), 4096)
    with pytest.raises(ValueError, match="edge_out"):   # not SiLU·mul
        nf4_gemv(x, units, None, _lut(), out, workspace=ws, n=4096, edge_out=edges)
    with pytest.raises(ValueError, match="edge_out"):   # SiLU·mul, but too few units for every warp
        nf4_gemv(x, units, None, _lut(), out[:, :2048], epilogue=_lib.NF4_SILU_MUL, workspace=ws, n=4096,
                 edge_out=edges)
    with pytest.raises(ValueError, match="edge_in"):   # with a norm prologue
        nf4_gemv(x, units, None, _lut(), out, workspace=ws, n=4096, norm_weight=x[0], edge_in=edges, edge_k=2560)


def test_attention_partials_and_head_sums_rejected_outside_their_shapes(cuda_lib):
    """attn_part (o_proj over the decode attention's split partials) takes only
    NF4_F32 at M = 1 on a K of 128 x (1..4) columns with at most 40 splits;
    add_heads needs a norm prologue."""
    from nova_b200 import _lib
    from nova_b200.kernels import gemv_workspace, heads_major, nf4_gemv, pack_native

    _, p, a = _weights(2560, 4096, 51)
    units = heads_major(pack_native(p, a), 2560, 4096, 8)
    x = torch.zeros(1, 512, dtype=torch.float16, device="cuda")
    part = torch.zeros(8 * 34 * 4 * 132, dtype=torch.float32, device="cuda")
    y = torch.zeros(1, 8 * 2560, dtype=torch.float32, device="cuda")
    ws = gemv_workspace(torch.device("cuda"), 8 * 2560)
    kw = dict(workspace=ws, n=8 * 2560, attn_part=part.data_ptr(), attn_heads=8)
    nf4_gemv(x, units, None, _lut(), y, epilogue=_lib.NF4_F32, attn_splits=34, **kw)   # accepted
    torch.cuda.synchronize()
    with pytest.raises(ValueError, match="attn_part"):   # not the fp32 epilogue
        nf4_gemv(x, units, None, _lut(), y.half(), attn_splits=34, **kw)
    with pytest.raises(ValueError, match="attn_part"):   # more splits than the merge holds
        nf4_gemv(x, units, None, _lut(), y, epilogue=_lib.NF4_F32, attn_splits=41, **kw)
    heads = torch.zeros(8, 2560, dtype=torch.float32, device="cuda")
    xr = torch.zeros(1, 2560, dtype=torch.float16, device="cuda")
    out = torch.empty(1, 4096, dtype=torch.float16, device="cuda")
    _, qp, qa = _weights(4096, 2560, 52)
    with pytest.raises(ValueError, match="add_heads"):   # no norm prologue
        nf4_gemv(xr, pack_native(qp, qa), None, _lut(), out, workspace=ws, n=4096, add_heads=heads)
