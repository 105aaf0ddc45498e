"""CPU: host-side logic of the product package that needs no GPU (codebook,
LUT packing, weight layout transforms, RoPE tables, argument checks)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import nf4 as onf4
from oracle import norm as onorm


def test_product_codebook_and_lut_equal_oracle():
    from nova_b200.kernels import build_nf4_lut
    from nova_b200.quant import nf4_codebook, nf4_midpoints

    code = nf4_codebook()
    np.testing.assert_array_equal(code.numpy(), onf4.nf4_codebook())
    np.testing.assert_array_equal(build_nf4_lut(code).numpy(), onf4.build_nf4_lut(onf4.nf4_codebook()))
    np.testing.assert_array_equal(nf4_midpoints(code).numpy(), onf4.nf4_midpoints(onf4.nf4_codebook()))
    g = golden("nf4.npz")
    np.testing.assert_array_equal(build_nf4_lut(code).numpy(), g["lut"])


def test_gate_up_interleave_roundtrip():
    from nova_b200.decoder import deinterleave_gate_up, interleave_gate_up

    g = torch.Generator().manual_seed(0)
    gp = torch.randint(0, 256, (64, 40), generator=g, dtype=torch.uint8)
    up = torch.randint(0, 256, (64, 40), generator=g, dtype=torch.uint8)
    ga, ua = torch.randn(2, 64, generator=g).half(), torch.randn(2, 64, generator=g).half()
    p, a = interleave_gate_up(gp, ga, up, ua)
    assert p.shape == (128, 40) and a.shape == (2, 128)
    # tile r: rows 16r..16r+7 gate 8r..8r+7, rows 16r+8.. up 8r..
    assert torch.equal(p[16:24], gp[8:16]) and torch.equal(p[24:32], up[8:16])
    assert torch.equal(a[:, 16:24], ga[:, 8:16]) and torch.equal(a[:, 24:32], ua[:, 8:16])
    back = deinterleave_gate_up(p, a)
    for x, y in zip(back, (gp, ga, up, ua)):
        assert torch.equal(x, y)


def test_rope_tables_match_reference_rotary():
    from nova_b200.decoder import rope_tables

    g = golden("norm_rope.npz")
    cos, sin = rope_tables(131072, device="cpu")
    pos = g["rope_pos"]
    np.testing.assert_array_equal(cos[pos].numpy().view(np.uint16), g["rope_cos"].view(np.uint16))
    np.testing.assert_array_equal(sin[pos].numpy().view(np.uint16), g["rope_sin"].view(np.uint16))
    oc, os_ = onorm.rope_cos_sin(np.arange(64))
    np.testing.assert_array_equal(cos[:64].numpy(), oc)


def test_kvquant_rejects_cpu_tensors_and_channel_axis():
    from nova_b200.kvquant import quantize_int8

    with pytest.raises(ValueError):
        quantize_int8(torch.zeros(1, 1, 64, 128, dtype=torch.float16), 64, "token")   # no CPU fallback
    with pytest.raises(ValueError):
        quantize_int8(torch.zeros(1, 1, 64, 128, dtype=torch.float16))                # reference default axis


def test_bytes_accounting_matches_format():
    from nova_b200.kvquant import bytes_per_token

    c = bytes_per_token(num_slots=1, num_kv_heads=8, head_dim=128)
    assert c["int8t64_kv"] == 2176             # per token per layer: 2048 B codes + 128 B scales (8 KV heads)
    assert c["fp16_kv"] == 4096


@pytest.mark.parametrize("max_len,batch", [(8448, 1), (33024, 1), (131328, 1), (33024, 4), (33024, 64), (320, 2)])
def test_pick_chunk_properties(max_len, batch):
    """Attention split size: a multiple of 64, at least 256 tokens, at most 8192 tokens
    once the context needs more than one split, and few enough splits that the last CTA
    of a KV head can stage every split's partials in one shared-memory copy."""
    from nova_b200.kvattn import GROUP_T, pick_chunk

    hq, hkv = 32, 8
    chunk = pick_chunk(max_len, batch, hkv, hq)
    n_splits = -(-max_len // chunk)
    cap = 73728 // ((hq // hkv) * 528) - 1
    assert chunk % GROUP_T == 0 and chunk >= 4 * GROUP_T
    assert n_splits <= cap
    if -(-max_len // 8192) <= cap:
        assert chunk <= 8192


def test_heads_major_reorders_units_by_column_block():
    """o_proj's head-major unit stream: native unit (row group r, k-block b)
    of an [N, K] matrix moves to block h = b // (K / 64 / heads), position
    (h * N / 32 + r) * (K / 64 / heads) + b % (K / 64 / heads)."""
    from nova_b200.kernels import heads_major

    n, k, heads, unit = 2560, 4096, 8, 1088
    rg, kb = n // 32, k // 64
    per = kb // heads
    ids = torch.arange(rg * kb, dtype=torch.int32)
    stream = ids.view(-1, 1).expand(-1, unit // 4).contiguous().view(torch.uint8).view(-1)   # unit u filled with u
    out = heads_major(stream, n, k, heads).view(-1, unit).view(torch.int32)[:, 0]
    r, b = ids // kb, ids % kb
    want_pos = ((b // per) * rg + r) * per + b % per
    assert torch.equal(out[want_pos.long()], ids)


def test_attention_partials_address():
    """The split partials start at byte 256 + align_up(batch * kv_heads * 4,
    256) of the attention workspace (the error word, then the per-head
    arrival counters), the layout nova_attn_workspace_bytes sizes."""
    from nova_b200.kvattn import attn_partials

    ws = torch.zeros(1 << 20, dtype=torch.uint8)
    base = ws.data_ptr()
    assert attn_partials(ws, 1, 8) - base == 256 + 256
    assert attn_partials(ws, 64, 8) - base == 256 + 2048
    assert attn_partials(ws, 3, 7) - base == 256 + 256
    from nova_b200.kvattn import attn_workspace_bytes   # the library sizes partials right after that offset

    assert attn_workspace_bytes(1, 32, 8, 33, True) == 256 + 256 + 8 * 34 * 4 * 132 * 4


def _heads_cta_range(c, G, nh, R, KB):
    """Python restatement of the head-aligned CTA range of nf4.cu (heads_cta_range)."""
    h = ((c + 1) * nh - 1) // G
    c0 = G * h // nh
    n = G * (h + 1) // nh - c0
    j = c - c0
    return (h * R + R * j // n) * KB, (h * R + R * (j + 1) // n) * KB, h


@pytest.mark.parametrize("G,nh,R,KB", [(148, 8, 80, 8), (132, 8, 80, 8), (148, 4, 80, 16), (148, 8, 64, 8)])
def test_head_aligned_o_proj_schedule_covers_every_row_group_once(G, nh, R, KB):
    """o_proj over the attention's partials, on shapes nova_nf4_gemv accepts
    (at least 16 units per CTA): the CTAs tile the (head, row group) stream
    exactly, each CTA inside one head with whole row groups, and its 16
    warps' consecutive ranges (1+ units each) tile the CTA's."""
    assert (R // -(-G // nh)) * KB >= 16   # the host check of attn_part
    seen = []
    for c in range(G):
        u0, u1, h = _heads_cta_range(c, G, nh, R, KB)
        assert u0 % KB == 0 and u1 % KB == 0 and u1 > u0
        assert h * R * KB <= u0 and u1 <= (h + 1) * R * KB, "a CTA crosses a head"
        assert (u1 - u0) // KB + 1 <= 16, "more row groups than warps to sum them"
        ws = [u0 + (u1 - u0) * w // 16 for w in range(17)]
        assert ws[0] == u0 and ws[-1] == u1 and all(b - a >= 1 for a, b in zip(ws, ws[1:]))
        seen.extend(range(u0, u1))
    assert seen == list(range(nh * R * KB))


def test_gate_up_cta_edges_match_the_consumer_boundaries():
    """gate|up with CTA edges (19456 x 2560 on 148 SMs): every row group split
    between CTAs has exactly two contributors (the last row group of one CTA,
    the first of the next), and these are exactly the boundaries the
    down_proj staging completes (edge_plan: u = units * b / G not a multiple
    of the k-blocks per row group)."""
    G, KB = 148, 40
    units = (19456 // 32) * KB
    ranges = [(units * c // G, units * (c + 1) // G) for c in range(G)]
    split = {}
    for c, (u0, u1) in enumerate(ranges):
        for rg in range(u0 // KB, (u1 - 1) // KB + 1):
            if not (u0 <= rg * KB and u1 >= (rg + 1) * KB):
                split.setdefault(rg, []).append(c)
    assert all(len(v) == 2 and v[1] == v[0] + 1 for v in split.values())
    plan = {units * b // G // KB: (b - 1, b) for b in range(1, G) if (units * b // G) % KB}
    assert plan == {rg: tuple(v) for rg, v in split.items()}
