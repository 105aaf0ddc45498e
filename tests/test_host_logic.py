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
