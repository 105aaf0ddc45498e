"""Generate the golden fixtures in this directory by running the REFERENCE's own
Python code (captain-wangrun-cn/Nova, ``src/nova``) on seeded inputs.

Run with the reference's ``src`` directory named in ``NOVA_REF_SRC`` (required):

    NOVA_REF_SRC=/path/to/Nova/src python tests/golden/make_golden.py [fixture ...]

The fixtures pin the CPU oracle (``oracle/``) to the reference; the GPU tests
then compare the CUDA kernels with the oracle.  Only the reference functions
that run without Triton/CUDA/bitsandbytes are used (kvquant, the KVInt8Cache
prefill + ring path on CPU, SDPA math on CPU, LeanRMSNorm "exact",
apply_rotary_pos_emb with the transformers Qwen3-VL rotary, build_nf4_lut,
extract_nf4 with a non-nested quant state, the chat CLI's sample_next (its
candidate ids and final probabilities), and the decoder: the reference's own
GraphDecoder (prefill + eager decode steps, quant="int8") over its
NovaForCausalLM / NovaTextModel / LeanDecoderLayer on a transformers
Qwen3VLTextModel at Qwen3-VL-4B widths, with every linear replaced by the
arithmetic of the reference's NF4 GEMV (fp16 codebook x absmax, fp32
accumulation, fp16 out) and KVInt8Cache.attend replaced by the single-softmax
ground truth of the reference's streaming test (tests/test_kvattn_stream.py:
68-83); the rest of the cache runs unchanged).
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))
if not os.environ.get("NOVA_REF_SRC"):
    raise SystemExit("set NOVA_REF_SRC to the reference's src directory (the one containing nova/)")
sys.path.insert(0, os.environ["NOVA_REF_SRC"])

from torch.nn.attention import SDPBackend, sdpa_kernel  # noqa: E402

from nova.kernels import build_nf4_lut as ref_build_nf4_lut  # noqa: E402
from nova.kvattn import KVInt8Cache as RefCache  # noqa: E402
from nova.kvquant import dequantize_int8 as ref_dequant  # noqa: E402
from nova.kvquant import quantize_int8 as ref_quant  # noqa: E402
from nova.layers import apply_rotary_pos_emb as ref_rope  # noqa: E402
from nova.norm import LeanRMSNorm  # noqa: E402
from nova.quant import extract_nf4 as ref_extract_nf4  # noqa: E402

from oracle.nf4 import nf4_codebook, quantize_nf4  # noqa: E402  (inputs only)

H_KV, HQ, D, GT = 8, 32, 128, 64


def _save(name: str, **arrays) -> None:
    path = HERE / name
    np.savez_compressed(path, **{k: (v.numpy() if isinstance(v, torch.Tensor) else np.asarray(v))
                                 for k, v in arrays.items()})
    print(f"wrote {path.name}: {', '.join(arrays)}")


def kvquant_fixture() -> None:
    """quantize_int8 / dequantize_int8, token axis, group 64 (src/nova/kvquant.py:118-176)."""
    torch.manual_seed(0)
    out = {}
    cases = {
        "rand": (torch.randn(1, 3, 150, D) * 3.0).to(torch.float16),          # ragged last group
        "outlier": None,
        "const": torch.full((1, 2, 70, D), 0.5, dtype=torch.float16),
    }
    x = (torch.randn(1, 2, 129, D) * 0.7)
    x[..., [3, 71, 120]] *= 65.0
    cases["outlier"] = x.to(torch.float16)
    for name, x in cases.items():
        q, mn, st = ref_quant(x, GT, "token")
        deq = ref_dequant(q, mn, st, GT, "token")
        out.update({f"{name}_x": x, f"{name}_q": q, f"{name}_mn": mn, f"{name}_st": st, f"{name}_deq": deq})
    _save("kvquant_token.npz", **out)


def ring_fixture() -> None:
    """KVInt8Cache prefill + decode updates on CPU (src/nova/kvattn.py:645-783)."""
    torch.manual_seed(1)
    slots, hkv, max_len, n0, steps = 2, 2, 320, 100, 100
    cache = RefCache(num_slots=slots, num_kv_heads=hkv, head_dim=D, max_len=max_len, num_q_heads=4 * hkv,
                     device="cpu")
    k = (torch.randn(slots, 1, hkv, n0 + steps, D) * 0.7).to(torch.float16)
    v = (torch.randn(slots, 1, hkv, n0 + steps, D) * 0.7).to(torch.float16)
    cache.begin_prefill(n0)
    cache.set_prefill_pos(0)
    for layer in range(slots):
        cache.update(k[layer, :, :, :n0], v[layer, :, :, :n0], layer)
    cache.finish_prefill(n0)
    for p in range(n0, n0 + steps):
        cache.pos.fill_(p)
        for layer in range(slots):
            cache.update(k[layer, :, :, p:p + 1], v[layer, :, :, p:p + 1], layer)
    qlen = int(cache._qlen.item())
    out = {"k": k, "v": v, "n0": n0, "steps": steps, "max_len": max_len,
           "written": int(cache._written.item()), "qlen": qlen, "pg": int(cache._pg.item())}
    for layer in range(slots):
        out[f"kq{layer}"] = cache.kq[layer][:, :, :qlen]
        out[f"vq{layer}"] = cache.vq[layer][:, :, :qlen]
        for nm in ("kmn", "kst", "vmn", "vst"):
            out[f"{nm}{layer}"] = getattr(cache, nm)[layer][:, :, :qlen // GT]
        out[f"tail_k{layer}"] = cache.tail_k[layer]
        out[f"tail_v{layer}"] = cache.tail_v[layer]
    out["ring_mask"] = cache.ring_mask().view(-1)
    _save("kv_ring.npz", **out)


def _sdpa_math(q, k, v):
    gq = q.shape[1] // k.shape[1]
    b, h, n, d = k.shape
    k = k[:, :, None].expand(b, h, gq, n, d).reshape(b, h * gq, n, d)
    v = v[:, :, None].expand(b, h, gq, n, d).reshape(b, h * gq, n, d)
    with sdpa_kernel([SDPBackend.MATH]):
        return F.scaled_dot_product_attention(q, k, v, scale=d ** -0.5)


def attention_fixture() -> None:
    """The reference attention ground truths: fused kernel (dequantize_int8 ->
    SDPA math, tests/test_kvattn.py:62-71) and streaming cache (int8 prefix +
    fp16 tail -> SDPA math, tests/test_kvattn_stream.py:68-83)."""
    out = {}
    hkv, hq = 2, 8   # 4 query heads per KV head like Qwen3-4B, fewer heads to keep the fixture small
    for used in (7, 64, 65, 513, 1000):
        torch.manual_seed(used)
        k = (torch.randn(1, hkv, used, D) * 0.7).to(torch.float16)
        v = (torch.randn(1, hkv, used, D) * 0.7).to(torch.float16)
        q = (torch.randn(1, hq, 1, D) * 0.7).to(torch.float16)
        kq, kmn, kst = ref_quant(k, GT, "token")
        vq, vmn, vst = ref_quant(v, GT, "token")
        kk = ref_dequant(kq, kmn, kst, GT, "token")
        vv = ref_dequant(vq, vmn, vst, GT, "token")
        want = _sdpa_math(q, kk, vv)
        out.update({f"fused{used}_q": q, f"fused{used}_k": k, f"fused{used}_v": v, f"fused{used}_out": want})
    for used in (40, 100, 320):
        torch.manual_seed(1000 + used)
        k = (torch.randn(1, hkv, used, D) * 0.7).to(torch.float16)
        v = (torch.randn(1, hkv, used, D) * 0.7).to(torch.float16)
        q = (torch.randn(1, hq, 1, D) * 0.7).to(torch.float16)
        prefix = used // GT * GT
        if prefix:
            kq, kmn, kst = ref_quant(k[:, :, :prefix], GT, "token")
            vq, vmn, vst = ref_quant(v[:, :, :prefix], GT, "token")
            kk = torch.cat([ref_dequant(kq, kmn, kst, GT, "token"), k[:, :, prefix:]], dim=2)
            vv = torch.cat([ref_dequant(vq, vmn, vst, GT, "token"), v[:, :, prefix:]], dim=2)
        else:
            kk, vv = k, v
        out.update({f"stream{used}_q": q, f"stream{used}_k": k, f"stream{used}_v": v,
                    f"stream{used}_out": _sdpa_math(q, kk, vv)})
    _save("attention.npz", **out)


def nf4_fixture() -> None:
    """LUT packing (src/nova/kernels.py:170-182) and the extract_nf4 layout
    transform (src/nova/quant.py:39-69) applied to a non-nested quant state
    built from our own quantizer's output, plus the dequant formula of
    tests/test_nf4_linear.py:46-57."""
    code = nf4_codebook()
    lut = ref_build_nf4_lut(torch.from_numpy(code))
    rng = np.random.default_rng(7)
    n, k = 96, 256
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float16)
    packed, absmax = quantize_nf4(w, code, absmax_dtype=np.float32)   # [N, K/2], [K/64, N]

    class _QS:   # the fields extract_nf4 reads from a bitsandbytes QuantState
        nested = False

    qs = _QS()
    qs.shape = torch.Size([n, k])
    qs.absmax = torch.from_numpy(np.ascontiguousarray(absmax.T).reshape(-1))    # bnb order: block-major per row
    qs.code = torch.from_numpy(code)
    weight = torch.from_numpy(packed.reshape(-1).copy())
    r_packed, r_absmax, r_code, shape = ref_extract_nf4(weight, qs)
    # tests/test_nf4_linear.py:_torch_dequant, restated on CPU tensors
    hi = r_packed.long() >> 4
    lo = r_packed.long() & 0x0F
    vals = torch.empty(n, k, dtype=torch.float32)
    vals[:, 0::2] = r_code[hi]
    vals[:, 1::2] = r_code[lo]
    deq16 = (vals * r_absmax.t().repeat_interleave(64, dim=1)).to(torch.float16)
    _save("nf4.npz", code=code, lut=lut, w=w, packed=r_packed, absmax=r_absmax, deq16=deq16,
          shape=np.array(shape))


def norm_rope_fixture() -> None:
    """LeanRMSNorm "exact" (src/nova/norm.py:34-42) and RoPE with the
    transformers Qwen3-VL rotary (src/nova/model.py:144, src/nova/layers.py:24-36)."""
    from transformers import Qwen3VLTextConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLTextRotaryEmbedding

    torch.manual_seed(3)
    out = {}
    for dim, rows in ((2560, 5), (128, 40)):
        norm = LeanRMSNorm(dim, eps=1e-6, impl="exact", dtype=torch.float16)
        with torch.no_grad():
            norm.weight.copy_((1.0 + 0.1 * torch.randn(dim)).to(torch.float16))
        x = (torch.randn(rows, dim) * 2.0).to(torch.float16)
        out[f"norm{dim}_x"] = x
        out[f"norm{dim}_w"] = norm.weight.detach()
        out[f"norm{dim}_y"] = norm(x).detach()
    cfg = Qwen3VLTextConfig(hidden_size=4096, num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                            rope_parameters={"rope_type": "default", "rope_theta": 5_000_000.0,
                                             "mrope_section": [24, 20, 20], "mrope_interleaved": True})
    rot = Qwen3VLTextRotaryEmbedding(cfg)
    pos = torch.tensor([0, 1, 2, 63, 100, 4096, 8191, 8447, 32767, 131071])
    position_ids = pos.view(1, 1, -1).expand(3, 1, -1)
    dummy = torch.zeros(1, dtype=torch.float16)
    cos, sin = rot(dummy, position_ids)
    q = (torch.randn(1, 4, len(pos), 128)).to(torch.float16)
    k = (torch.randn(1, 2, len(pos), 128)).to(torch.float16)
    qe, ke = ref_rope(q, k, cos, sin)
    out.update({"rope_pos": pos, "rope_cos": cos[0], "rope_sin": sin[0], "rope_q": q, "rope_k": k,
                "rope_qe": qe, "rope_ke": ke})
    _save("norm_rope.npz", **out)


def sampling_fixture() -> None:
    """sample_next (src/chat.py:46-75): the top-k candidate ids and the final
    probabilities it hands to torch.multinomial (captured by wrapping
    torch.topk / torch.multinomial), for several argument sets; greedy
    (temperature 0) returns the argmax.  The 300 largest logits are distinct so
    that no tie sits at the top-k boundary."""
    import types
    os.environ.setdefault("TMPDIR", "/tmp")
    import chat as ref_chat

    V = 32768
    g = torch.Generator().manual_seed(5)
    cases = [(0.7, 20, 0.8, 1.05), (1.0, 0, 1.0, 1.0), (0.3, 50, 0.95, 1.3), (1.3, 256, 0.5, 1.0), (0.0, 20, 0.8, 1.05)]
    out = {}
    orig_topk, orig_mult = torch.topk, torch.multinomial
    for ci, (temp, top_k, top_p, rep) in enumerate(cases):
        logits = (torch.randn(V, generator=g) * 2.0).to(torch.float16)
        top = torch.randperm(V, generator=g)[:300]
        logits[top] = (torch.arange(300, dtype=torch.float32) * 0.03125 + 9.0).to(torch.float16)[torch.randperm(300, generator=g)]
        seen = torch.rand(V, generator=g) < 0.05
        seen[top[:40]] = True
        cap = {}

        def topk(x, k, **kw):
            r = orig_topk(x, k, **kw)
            cap["idx"] = r[1].clone()
            return r

        def multinomial(p, *a, **kw):
            cap["probs"] = p.clone()
            return orig_mult(p, *a, **kw)

        torch.topk, torch.multinomial = topk, multinomial
        try:
            args = types.SimpleNamespace(temperature=temp, top_k=top_k, top_p=top_p, repetition_penalty=rep)
            tok = ref_chat.sample_next(logits.view(1, V), args, seen, torch.Generator().manual_seed(ci))
        finally:
            torch.topk, torch.multinomial = orig_topk, orig_mult
        out[f"logits{ci}"] = logits
        out[f"seen{ci}"] = seen
        out[f"args{ci}"] = np.array([temp, top_k, top_p, rep], dtype=np.float64)
        out[f"token{ci}"] = tok.view(-1)
        if temp > 0:
            out[f"idx{ci}"] = cap["idx"].view(-1)
            out[f"probs{ci}"] = cap["probs"].view(-1)
    _save("sampling.npz", **out)


# decoder fixture: Qwen3-VL-4B widths, 2 layers, a smaller vocabulary (keeps the fixture and the CPU check small)
DECODER = dict(vocab=4096, hidden=2560, layers=2, q_heads=32, kv_heads=8, inter=9728)
DECODER_SEED, DECODER_PROMPT, DECODER_STEPS, DECODER_MAX_LEN = 20, 150, 72, 256


class _NF4GemvLinear(nn.Module):
    """The arithmetic of the reference's NF4 linear (src/nova/kernels.py:187-240
    with build_nf4_lut :170-182): W = fp16(code)[idx] * absmax, x in fp32,
    fp32 accumulation, fp16 output.  Layout as tests/test_nf4_linear.py:46-57
    (high nibble = even element)."""

    def __init__(self, packed: np.ndarray, absmax: np.ndarray, code: np.ndarray) -> None:
        super().__init__()
        pk = torch.from_numpy(np.ascontiguousarray(packed)).long()
        n, k2 = pk.shape
        c16 = torch.from_numpy(code).to(torch.float16).float()
        vals = torch.empty(n, 2 * k2, dtype=torch.float32)
        vals[:, 0::2] = c16[pk >> 4]
        vals[:, 1::2] = c16[pk & 0x0F]
        am = torch.from_numpy(np.ascontiguousarray(absmax)).float().t().repeat_interleave(64, dim=1)
        self.register_buffer("w", vals * am)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return (x.float() @ self.w.t()).to(torch.float16)


def _streaming_truth(self, query: torch.Tensor, layer_idx: int) -> torch.Tensor:
    """KVInt8Cache.attend ground truth (tests/test_kvattn_stream.py:68-83): the
    int8 prefix [0, _qlen) dequantized by the reference's dequantize_int8 and
    the ring tokens [_qlen, _written) in fp16, one softmax, fp32 math, fp16 out."""
    qlen, written = int(self._qlen.item()), int(self._written.item())
    ks, vs = [], []
    if qlen:
        g = qlen // self.group
        ks.append(ref_dequant(self.kq[layer_idx][:, :, :qlen], self.kmn[layer_idx][:, :, :g],
                              self.kst[layer_idx][:, :, :g], self.group, "token"))
        vs.append(ref_dequant(self.vq[layer_idx][:, :, :qlen], self.vmn[layer_idx][:, :, :g],
                              self.vst[layer_idx][:, :, :g], self.group, "token"))
    slots = torch.arange(qlen, written) % self.group
    ks.append(self.tail_k[layer_idx][:, :, slots])
    vs.append(self.tail_v[layer_idx][:, :, slots])
    k, v = torch.cat(ks, dim=2).float(), torch.cat(vs, dim=2).float()
    b, h, n, d = k.shape
    gq = query.shape[1] // h
    k = k[:, :, None].expand(b, h, gq, n, d).reshape(b, h * gq, n, d)
    v = v[:, :, None].expand(b, h, gq, n, d).reshape(b, h * gq, n, d)
    with sdpa_kernel([SDPBackend.MATH]):
        out = F.scaled_dot_product_attention(query.float(), k, v, scale=d ** -0.5)
    return out.to(torch.float16)


def decoder_fixture() -> None:
    """The reference's int8 greedy decode (GraphDecoder, src/nova/decode.py:
    224-320) on a random-init model: prompt prefill, then eager ``_body`` steps
    (the step the reference captures), logits and greedy tokens saved."""
    from transformers import Qwen3VLTextConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLTextModel, Qwen3VLTextRotaryEmbedding

    from nova.config import NovaConfig
    from nova.decode import GraphDecoder
    from nova.model import NovaForCausalLM, NovaTextModel
    from oracle.decoder import random_weights   # inputs only: the seeded NF4 weights

    c = DECODER
    W = random_weights(**c, seed=DECODER_SEED)
    hcfg = Qwen3VLTextConfig(vocab_size=c["vocab"], hidden_size=c["hidden"], intermediate_size=c["inter"],
                             num_hidden_layers=c["layers"], num_attention_heads=c["q_heads"],
                             num_key_value_heads=c["kv_heads"], head_dim=D, rms_norm_eps=1e-6,
                             rope_parameters={"rope_type": "default", "rope_theta": 5_000_000.0,
                                              "mrope_section": [24, 20, 20], "mrope_interleaved": True})
    torch.manual_seed(0)
    hf = Qwen3VLTextModel(hcfg).to(torch.float16).eval()
    # from_pretrained(dtype=float16), as the reference loads the model (src/nova/loader.py:29-42),
    # leaves the rotary's inv_freq buffer in fp32; .to(float16) above rounded it, so rebuild it
    hf.rotary_emb = Qwen3VLTextRotaryEmbedding(hcfg)
    code = W["code"]
    qd, kvd = c["q_heads"] * D, c["kv_heads"] * D
    with torch.no_grad():
        hf.embed_tokens.weight.copy_(torch.from_numpy(W["embed"]))
        hf.norm.weight.copy_(torch.from_numpy(W["final_norm"]))
        for layer, lw in zip(hf.layers, W["layers"]):
            layer.input_layernorm.weight.copy_(torch.from_numpy(lw["input_ln"]))
            layer.post_attention_layernorm.weight.copy_(torch.from_numpy(lw["post_ln"]))
            layer.self_attn.q_norm.weight.copy_(torch.from_numpy(lw["q_norm"]))
            layer.self_attn.k_norm.weight.copy_(torch.from_numpy(lw["k_norm"]))
            pk, am = lw["qkv"]
            for name, r0, r1 in (("q_proj", 0, qd), ("k_proj", qd, qd + kvd), ("v_proj", qd + kvd, qd + 2 * kvd)):
                setattr(layer.self_attn, name, _NF4GemvLinear(pk[r0:r1], am[:, r0:r1], code))
            layer.self_attn.o_proj = _NF4GemvLinear(*lw["o"], code)
            layer.mlp.gate_proj = _NF4GemvLinear(*lw["gate"], code)
            layer.mlp.up_proj = _NF4GemvLinear(*lw["up"], code)
            layer.mlp.down_proj = _NF4GemvLinear(*lw["down"], code)
    ncfg = NovaConfig.from_hf(hcfg, num_prefix_layers=1, num_suffix_layers=0, num_paths=1)
    nova = NovaForCausalLM(NovaTextModel(hf, ncfg, norm_impl="exact")).eval()
    nova.lm_head4 = _NF4GemvLinear(*W["lm_head"], code)
    RefCache.attend = _streaming_truth
    dec = GraphDecoder(nova, max_len=DECODER_MAX_LEN, batch=1, device="cpu", quant="int8")
    prompt = torch.randint(0, c["vocab"], (1, DECODER_PROMPT), generator=torch.Generator().manual_seed(DECODER_SEED))
    tokens, logits = [], []
    with torch.inference_mode():
        out = dec.prefill(prompt)
        prefill_logits = out[0, -1].clone()
        tokens.append(int(dec.input_ids.item()))
        cache, q = dec.cache, DECODER_PROMPT // GT * GT
        state = {}   # the cache after the prefill, so the decode steps can be checked on their own
        for li in range(c["layers"]):
            for nm in ("kq", "vq"):
                state[f"state_{nm}{li}"] = getattr(cache, nm)[li][:, :, :q].clone()
            for nm in ("kmn", "kst", "vmn", "vst"):
                state[f"state_{nm}{li}"] = getattr(cache, nm)[li][:, :, :q // GT].clone()
            state[f"state_tail_k{li}"] = cache.tail_k[li].clone()
            state[f"state_tail_v{li}"] = cache.tail_v[li].clone()
        for _ in range(DECODER_STEPS):
            lg = dec._body()
            logits.append(lg[0, -1].clone())
            tokens.append(int(dec.input_ids.item()))
    _save("decoder.npz", prompt=prompt[0], prefill_logits=prefill_logits, tokens=np.array(tokens, np.int64),
          logits=torch.stack(logits), seed=DECODER_SEED, max_len=DECODER_MAX_LEN,
          dims=np.array([c[k] for k in ("vocab", "hidden", "layers", "q_heads", "kv_heads", "inter")]), **state)


def main() -> None:
    which = set(sys.argv[1:]) or {"kvquant", "ring", "attention", "nf4", "norm_rope", "sampling", "decoder"}
    if "kvquant" in which:
        kvquant_fixture()
    if "ring" in which:
        ring_fixture()
    if "attention" in which:
        attention_fixture()
    if "nf4" in which:
        nf4_fixture()
    if "norm_rope" in which:
        norm_rope_fixture()
    if "sampling" in which:
        sampling_fixture()
    if "decoder" in which:
        decoder_fixture()


if __name__ == "__main__":
    main()
