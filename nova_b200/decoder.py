"""Lean Qwen3-VL-4B text decoder on B200: NF4 weights, streaming int8 KV,
greedy decode captured in one CUDA graph.

This is the B200 counterpart of the reference's graph-decode path:
``GraphDecoder`` (src/nova/decode.py:87-526) driving ``NovaTextModel`` /
``LeanDecoderLayer`` (src/nova/model.py:115-204, src/nova/layers.py:99-218)
with ``KVInt8Cache`` (src/nova/kvattn.py:488-880) and NF4 linears
(src/nova/quant.py).  One decode step is 5 kernel launches per layer plus
one for the lm_head:

    1. nova_nf4_gemv      input_layernorm (prologue) + fused q|k|v projection
    2. nova_qk_append_attn_int8   q_norm/k_norm, RoPE, ring write, group requant
                          (prologue), then int8 prefix + fp16 ring attention,
                          split-K, merged
    3. nova_nf4_gemv      o_proj + residual add (epilogue, in place)
    4. nova_nf4_gemv      post_attention_layernorm (prologue) + gate|up + SiLU*up
    5. nova_nf4_gemv      down_proj + residual add

(``attn_fused=False`` runs step 2 as nova_qk_norm_rope_append followed by
nova_attn_decode_int8.)
    final: nova_nf4_gemv  final norm (prologue) + 4-bit lm_head + greedy argmax
           + input_ids / pos update + next-token embedding gather (last warp)

Weights: the reference keeps q/k/v and gate/up as separate modules; here
q|k|v are concatenated row-wise and gate|up are interleaved per 16-row tile
(8 gate rows, then the same 8 up rows) so one GEMV produces SiLU(gate)*up.
The tied lm_head is the NF4 copy of ``embed_tokens`` (src/nova/loader.py:67-119).

Tensor parallelism (``tp=TPContext(rank, world, group)``): each rank holds
its KV heads and intermediate slice (``nova_b200.tp``); o_proj and down_proj
write fp32 partial sums (``NOVA_NF4_F32``), an NCCL all-reduce inside the
graph sums them and ``nova_residual_add_f32`` adds them to the replicated
residual stream: 8 launches per layer of this library plus 2 all-reduces.

Prefill (not the hot path) runs eagerly on this library's kernels: the
batched NF4 GEMM on the tensor cores in 64-row launches (with the decode
step's residual / SiLU*up epilogues), nova_rmsnorm, nova_qk_prefill (q/k norm
+ RoPE) and nova_attn_prefill_int8 (causal attention over the int8 prefix in
place and the fp16 keys); then the complete 64-token groups of every layer's
K/V are quantized with ``nova_kv_quant_int8`` and the tail goes to the fp16
ring (same result as ``KVInt8Cache.finish_prefill``).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import _lib
from .kernels import (build_nf4_lut, gemm_workspace, gemv_workspace, nf4_gemm, nf4_gemv, pack_native, pack_tc,
                      slots_buffer, edge_buffer, heads_major)
from .kvattn import CHUNK, GROUP_T, KVInt8Cache, attn_partials, launch_attention, pick_chunk, prefill_attention
from .quant import nf4_codebook, quantize_nf4
from .tp import P2PAllReduce, TPContext, all_reduce_sum, shard_ranges, shard_weights


MAX_BATCH = 64
GEMV_ROWS = 8   # rows per nova_nf4_gemv launch; larger batches use the batched GEMM (nova_nf4_gemm)


@dataclass
class DecoderConfig:
    """Qwen3-VL-4B text tower dimensions (src/nova/config.py:14-37)."""

    vocab_size: int = 151936
    hidden_size: int = 2560
    num_hidden_layers: int = 36
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 9728
    rms_norm_eps: float = 1e-6
    rope_theta: float = 5_000_000.0

    @property
    def q_dim(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_key_value_heads * self.head_dim


def interleave_gate_up(gate_p, gate_a, up_p, up_a):
    """Interleave gate and up NF4 weights per 16-row tile: rows 16r..16r+7 =
    gate rows 8r..8r+7, rows 16r+8..16r+15 = up rows 8r..8r+7 (the layout the
    SILU_MUL epilogue expects).  packed ``[N, K/2]``, absmax ``[K/64, N]``."""
    n, k2 = gate_p.shape
    if n % 8:
        raise ValueError("intermediate size must be a multiple of 8")
    packed = torch.stack([gate_p.view(n // 8, 8, k2), up_p.view(n // 8, 8, k2)], dim=1).reshape(2 * n, k2)
    kb = gate_a.shape[0]
    absmax = torch.stack([gate_a.view(kb, n // 8, 8), up_a.view(kb, n // 8, 8)], dim=2).reshape(kb, 2 * n)
    return packed.contiguous(), absmax.contiguous()


def deinterleave_gate_up(packed, absmax):
    """Inverse of :func:`interleave_gate_up` -> (gate_p, gate_a, up_p, up_a)."""
    n2, k2 = packed.shape
    n = n2 // 2
    p = packed.view(n // 8, 2, 8, k2)
    kb = absmax.shape[0]
    a = absmax.view(kb, n // 8, 2, 8)
    return (p[:, 0].reshape(n, k2), a[:, :, 0].reshape(kb, n), p[:, 1].reshape(n, k2), a[:, :, 1].reshape(kb, n))


@dataclass
class NF4Weight:
    packed: torch.Tensor               # uint8 [N, K/2] (reference layout; prefill, tests)
    absmax: torch.Tensor               # fp16 [K/64, N]
    units: torch.Tensor | None = None  # B200-native unit stream (decode GEMVs)
    tc: torch.Tensor | None = None     # unit stream of the tcgen05 GEMM (batched decode), made on demand

    def __post_init__(self) -> None:
        if self.units is None:
            self.units = pack_native(self.packed, self.absmax)

    def tc_units(self) -> torch.Tensor:
        if self.tc is None:
            self.tc = pack_tc(self.packed, self.absmax)
        return self.tc

    @property
    def n(self) -> int:
        return int(self.packed.shape[0])

    @property
    def shape(self):
        return self.packed.shape[0], self.packed.shape[1] * 2

    @property
    def stream_bytes(self) -> int:
        """Bytes one GEMV streams: NF4 codes + fp16 absmax."""
        return int(self.units.numel())


@dataclass
class LayerWeights:
    qkv: NF4Weight          # [q_dim + 2 kv_dim, hidden]
    o: NF4Weight            # [hidden, q_dim]
    gate_up: NF4Weight      # [2 inter, hidden], interleaved
    down: NF4Weight         # [hidden, inter]
    input_ln: torch.Tensor  # fp16 [hidden]
    post_ln: torch.Tensor
    q_norm: torch.Tensor    # fp16 [head_dim]
    k_norm: torch.Tensor


@dataclass
class DecoderWeights:
    cfg: DecoderConfig
    embed: torch.Tensor          # fp16 [vocab, hidden]
    lm_head: NF4Weight           # NF4 copy of embed (tied)
    final_norm: torch.Tensor
    layers: list = field(default_factory=list)
    code: torch.Tensor | None = None

    @classmethod
    def random_init(cls, cfg: DecoderConfig, seed: int = 0, device="cuda", std: float = 0.02,
                    norm_jitter: float = 0.0) -> "DecoderWeights":
        """Random-init weights like the HF initializer (normal(0, std) for
        linear and embedding weights, RMSNorm weights 1), quantized to NF4
        (blocksize 64, fp16 absmax).  ``norm_jitter`` > 0 perturbs the norm
        weights (1 + jitter*N(0,1)) to exercise them in tests."""
        g = torch.Generator(device=device).manual_seed(seed)
        code = nf4_codebook()

        def lin(n, k):
            w = (torch.randn(n, k, generator=g, device=device, dtype=torch.float32) * std).to(torch.float16)
            p, a = quantize_nf4(w, code)
            return p, a

        def nw(n):
            if norm_jitter:
                return (1.0 + norm_jitter * torch.randn(n, generator=g, device=device)).to(torch.float16)
            return torch.ones(n, dtype=torch.float16, device=device)

        layers = []
        for _ in range(cfg.num_hidden_layers):
            qp, qa = lin(cfg.q_dim, cfg.hidden_size)
            kp, ka = lin(cfg.kv_dim, cfg.hidden_size)
            vp, va = lin(cfg.kv_dim, cfg.hidden_size)
            op, oa = lin(cfg.hidden_size, cfg.q_dim)
            gp, ga = lin(cfg.intermediate_size, cfg.hidden_size)
            up, ua = lin(cfg.intermediate_size, cfg.hidden_size)
            dp, da = lin(cfg.hidden_size, cfg.intermediate_size)
            gu_p, gu_a = interleave_gate_up(gp, ga, up, ua)
            layers.append(LayerWeights(
                qkv=NF4Weight(torch.cat([qp, kp, vp]), torch.cat([qa, ka, va], dim=1).contiguous()),
                o=NF4Weight(op, oa), gate_up=NF4Weight(gu_p, gu_a), down=NF4Weight(dp, da),
                input_ln=nw(cfg.hidden_size), post_ln=nw(cfg.hidden_size),
                q_norm=nw(cfg.head_dim), k_norm=nw(cfg.head_dim)))
        embed = (torch.randn(cfg.vocab_size, cfg.hidden_size, generator=g, device=device) * std).to(torch.float16)
        lp, la = quantize_nf4(embed, code)
        return cls(cfg=cfg, embed=embed, lm_head=NF4Weight(lp, la), final_norm=nw(cfg.hidden_size), layers=layers,
                   code=code)

    def nbytes_per_token(self) -> int:
        """Weight bytes one decode step streams (NF4 codes + fp16 absmax)."""
        tot = sum(w.stream_bytes for lw in self.layers for w in (lw.qkv, lw.o, lw.gate_up, lw.down))
        return tot + self.lm_head.stream_bytes


def rope_tables(max_pos: int, head_dim: int = 128, theta: float = 5_000_000.0, device="cuda"):
    """fp16 cos/sin ``[max_pos, head_dim]`` computed exactly like the HF
    rotary for text tokens (fp32 inv_freq = 1/theta**(2i/d), fp32 pos*inv_freq,
    cat(freqs, freqs), fp32 cos/sin, cast to fp16), on the CPU."""
    e = torch.arange(0, head_dim, 2, dtype=torch.int64).to(dtype=torch.float) / head_dim
    inv = 1.0 / (theta ** e)
    pos = torch.arange(max_pos, dtype=torch.float32)
    freqs = pos[:, None] * inv[None, :]
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(torch.float16).to(device), emb.sin().to(torch.float16).to(device)


class NovaDecoder:
    """Greedy graph decoder (src/nova/decode.py:87-526) for the NF4 / int8-KV
    Qwen3-VL text model.

        dec = NovaDecoder(weights, max_len=8448, batch=1)
        dec.prefill(prompt_ids)      # eager; fills the int8 cache, sets input_ids
        dec.capture()                # one decode step -> CUDA graph
        for _ in range(n): dec.step()  # one replay = one token per row

    ``input_ids`` (int64 ``[batch]``) holds the latest greedy token and ``pos``
    the next position, like the reference's ``GraphDecoder``; ``logits``
    (fp16 ``[batch, vocab]``) the last step's logits.
    """

    def __init__(self, weights: DecoderWeights, max_len: int, batch: int = 1, chunk: int | None = None,
                 device="cuda", pdl: bool = True, tp: TPContext | None = None, attn_fused: bool = True) -> None:
        cfg = weights.cfg
        if batch < 1 or batch > MAX_BATCH:
            raise ValueError(f"the decode path handles batch 1..{MAX_BATCH}")
        self.tp = tp if tp is not None else TPContext()
        sr = shard_ranges(cfg, self.tp.rank, self.tp.world)
        self.w = shard_weights(weights, self.tp.rank, self.tp.world) if self.tp.active else weights
        self.cfg = cfg
        # this rank's dimensions (the whole model without tensor parallelism)
        self.hq = sr.q_heads[1] - sr.q_heads[0]
        self.hkv = sr.kv_heads[1] - sr.kv_heads[0]
        self.q_dim, self.kv_dim = self.hq * cfg.head_dim, self.hkv * cfg.head_dim
        self.inter = sr.inter[1] - sr.inter[0]
        self.batch = int(batch)
        self.max_len = int(max_len)
        self.device = torch.device(device)
        if chunk is None:
            chunk = self._pick_chunk()
        self.cache = KVInt8Cache(num_slots=cfg.num_hidden_layers, num_kv_heads=self.hkv,
                                 head_dim=cfg.head_dim, max_len=self.max_len, num_q_heads=self.hq,
                                 batch=self.batch, device=self.device, chunk=chunk)
        self.lut = build_nf4_lut(weights.code if weights.code is not None else nf4_codebook()).to(self.device)
        self.cos, self.sin = rope_tables(self.max_len + 1, cfg.head_dim, cfg.rope_theta, self.device)
        B, dev, f16 = self.batch, self.device, torch.float16
        self.resid = torch.zeros(B, cfg.hidden_size, dtype=f16, device=dev)
        self.qkv = torch.zeros(B, self.q_dim + 2 * self.kv_dim, dtype=f16, device=dev)
        self.q_rot = torch.zeros(B, self.q_dim, dtype=f16, device=dev)
        self.attn = torch.zeros(B, self.q_dim, dtype=f16, device=dev)
        self.act = torch.zeros(B, self.inter, dtype=f16, device=dev)
        self.part32 = torch.zeros(B, cfg.hidden_size, dtype=torch.float32, device=dev) if self.tp.active else None
        self.p2p = (P2PAllReduce(self.tp, B, cfg.hidden_size, dev)
                    if self.tp.active and self.tp.allreduce == "p2p" else None)
        self.logits = torch.zeros(B, cfg.vocab_size, dtype=f16, device=dev)
        self.argmax_slot = torch.zeros(B, dtype=torch.int64, device=dev)
        self.input_ids = torch.zeros(B, dtype=torch.int64, device=dev)
        n_max = max(cfg.vocab_size, 2 * self.inter, self.q_dim + 2 * self.kv_dim, cfg.hidden_size,
                    self.hkv * cfg.hidden_size)
        self.gemv_ws = gemv_workspace(dev, n_max).clone()   # shared by every GEMV of the step
        # batched GEMM (decode above 8 rows, and every prefill): one workspace for every shape
        shapes = [(self.q_dim + 2 * self.kv_dim, cfg.hidden_size), (cfg.hidden_size, self.q_dim),
                  (2 * self.inter, cfg.hidden_size), (cfg.hidden_size, self.inter), (cfg.vocab_size, cfg.hidden_size)]
        self.gemm_ws = max((gemm_workspace(dev, n, k) for n, k in shapes), key=lambda t: t.numel()).clone()
        if self.batch > GEMV_ROWS:   # decode GEMM units packed before any graph capture; normalized-x scratch
            for w in [self.w.lm_head] + [x for lw in self.w.layers for x in (lw.qkv, lw.o, lw.gate_up, lw.down)]:
                w.tc_units()
            self.xn = torch.zeros(B, cfg.hidden_size, dtype=f16, device=dev)
        else:
            self.xn = None
        self.graph: torch.cuda.CUDAGraph | None = None
        self.pdl = bool(pdl)
        # attn_fused=True: the q/k norm + RoPE + ring append runs in the attention's prologue (one launch
        # and one kernel boundary fewer per layer)
        self.attn_fused = bool(attn_fused)
        # batch 1 on one GPU (when the shapes fit): o_proj and down_proj run on every SM over equal shares of
        # their k-blocks and leave fp32 sums per CTA (NF4_SLOTS); the next GEMV adds them to the residual while
        # it stages its input, alternating between two residual buffers.  Otherwise (tensor parallelism,
        # batches above 1) they add into the residual in their own epilogue.
        self.deferred = self.batch == 1 and not self.tp.active and self._deferred_fits()
        self.slots = slots_buffer(self.device) if self.deferred else None
        self.resid_alt = torch.zeros_like(self.resid) if self.deferred else None
        # with the deferred reductions, gate|up also leaves the row groups split between its CTAs as fp32
        # sums (edge_out) that down_proj completes while staging its input: no cross-CTA reduction
        self.edges = edge_buffer(self.device) if self.deferred and self._edges_fit() else None
        # and the attention leaves its split partials to o_proj, which merges each KV head's while staging
        # its input (head-aligned CTAs over a head-major copy of o_proj) and writes fp32 sums per head that
        # gate|up adds: the attention launch has no arrival counters and no per-head merge
        self.heads = self.deferred and self._heads_fit()
        self.y_heads = (torch.zeros(self.hkv, cfg.hidden_size, dtype=torch.float32, device=self.device)
                        if self.heads else None)
        self.o_heads = ([heads_major(lw.o.units, cfg.hidden_size, self.q_dim, self.hkv) for lw in self.w.layers]
                        if self.heads else None)
        self._staged = None   # fp16 K/V per layer of the positions prefilled / injected since the last reset

    def _deferred_fits(self) -> bool:
        """The deferred reduction's shape limits (nova_nf4_gemv with NF4_SLOTS /
        add_slots): at most one row group per SM, at most four CTAs per row
        group, and the consumer's input in one 8-column chunk per thread."""
        h = self.cfg.hidden_size
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        if h % 32 or h // 32 > sms or h // 8 > 512:
            return False
        for k in (self.q_dim, self.inter):
            kb = k // 64
            units = (h // 32) * kb
            if k % 64 or (kb - 1) * sms // units + 2 > 4 or (units + kb) * sms >= 2 ** 31:
                return False
        return True

    def _edges_fit(self) -> bool:
        """gate|up's edge_out limits (nova_nf4_gemv): every warp of every SM
        busy (8 units each at least), 2 to 15 row groups per SM."""
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        kb = self.cfg.hidden_size // 64
        units = (2 * self.inter // 32) * kb
        per = -(-units // sms)
        return (units >= 8 * 16 * sms and units // sms >= 2 * kb and -(-per // kb) + 1 <= 16
                and 2 * (sms - 1) <= 512 and (units + 1) * 16 * sms < 2 ** 31)

    def _heads_fit(self) -> bool:
        """o_proj's attn_part limits (nova_nf4_gemv): head_dim 128, 1 to 4 q
        heads per KV head, at most 40 splits (with the ring), and 1 to 15 row
        groups of each head per SM with 16 units per SM at least."""
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        h, hkv = self.cfg.hidden_size, self.hkv
        gq = self.hq // hkv
        if self.cfg.head_dim != 128 or not 1 <= gq <= 4 or self.cache.n_splits + 1 > 40 or hkv > sms or h % 32:
            return False
        rg, nmax = h // 32, -(-sms // hkv)
        return rg >= nmax and rg // (sms // hkv) + 1 <= 16 and (rg // nmax) * 2 * gq >= 16

    def _pick_chunk(self) -> int:
        """Split size for the attention (``kvattn.pick_chunk``)."""
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        return pick_chunk(self.max_len, self.batch, self.hkv, self.hq, sms)

    @property
    def pos(self) -> torch.Tensor:
        return self.cache.pos

    # ---------------------------------------------------------------- prefill

    PREFILL_ROWS = 4096   # rows per batched-GEMM launch in the prefill (the wide tcgen05 kernel above 64)

    def _norm(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """RMSNorm of the rows of x ``[R, n]`` (nova_rmsnorm)."""
        y = torch.empty_like(x)
        _lib.call("nova_rmsnorm", x.data_ptr(), x.stride(0), None, 0, None, 0, w.data_ptr(), y.data_ptr(),
                  y.stride(0), x.shape[0], x.shape[1], float(self.cfg.rms_norm_eps), _lib.stream_of(self.device))
        return y

    def _gemm_rows(self, x: torch.Tensor, w: NF4Weight, out: torch.Tensor, epilogue: int = _lib.NF4_PLAIN,
                   residual: torch.Tensor | None = None) -> torch.Tensor:
        """x ``[R, K]`` @ W^T into out, PREFILL_ROWS rows per nova_nf4_gemm launch
        (the tcgen05 tensor cores, fp32 accumulation, the decode step's epilogues)."""
        units = w.tc_units()
        for r0 in range(0, x.shape[0], self.PREFILL_ROWS):
            sl = slice(r0, min(x.shape[0], r0 + self.PREFILL_ROWS))
            nf4_gemm(x[sl], units, self.lut, out[sl], n=w.n, epilogue=epilogue,
                     residual=None if residual is None else residual[sl], workspace=self.gemm_ws)
        return out

    def _row_parallel_add(self, x: torch.Tensor, w: NF4Weight, h: torch.Tensor) -> None:
        """h += x @ W^T for o_proj / down_proj (h ``[R, H]`` fp16, in place): the
        residual epilogue, or with tensor parallelism the fp32 partial sums of
        every rank all-reduced, then one fp16 rounding and the residual add."""
        if not self.tp.active:
            self._gemm_rows(x, w, h, epilogue=_lib.NF4_RESIDUAL, residual=h)
            return
        part = torch.empty(x.shape[0], w.n, dtype=torch.float32, device=self.device)
        self._gemm_rows(x, w, part, epilogue=_lib.NF4_F32)
        all_reduce_sum(part, self.tp)
        _lib.call("nova_residual_add_f32", part.data_ptr(), part.stride(0), h.data_ptr(), h.stride(0), h.shape[0],
                  h.shape[1], _lib.stream_of(self.device))

    def _layer_qkv(self, li: int, lw, h: torch.Tensor, pos0: int, want_pre: bool = False):
        """Prefill projections of layer li for hidden states h ``[B, T, H]`` at
        positions pos0 .. pos0 + T - 1: q (RoPE applied, ``[B, Hq, T, D]``), k
        after k_norm before RoPE (``want_pre``, else None), k after RoPE and v
        (``[B, Hkv, T, D]``).  Input norm, the q|k|v GEMM and nova_qk_prefill."""
        cfg = self.cfg
        B, T, H = h.shape
        d = cfg.head_dim
        x = self._norm(h.view(B * T, H), lw.input_ln)
        qkv = self._gemm_rows(x, lw.qkv, torch.empty(B * T, lw.qkv.n, dtype=torch.float16, device=self.device))
        f16 = dict(dtype=torch.float16, device=self.device)
        q = torch.empty(B, self.hq, T, d, **f16)
        k = torch.empty(B, self.hkv, T, d, **f16)
        v = torch.empty(B, self.hkv, T, d, **f16)
        k_pre = torch.empty(B, self.hkv, T, d, **f16) if want_pre else None
        a = _lib.QKPrefillArgs()
        a.qkv, a.qkv_b_stride, a.qkv_t_stride = qkv.data_ptr(), T * lw.qkv.n, lw.qkv.n
        a.q_norm_weight, a.k_norm_weight, a.eps = lw.q_norm.data_ptr(), lw.k_norm.data_ptr(), cfg.rms_norm_eps
        a.cos, a.sin, a.rope_len = self.cos.data_ptr(), self.sin.data_ptr(), self.cos.shape[0]
        a.q_out, a.k_out, a.k_pre, a.v_out = q.data_ptr(), k.data_ptr(), _lib.ptr(k_pre), v.data_ptr()
        a.q_b_stride, a.q_h_stride = q.stride(0), q.stride(1)
        a.kv_b_stride, a.kv_h_stride = k.stride(0), k.stride(1)
        a.batch, a.q_heads, a.kv_heads, a.head_dim, a.n, a.pos0 = B, self.hq, self.hkv, d, T, int(pos0)
        _lib.check(_lib.lib().nova_qk_prefill(_lib.ctypes.byref(a), _lib.stream_of(self.device)), "nova_qk_prefill")
        return q, k_pre, k, v

    def _attend_prefill(self, li: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, prefix: int,
                        int8_len: int = 0) -> torch.Tensor:
        """Causal attention of the chunk queries q ``[B, Hq, n, D]`` at positions
        [prefix, prefix + n) over positions [0, int8_len) of layer li's int8
        cache and the fp16 k / v ``[B, Hkv, *, D]`` of [int8_len, prefix + n)
        (nova_attn_prefill_int8) -> ``[B, n, Hq * D]``."""
        c = self.cache
        int8 = (c.kq[li], c.kmn[li], c.kst[li], c.vq[li], c.vmn[li], c.vst[li]) if int8_len else None
        return prefill_attention(q, k, v, prefix=prefix, int8=int8, int8_len=int8_len)

    def _layer_rest(self, lw, h: torch.Tensor, o: torch.Tensor) -> None:
        """o_proj + residual, post-attention norm, gate|up with SiLU*up, down_proj
        + residual, in place on h ``[B, T, H]`` (o ``[B, T, Hq * D]``)."""
        B, T, H = h.shape
        h2 = h.view(B * T, H)
        self._row_parallel_add(o.view(B * T, -1), lw.o, h2)
        x = self._norm(h2, lw.post_ln)
        act = self._gemm_rows(x, lw.gate_up, torch.empty(B * T, self.inter, dtype=torch.float16, device=self.device),
                              epilogue=_lib.NF4_SILU_MUL)
        self._row_parallel_add(act, lw.down, h2)

    def _first_token(self, h_last: torch.Tensor) -> torch.Tensor:
        """Final norm + 4-bit lm_head + greedy argmax of the prompt's last
        position (the decode step's ARGMAX epilogue), the token's embedding as
        the next step's input."""
        self.argmax_slot.zero_()
        self._gemv(h_last, self.w.lm_head, self.logits, epilogue=_lib.NF4_ARGMAX, norm_weight=self.w.final_norm,
                   argmax=self.argmax_slot, token_out=self.input_ids, embed=self.w.embed, embed_out=self.resid)
        return self.input_ids.clone()

    def _commit_kv(self, li: int, k: torch.Tensor, v: torch.Tensor, total: int) -> None:
        """Quantize the complete 64-token groups of the fp16 K/V ``[B, Hkv, total, D]``
        into layer li's int8 cache and put the last <= 64 tokens into the ring
        (src/nova/kvattn.py:745-783)."""
        cache, d = self.cache, self.cfg.head_dim
        q_full = (total // GROUP_T) * GROUP_T
        stream = _lib.stream_of(self.device)
        if q_full:
            for src, dst, mn, st in ((k, cache.kq[li], cache.kmn[li], cache.kst[li]),
                                     (v, cache.vq[li], cache.vmn[li], cache.vst[li])):
                _lib.call("nova_kv_quant_int8", src.data_ptr(), src.stride(1), dst.data_ptr(), self.max_len * d,
                          mn.data_ptr(), st.data_ptr(), mn.shape[2] * d, self.batch * self.hkv, q_full, d, GROUP_T,
                          stream)
        cache.write_ring(li, k[:, :, :total], v[:, :, :total], total)

    def _set_scalars(self, total: int) -> None:
        self.cache.set_lengths(total)
        self.argmax_slot.zero_()

    def _dequant_prefix(self, li: int, n: int) -> tuple[torch.Tensor, torch.Tensor]:
        """fp16 K/V ``[B, Hkv, n, D]`` of the first n (a multiple of 64) cached
        positions of layer li, dequantized from the int8 cache
        (``nova_kv_dequant_int8``, src/nova/kvquant.py:152-176)."""
        cache, d = self.cache, self.cfg.head_dim
        stream = _lib.stream_of(self.device)
        outs = []
        for codes, mn, st in ((cache.kq[li], cache.kmn[li], cache.kst[li]), (cache.vq[li], cache.vmn[li], cache.vst[li])):
            out = torch.empty(self.batch, self.hkv, n, d, dtype=torch.float16, device=self.device)
            _lib.call("nova_kv_dequant_int8", codes.data_ptr(), self.max_len * d, mn.data_ptr(), st.data_ptr(),
                      mn.shape[2] * d, out.data_ptr(), n * d, self.batch * self.hkv, n, d, GROUP_T, stream)
            outs.append(out)
        return outs[0], outs[1]

    def _prefill_chunked(self, input_ids: torch.Tensor, chunk: int) -> torch.Tensor:
        """Prefill in chunks of ``chunk`` tokens (a multiple of 64) straight into
        the int8 cache, the reference's planned replacement of its whole-prompt
        fp16 staging (reports/kv-int8-streaming-cache.md, section 5.1): each
        chunk attends to the int8 prefix of the earlier chunks (dequantized one
        layer at a time) and to its own fp16 K/V, causally; its complete
        64-token groups are quantized when the layer is done, the last <= 64
        tokens of the prompt go into the ring.  No fp16 K/V outlives a layer."""
        cfg, cache = self.cfg, self.cache
        B, T = input_ids.shape
        ids = input_ids.to(self.device)
        d = cfg.head_dim
        stream = _lib.stream_of(self.device)
        take0 = T - min(T, GROUP_T)   # first position that goes into the ring
        h = None
        for c0 in range(0, T, chunk):
            c1 = min(T, c0 + chunk)
            n = c1 - c0
            h = torch.index_select(self.w.embed, 0, ids[:, c0:c1].reshape(-1)).view(B, n, -1)
            for li, lw in enumerate(self.w.layers):
                q, _, k, v = self._layer_qkv(li, lw, h, c0)
                o = self._attend_prefill(li, q, k, v, prefix=c0, int8_len=c0)
                self._layer_rest(lw, h, o)
                full = (n // GROUP_T) * GROUP_T   # complete groups of this chunk (chunk starts are group-aligned)
                if full:
                    g0 = c0 // GROUP_T
                    for src, dst, mn, st in ((k, cache.kq[li], cache.kmn[li], cache.kst[li]),
                                             (v, cache.vq[li], cache.vmn[li], cache.vst[li])):
                        _lib.call("nova_kv_quant_int8", src.data_ptr(), src.stride(1), dst[:, :, c0:].data_ptr(),
                                  self.max_len * d, mn[:, :, g0:].data_ptr(), st[:, :, g0:].data_ptr(),
                                  mn.shape[2] * d, B * self.hkv, full, d, GROUP_T, stream)
                if c1 > take0:   # positions of the prompt's last <= 64 tokens into the ring
                    cache.write_ring(li, k, v, c1)
        first = self._first_token(h[:, -1])
        self._set_scalars(T)
        return first

    @torch.inference_mode()
    def prefill(self, input_ids: torch.Tensor, offset: int | None = None, reset: bool = True,
                chunk: int | None = None) -> torch.Tensor:
        """Eager prefill of ``input_ids`` ``[batch, T]`` at positions
        [offset, offset + T); returns the first greedy token ``[batch]`` (also
        left in ``input_ids``, src/nova/decode.py:224-297).

        ``reset=True`` (default) starts from an empty cache at offset 0.
        ``reset=False`` continues after the positions written so far (a
        previous prefill or ``inject``; ``offset`` defaults to ``pos``): the
        new tokens attend to the staged fp16 K/V of those positions, as the
        reference's staged prefill does, and the int8 cache is re-quantized
        over all of them.  The staged fp16 K/V is kept until ``capture()``
        (or ``release_staging()``).

        ``chunk`` (a multiple of 64, with ``reset=True``): prefill straight into
        the int8 cache chunk by chunk, later chunks attending to the int8 prefix
        (see ``_prefill_chunked``); a prompt no longer than ``chunk`` takes the
        path above unchanged."""
        cfg, cache = self.cfg, self.cache
        B, T = input_ids.shape
        if chunk is not None and T > int(chunk):
            chunk = int(chunk)
            if chunk < GROUP_T or chunk % GROUP_T or not reset or offset:
                raise ValueError("chunked prefill needs a chunk that is a multiple of 64, from position 0")
            if B != self.batch or T >= self.max_len:
                raise ValueError(f"prompt shape {tuple(input_ids.shape)} does not fit batch={self.batch}, "
                                 f"max_len={self.max_len}")
            cache.reset()
            self._staged = None
            return self._prefill_chunked(input_ids, chunk)
        if reset:
            cache.reset()
            self._staged = None
            offset = 0 if offset is None else int(offset)
        elif offset is None:
            offset = int(cache.pos.item())
        offset = int(offset)
        if B != self.batch or T < 1 or offset + T >= self.max_len:
            raise ValueError(f"prompt shape {tuple(input_ids.shape)} at offset {offset} does not fit "
                             f"batch={self.batch}, max_len={self.max_len}")
        have = 0 if self._staged is None else self._staged[0][0].shape[2]
        if offset != have:
            raise ValueError(f"offset {offset} must equal the {have} positions written since the last reset")
        total = offset + T
        ids = input_ids.to(self.device)
        h = torch.index_select(self.w.embed, 0, ids.reshape(-1)).view(B, T, -1)   # [B, T, H]
        staged = []
        for li, lw in enumerate(self.w.layers):
            q, _, k, v = self._layer_qkv(li, lw, h, offset)
            if offset:   # the staged fp16 K/V of the positions written before
                k = torch.cat([self._staged[li][0], k], dim=2)
                v = torch.cat([self._staged[li][1], v], dim=2)
            o = self._attend_prefill(li, q, k, v, prefix=offset)
            self._layer_rest(lw, h, o)
            self._commit_kv(li, k, v, total)
            staged.append((k, v))
        self._staged = staged
        first = self._first_token(h[:, -1])
        self._set_scalars(total)
        return first

    @torch.inference_mode()
    def capture_kv(self, input_ids: torch.Tensor, span: tuple[int, int]) -> tuple[torch.Tensor, torch.Tensor]:
        """K (after k_norm, before RoPE) and V of positions [span[0], span[1])
        on every layer, from a forward over ``input_ids`` ``[1, T]`` that does
        not touch the cache (capture_kv, src/nova/memory.py:176-217):
        ``[layers, kv_heads, m, head_dim]`` fp16 each."""
        B, T = input_ids.shape
        s0, s1 = int(span[0]), int(span[1])
        if B != 1 or not 0 <= s0 < s1 <= T:
            raise ValueError(f"capture needs batch 1 and 0 <= {s0} < {s1} <= {T}")
        h = torch.index_select(self.w.embed, 0, input_ids.to(self.device).reshape(-1)).view(B, T, -1)
        ks, vs = [], []
        for li, lw in enumerate(self.w.layers):
            q, k_pre, k, v = self._layer_qkv(li, lw, h, 0, want_pre=True)
            ks.append(k_pre[0, :, s0:s1].clone())
            vs.append(v[0, :, s0:s1].clone())
            self._layer_rest(lw, h, self._attend_prefill(li, q, k, v, prefix=0))
        return torch.stack(ks), torch.stack(vs)

    @torch.inference_mode()
    def inject(self, k: torch.Tensor, v: torch.Tensor, offset: int = 0) -> int:
        """Write captured K/V (``[layers, kv_heads, m, head_dim]``, K before
        RoPE) into positions [offset, offset + m), K rotated to those
        positions (MemoryStore.inject, src/nova/memory.py:447-475, which writes
        the reference's fp16 cache only -- its int8 cache is documented as
        incompatible, src/nova/kvattn.py:544-546); returns offset + m.  The
        int8 cache holds the quantized groups and the ring exactly as after a
        prefill of the same positions; the fp16 values stay staged for a
        following ``prefill(..., reset=False)``.  ``offset`` 0 resets the
        cache; otherwise it must equal the positions written so far.  Batch 1."""
        L, hkv, m, d = k.shape
        if self.batch != 1 or L != self.cfg.num_hidden_layers or hkv != self.hkv or d != self.cfg.head_dim:
            raise ValueError(f"K/V shape {tuple(k.shape)} does not match the model (batch must be 1)")
        if v.shape != k.shape:
            raise ValueError("K and V shapes differ")
        offset = int(offset)
        if offset == 0:
            self.cache.reset()
            self._staged = None
        have = 0 if self._staged is None else self._staged[0][0].shape[2]
        if offset != have or offset + m >= self.max_len:
            raise ValueError(f"offset {offset}: {have} positions written, capacity {self.max_len}")
        total = offset + m
        cos, sin = self.cos[offset:total][None], self.sin[offset:total][None]
        staged = []
        for li in range(L):
            kk = k[li].to(self.device, torch.float16)
            kr = (kk * cos + _rotate_half(kk) * sin)[None].contiguous()
            vv = v[li].to(self.device, torch.float16)[None].contiguous()
            if offset:
                kr = torch.cat([self._staged[li][0], kr], dim=2)
                vv = torch.cat([self._staged[li][1], vv], dim=2)
            self._commit_kv(li, kr, vv, total)
            staged.append((kr, vv))
        self._staged = staged
        self._set_scalars(total)
        return total

    def release_staging(self) -> None:
        """Drop the fp16 K/V kept for segmented prefill / injection."""
        self._staged = None

    def grow(self, new_max_len: int) -> None:
        """Move the int8 KV cache into a larger capacity bucket without a
        rebuild (src/nova/decode.py:444-500; the reference raises
        NotImplementedError for its int8 cache): the written groups, scales,
        ring and scalars are copied, the RoPE tables extended, and the decode
        graph dropped -- call ``capture()`` again.  Decoding continues
        bit-identically (the attention keeps its split size)."""
        new_max_len = int(new_max_len)
        if new_max_len <= self.max_len:
            return
        self.cache = self.cache.grow(new_max_len)
        self.max_len = new_max_len
        self.cos, self.sin = rope_tables(self.max_len + 1, self.cfg.head_dim, self.cfg.rope_theta, self.device)
        if self.heads and not self._heads_fit():   # more splits than o_proj's merge holds: the slots path
            self.heads = False
        self.graph = None

    # ---------------------------------------------------------------- decode

    def _gemv(self, x, w: NF4Weight, out, *, epilogue: int = _lib.NF4_PLAIN, norm_weight=None, residual=None,
              argmax=None, token_out=None, pos=None, embed=None, embed_out=None, add=None, resid_out=None,
              edge_out=None, edge_in=None, attn_part=None, add_heads=None) -> None:
        """The step's NF4 projection: nova_nf4_gemv up to GEMV_ROWS rows, else
        nova_nf4_gemm (after nova_rmsnorm when the projection has a norm prologue)."""
        B = x.shape[0]
        eps = self.cfg.rms_norm_eps
        if B > GEMV_ROWS:   # batched GEMM: weights read once for all rows; the norm runs first
            if norm_weight is not None:
                n_in = x.shape[1]
                _lib.call("nova_rmsnorm", x.data_ptr(), x.stride(0), None, 0, None, 0, norm_weight.data_ptr(),
                          self.xn.data_ptr(), self.xn.stride(0), B, n_in, float(eps), _lib.stream_of(self.device))
                x = self.xn[:, :n_in]
            nf4_gemm(x, w.tc_units(), self.lut, out, n=w.n, epilogue=epilogue, residual=residual, argmax=argmax,
                     token_out=token_out, pos=pos, embed=embed, embed_out=embed_out, workspace=self.gemm_ws)
            return
        for r in range(0, B, GEMV_ROWS):
            sl = slice(r, min(B, r + GEMV_ROWS))
            last = sl.stop == B
            o = out if epilogue == _lib.NF4_SLOTS else out[sl]   # the slot buffer is per launch, not per row
            nf4_gemv(x[sl], w.units, None, self.lut, o, epilogue=epilogue, norm_weight=norm_weight, eps=eps,
                     residual=None if residual is None else residual[sl],
                     argmax=None if argmax is None else argmax[sl],
                     token_out=None if token_out is None else token_out[sl], pos=pos if last else None,
                     embed=embed, embed_out=None if embed_out is None else embed_out[sl],
                     workspace=self.gemv_ws, n=w.n, add_slots=None if add is None else add[0],
                     add_k=0 if add is None else add[1], resid_out=resid_out, edge_out=edge_out,
                     edge_in=None if edge_in is None else edge_in[0], edge_k=0 if edge_in is None else edge_in[1],
                     attn_part=None if attn_part is None else attn_part[0],
                     attn_splits=0 if attn_part is None else attn_part[1],
                     attn_heads=0 if attn_part is None else attn_part[2], add_heads=add_heads)

    def _qk_args(self, li: int, lw) -> "_lib.QKArgs":
        cfg, cache = self.cfg, self.cache
        qa = _lib.QKArgs()
        qa.qkv, qa.qkv_stride = self.qkv.data_ptr(), self.qkv.stride(0)
        qa.q_norm_weight, qa.k_norm_weight, qa.eps = lw.q_norm.data_ptr(), lw.k_norm.data_ptr(), cfg.rms_norm_eps
        qa.cos, qa.sin, qa.rope_len = self.cos.data_ptr(), self.sin.data_ptr(), self.cos.shape[0]
        qa.q_out, qa.q_out_stride = self.q_rot.data_ptr(), self.q_rot.stride(0)
        qa.tail_k, qa.tail_v = cache.tail_k[li].data_ptr(), cache.tail_v[li].data_ptr()
        qa.kq, qa.vq = cache.kq[li].data_ptr(), cache.vq[li].data_ptr()
        qa.kmn, qa.kst = cache.kmn[li].data_ptr(), cache.kst[li].data_ptr()
        qa.vmn, qa.vst = cache.vmn[li].data_ptr(), cache.vst[li].data_ptr()
        qa.pos, qa.written = cache.pos.data_ptr(), cache._written.data_ptr()
        qa.qlen, qa.pg = cache._qlen.data_ptr(), cache._pg.data_ptr()
        qa.batch, qa.q_heads, qa.kv_heads = self.batch, self.hq, self.hkv
        qa.head_dim, qa.max_len, qa.group = cfg.head_dim, self.max_len, GROUP_T
        return qa

    def _step_body(self) -> None:
        cfg, cache, lut = self.cfg, self.cache, self.lut
        eps = cfg.rms_norm_eps
        B = self.batch
        stream = _lib.stream_of(self.device)
        q3 = self.q_rot.view(B, self.hq, cfg.head_dim)
        a3 = self.attn.view(B, self.hq, cfg.head_dim)
        ws = self.gemv_ws
        tp = self.tp

        def row_parallel(x, w):   # o_proj / down_proj + residual add
            if not tp.active:
                self._gemv(x, w, self.resid, epilogue=_lib.NF4_RESIDUAL, residual=self.resid)
                return
            self._gemv(x, w, self.part32, epilogue=_lib.NF4_F32)
            if self.p2p is not None:   # fused NVLink all-reduce + residual add
                self.p2p(self.part32, self.resid)
                return
            all_reduce_sum(self.part32, tp)
            _lib.call("nova_residual_add_f32", self.part32.data_ptr(), self.part32.stride(0), self.resid.data_ptr(),
                      self.resid.stride(0), B, cfg.hidden_size, stream)

        if self.deferred:
            self._step_body_deferred(q3, a3)
            return
        for li, lw in enumerate(self.w.layers):
            qk = None
            if self.attn_fused:
                self._gemv(self.resid, lw.qkv, self.qkv, norm_weight=lw.input_ln)
                qk = self._qk_args(li, lw)
            else:
                self._qkv_step(li, lw)
            launch_attention(q3, (cache.kq[li], cache.kmn[li], cache.kst[li], cache.vq[li], cache.vmn[li],
                                  cache.vst[li]), (cache.tail_k[li], cache.tail_v[li]), a3, None, cache._qlen,
                             cache._pg, cache._written, cache.first, cache.workspace, max_len=self.max_len,
                             n_splits=cache.n_splits, chunk=cache.chunk, window=cache.window, qk=qk)
            row_parallel(self.attn, lw.o)
            self._gemv(self.resid, lw.gate_up, self.act, epilogue=_lib.NF4_SILU_MUL, norm_weight=lw.post_ln)
            row_parallel(self.act, lw.down)
        self._gemv(self.resid, self.w.lm_head, self.logits, epilogue=_lib.NF4_ARGMAX, norm_weight=self.w.final_norm,
                   argmax=self.argmax_slot, token_out=self.input_ids, pos=cache.pos, embed=self.w.embed,
                   embed_out=self.resid)

    def _o_heads(self, li: int) -> None:
        """o_proj of layer li over the attention's split partials (one KV head per CTA, fp32 sums per head
        into y_heads; nova_nf4_gemv attn_part)."""
        cache, k = self.cache, self.q_dim // self.hkv
        nf4_gemv(self.attn[:, :k], self.o_heads[li], None, self.lut, self.y_heads.view(1, -1),
                 epilogue=_lib.NF4_F32, workspace=self.gemv_ws, n=self.hkv * self.cfg.hidden_size,
                 attn_part=attn_partials(cache.workspace, self.batch, self.hkv), attn_splits=cache.n_splits + 1,
                 attn_heads=self.hkv)

    def _step_body_deferred(self, q3, a3) -> None:
        """The step with o_proj / down_proj reductions deferred into the next
        GEMV's input staging: the residual lives in resid (step input, R0) and
        resid_alt (R1); q|k|v of layer l >= 1 reads R1 + down(l-1) and writes
        R0, gate|up reads R0 + o(l) and writes R1, the lm_head reads R1 +
        down(35) (and its step finalize writes the next embedding to R0)."""
        cfg, cache = self.cfg, self.cache
        r0, r1, slots = self.resid, self.resid_alt, self.slots
        for li, lw in enumerate(self.w.layers):
            if li == 0:
                self._gemv(r0, lw.qkv, self.qkv, norm_weight=lw.input_ln)
            else:
                self._gemv(r1, lw.qkv, self.qkv, norm_weight=lw.input_ln, add=(slots, self.inter), resid_out=r0)
            qa = self._qk_args(li, lw)
            launch_attention(q3, (cache.kq[li], cache.kmn[li], cache.kst[li], cache.vq[li], cache.vmn[li],
                                  cache.vst[li]), (cache.tail_k[li], cache.tail_v[li]), a3, None, cache._qlen,
                             cache._pg, cache._written, cache.first, cache.workspace, max_len=self.max_len,
                             n_splits=cache.n_splits, chunk=cache.chunk, window=cache.window, qk=qa,
                             defer_merge=self.heads)
            edges = self.edges
            if self.heads:
                self._o_heads(li)
                self._gemv(r0, lw.gate_up, self.act, epilogue=_lib.NF4_SILU_MUL, norm_weight=lw.post_ln,
                           resid_out=r1, edge_out=edges, add_heads=self.y_heads)
            else:
                self._gemv(self.attn, lw.o, slots, epilogue=_lib.NF4_SLOTS)
                self._gemv(r0, lw.gate_up, self.act, epilogue=_lib.NF4_SILU_MUL, norm_weight=lw.post_ln,
                           add=(slots, self.q_dim), resid_out=r1, edge_out=edges)
            self._gemv(self.act, lw.down, slots, epilogue=_lib.NF4_SLOTS,
                       edge_in=None if edges is None else (edges, cfg.hidden_size))
        self._gemv(r1, self.w.lm_head, self.logits, epilogue=_lib.NF4_ARGMAX, norm_weight=self.w.final_norm,
                   argmax=self.argmax_slot, token_out=self.input_ids, pos=cache.pos, embed=self.w.embed,
                   embed_out=r0, add=(slots, self.inter))

    def _qkv_step(self, li: int, lw) -> None:
        """input norm + q|k|v projection, then q/k norm + RoPE + KV append of layer li as a launch of
        its own (the decoder's default runs the latter inside the attention launch)."""
        stream = _lib.stream_of(self.device)
        qa = self._qk_args(li, lw)
        self._gemv(self.resid, lw.qkv, self.qkv, norm_weight=lw.input_ln)
        _lib.check(_lib.lib().nova_qk_norm_rope_append(_lib.ctypes.byref(qa), stream), "qk_norm_rope_append")

    def errors(self) -> dict:
        """Error words of the step's kernels (synchronizes; each is read and
        cleared): non-zero means a bounded wait inside a launch gave up and that
        launch's output -- hence the step's tokens -- is not valid."""
        import ctypes

        torch.cuda.synchronize(self.device)
        lib = _lib.lib()
        out = {}

        def word(name, fn, *args):
            v = ctypes.c_int(0)
            _lib.check(fn(*args, ctypes.byref(v)), name)
            out[name] = int(v.value)

        c = self.cache
        word("attention", lib.nova_attn_read_error, c.workspace.data_ptr(), self.batch, self.hkv)
        word("gemv", lib.nova_nf4_gemv_read_error, self.gemv_ws.data_ptr())
        if self.gemm_ws is not None:
            word("gemm", lib.nova_nf4_gemm_read_error, self.gemm_ws.data_ptr())
        if self.p2p is not None:
            out["allreduce"] = self.p2p.error()
        return out

    def check_errors(self) -> None:
        """Raise RuntimeError when any error word of the step's kernels is set."""
        bad = {k: v for k, v in self.errors().items() if v}
        if bad:
            raise RuntimeError(f"decode step kernels reported bounded-wait failures: {bad}")

    def close(self) -> None:
        """Release the graph and the peer mappings of the tensor-parallel
        all-reduce (before the process group is destroyed)."""
        self.graph = None
        if self.p2p is not None:
            torch.cuda.synchronize(self.device)
            self.p2p.close()

    def launches_per_step(self) -> int:
        """Kernels of this library per step (NCCL all-reduces not counted)."""
        if self.batch > GEMV_ROWS:
            per_layer = 8          # 2 norms + 4 GEMMs + q/k norm-RoPE-append + attention
        else:
            per_layer = 6
        if self.attn_fused:
            per_layer -= 1       # the q/k norm-RoPE-append runs inside the attention launch
        if self.tp.active:
            per_layer += 2       # fused all-reduce + residual add (or the residual add after NCCL), twice
        return per_layer * self.cfg.num_hidden_layers + (2 if self.batch > GEMV_ROWS else 1)

    @torch.inference_mode()
    def fill_random(self, ctx: int, seed: int = 0) -> None:
        """Decode state after a ``ctx``-token context without running the
        prefill: uniform random int8 codes and small random min/step scales in
        every layer's cache, a random fp16 ring, random current tokens.  For
        throughput measurement at batch sizes / contexts where an eager prefill
        would take minutes (the kernels' cost does not depend on the values)."""
        c = self.cache
        if ctx < 1 or ctx >= self.max_len:
            raise ValueError(f"ctx {ctx} outside [1, {self.max_len})")
        g = torch.Generator(device=self.device).manual_seed(seed)
        for li in range(self.cfg.num_hidden_layers):
            for t in (c.kq[li], c.vq[li]):
                t.random_(0, 256, generator=g)
            for t in (c.kst[li], c.vst[li]):
                t.uniform_(0.0, 0.02, generator=g)
            for t in (c.kmn[li], c.vmn[li]):
                t.uniform_(-2.5, -1.5, generator=g)
            for t in (c.tail_k[li], c.tail_v[li]):
                t.normal_(0.0, 1.0, generator=g)
        c.set_lengths(ctx)
        self.input_ids.copy_(torch.randint(0, self.cfg.vocab_size, (self.batch,), generator=g, device=self.device))
        self.resid.copy_(self.w.embed[self.input_ids])
        self.argmax_slot.zero_()

    @torch.inference_mode()
    def step_eager(self) -> torch.Tensor:
        """One decode step without a graph (same kernels); returns input_ids."""
        self._step_body()
        return self.input_ids

    @torch.inference_mode()
    def capture(self) -> None:
        """Capture one decode step.  Capture does not execute anything, so the
        decode state is untouched.  With ``pdl`` the kernels are captured with
        programmatic dependencies: each one's weight prefetch and LUT build
        overlap the previous kernel."""
        self.graph = None
        self._staged = None   # a segmented prefill ends with the first captured step
        if self.tp.active:   # the communicator must exist before its first captured collective
            all_reduce_sum(torch.zeros_like(self.part32), self.tp)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        prev = _lib.pdl_enabled()
        _lib.set_pdl(self.pdl)
        try:
            with torch.cuda.graph(g):
                self._step_body()
        finally:
            _lib.set_pdl(prev)
        self.graph = g

    def step(self) -> torch.Tensor:
        """One greedy token per row: a single graph replay."""
        if self.graph is None:
            raise RuntimeError("call capture() first")
        self.graph.replay()
        return self.input_ids

    def step_sample(self, temperature: float, top_k: int = 20, top_p: float = 1.0, repetition_penalty: float = 1.0,
                    seen: torch.Tensor | None = None, gen: torch.Generator | None = None) -> torch.Tensor:
        """One graph replay, then the next token drawn outside the graph from
        the step's logits (the chat CLI's pattern, src/chat.py:205-214): the
        sampled token replaces the graph's argmax in ``input_ids`` and its
        embedding row becomes the next step's input; ``seen`` (bool/uint8
        ``[batch, vocab]`` or ``[vocab]``) is read for the repetition penalty
        and gets the new token marked.  Temperature <= 0 keeps the argmax."""
        from .sampling import sample_topk

        if self.graph is None:
            raise RuntimeError("call capture() first")
        self.graph.replay()
        u = None
        if temperature > 0:
            u = torch.rand(self.batch, generator=gen, device=self.device if gen is None else gen.device)
            u = u.to(self.device, torch.float32)
        sample_topk(self.logits, temperature=temperature, top_k=top_k, top_p=top_p,
                    repetition_penalty=repetition_penalty, seen=seen, uniform=u, token_out=self.input_ids,
                    embed=self.w.embed, embed_out=self.resid, seen_mark=seen)
        return self.input_ids

    def step_host(self, tokens_in: torch.Tensor, tokens_out: torch.Tensor) -> torch.Tensor:
        """Streaming API with host buffers (pinned for async copies): the step's
        input tokens are copied in, their embedding rows gathered, the decode
        graph replayed and the greedy tokens copied back; returns
        ``tokens_out`` once the stream has finished the step."""
        if self.graph is None:
            raise RuntimeError("call capture() first")
        self.input_ids.copy_(tokens_in, non_blocking=True)
        torch.index_select(self.w.embed, 0, self.input_ids, out=self.resid)
        self.graph.replay()
        tokens_out.copy_(self.input_ids, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return tokens_out

    def state(self) -> dict:
        """Host copy of the decode state (cache + scalars), e.g. to seed the
        CPU oracle."""
        c = self.cache
        arr = lambda t: t.cpu().numpy()  # noqa: E731
        return {
            "pos": int(c.pos.item()), "written": int(c._written.item()), "qlen": int(c._qlen.item()),
            "input_ids": arr(self.input_ids), "resid": arr(self.resid),
            "kq": [arr(t) for t in c.kq], "vq": [arr(t) for t in c.vq], "kmn": [arr(t) for t in c.kmn],
            "kst": [arr(t) for t in c.kst], "vmn": [arr(t) for t in c.vmn], "vst": [arr(t) for t in c.vst],
            "tail_k": [arr(t) for t in c.tail_k], "tail_v": [arr(t) for t in c.tail_v],
        }


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    x1 = x[..., : x.shape[-1] // 2]
    x2 = x[..., x.shape[-1] // 2:]
    return torch.cat((-x2, x1), dim=-1)


def weights_to_numpy(w: DecoderWeights) -> dict:
    """Host copies of the NF4 weights (for the CPU oracle in tests)."""
    out = {"embed": w.embed.cpu().numpy(), "lm_head": (w.lm_head.packed.cpu().numpy(), w.lm_head.absmax.cpu().numpy()),
           "final_norm": w.final_norm.cpu().numpy(), "code": (w.code if w.code is not None else nf4_codebook()).numpy(),
           "layers": []}
    for lw in w.layers:
        gp, ga, up, ua = deinterleave_gate_up(lw.gate_up.packed, lw.gate_up.absmax)
        out["layers"].append({
            "qkv": (lw.qkv.packed.cpu().numpy(), lw.qkv.absmax.cpu().numpy()),
            "o": (lw.o.packed.cpu().numpy(), lw.o.absmax.cpu().numpy()),
            "gate": (gp.cpu().numpy(), ga.cpu().numpy()), "up": (up.cpu().numpy(), ua.cpu().numpy()),
            "down": (lw.down.packed.cpu().numpy(), lw.down.absmax.cpu().numpy()),
            "input_ln": lw.input_ln.cpu().numpy(), "post_ln": lw.post_ln.cpu().numpy(),
            "q_norm": lw.q_norm.cpu().numpy(), "k_norm": lw.k_norm.cpu().numpy()})
    return out


__all__ = ["DecoderConfig", "DecoderWeights", "NovaDecoder", "interleave_gate_up", "deinterleave_gate_up",
           "rope_tables", "weights_to_numpy"]
