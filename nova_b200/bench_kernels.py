"""Per-kernel microbenchmarks of the decode hot path (device time via CUDA
events around CUDA-graph replays; each launch in the graph reads its own
weight / KV set so that the working set exceeds the 126 MB L2).

    python -m nova_b200.bench_kernels gemv --n 19456 --k 2560 --epilogue silu --norm
    python -m nova_b200.bench_kernels attn --ctx 32768 --batch 1
    python -m nova_b200.bench_kernels gemm --n 151936 --k 2560 --m 64   # batched tcgen05 GEMM
    python -m nova_b200.bench_kernels prefill --n 512 --prefix 8192      # prefill attention
    python -m nova_b200.bench_kernels prefill_e2e --prompt 8192          # decoder prefill
    python -m nova_b200.bench_kernels all          # the config-2 shapes + config-3 sweep

Prints one JSON line per case with the launch time and achieved GB/s
(algorithmic bytes: NF4 codes + fp16 absmax for the GEMV; 272 B per cached
token and KV head + the fp16 ring + q/out for the attention).
"""

from __future__ import annotations

import argparse
import json

import torch

from . import _lib
from .decoder import interleave_gate_up
from .kernels import (build_nf4_lut, edge_buffer, gemm_workspace, gemv_workspace, heads_major, nf4_gemm, nf4_gemv,
                      pack_native, pack_tc)
from .kvattn import GROUP_T, launch_attention, new_workspace, pick_chunk
from .quant import nf4_codebook, quantize_nf4

EPI = {"plain": _lib.NF4_PLAIN, "residual": _lib.NF4_RESIDUAL, "silu": _lib.NF4_SILU_MUL, "argmax": _lib.NF4_ARGMAX,
       "f32": _lib.NF4_F32}


def _graph_time(fn, sets: int, iters: int) -> float:
    """Microseconds per launch of ``fn(i)`` for i over ``sets``, from graph replays."""
    for i in range(sets):
        fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for i in range(sets):
                fn(i)
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / (iters * sets)


def bench_gemv(n: int, k: int, m: int = 1, epilogue: str = "plain", norm: bool = False, sets: int = 0,
               iters: int = 20, seed: int = 0, layout: str = "native", edges: bool = False,
               heads: int = 0, splits: int = 34) -> dict:
    dev = torch.device("cuda")
    code = nf4_codebook()
    lut = build_nf4_lut(code).to(dev)
    nbytes = n * k // 2 + (k // 64) * n * 2
    sets = sets or max(2, min(64, (512 << 20) // nbytes + 1))
    g = torch.Generator(device=dev).manual_seed(seed)
    weights = []
    for _ in range(sets):
        w = (torch.randn(n, k, generator=g, device=dev) * 0.02).half()
        if epilogue == "silu":
            gp, ga = quantize_nf4(w[: n // 2].contiguous(), code)
            up, ua = quantize_nf4(w[n // 2:].contiguous(), code)
            pa = interleave_gate_up(gp, ga, up, ua)
        else:
            pa = quantize_nf4(w, code)
        if heads:   # o_proj over the attention's split partials: the head-major unit stream
            weights.append((heads_major(pack_native(*pa), n, k, heads), None))
        else:
            weights.append((pack_native(*pa), None) if layout == "native" else pa)
        del w
    x = torch.randn(m, k // max(1, heads), generator=g, device=dev).half()
    nw = torch.ones(k, dtype=torch.float16, device=dev) if norm else None
    nout = n // 2 if epilogue == "silu" else n
    out = torch.zeros(m, nout, dtype=torch.float16, device=dev)
    ws = gemv_workspace(dev, max(n, n * heads)).clone()
    kw = {}
    if epilogue == "residual":
        kw["residual"] = out
    if epilogue == "argmax":
        kw["argmax"] = torch.zeros(m, dtype=torch.int64, device=dev)
    if edges:   # SiLU·mul leaving its CTA-edge row groups as fp32 sums (the batch-1 decode's gate|up)
        kw["edge_out"] = edge_buffer(dev)
    if heads:   # partials of a decode attention with `splits` splits (random m, l, acc), fp32 sums per head
        gq = (k // heads) // 128
        part = torch.randn(heads * splits * gq * 132, generator=g, device=dev).abs() + 0.5
        kw.update(attn_part=part.data_ptr(), attn_splits=splits, attn_heads=heads, n=n * heads)
        out = torch.zeros(m, n * heads, dtype=torch.float32, device=dev)
        kw["_part"] = part

    part_keep = kw.pop("_part", None)   # keeps the partials alive
    kw.setdefault("n", n)

    def fn(i):
        p, a = weights[i]
        nf4_gemv(x, p, a, lut, out, epilogue=EPI[epilogue], norm_weight=nw, workspace=ws, **kw)

    us = _graph_time(fn, sets, iters)
    return {"kernel": "nf4_gemv", "layout": layout, "n": n, "k": k, "m": m, "epilogue": epilogue, "norm": norm,
            "edges": edges, "heads": heads, "sets": sets, "us": round(us, 3), "bytes": nbytes, "gbs": round(nbytes / (us * 1e-6) / 1e9, 1)}


def bench_gemm(n: int, k: int, m: int = 64, epilogue: str = "plain", sets: int = 0, iters: int = 20,
               seed: int = 0) -> dict:
    """nova_nf4_gemm (tcgen05, layout 2) on M batch rows; algorithmic bytes =
    the NF4 weight stream (x and the output are L2-resident)."""
    dev = torch.device("cuda")
    code = nf4_codebook()
    lut = build_nf4_lut(code).to(dev)
    nbytes = n * k // 2 + (k // 64) * n * 2
    sets = sets or max(2, min(64, (512 << 20) // nbytes + 1))
    g = torch.Generator(device=dev).manual_seed(seed)
    weights = []
    for _ in range(sets):
        w = (torch.randn(n, k, generator=g, device=dev) * 0.02).half()
        if epilogue == "silu":
            gp, ga = quantize_nf4(w[: n // 2].contiguous(), code)
            up, ua = quantize_nf4(w[n // 2:].contiguous(), code)
            weights.append(pack_tc(*interleave_gate_up(gp, ga, up, ua)))
        else:
            weights.append(pack_tc(*quantize_nf4(w, code)))
        del w
    x = torch.randn(m, k, generator=g, device=dev).half()
    nout = n // 2 if epilogue == "silu" else n
    out = torch.zeros(m, nout, dtype=torch.float16, device=dev)
    ws = gemm_workspace(dev, n, k)
    kw = {}
    if epilogue == "residual":
        kw["residual"] = out
    if epilogue == "argmax":
        kw["argmax"] = torch.zeros(m, dtype=torch.int64, device=dev)

    def fn(i):
        nf4_gemm(x, weights[i], lut, out, n=n, epilogue=EPI[epilogue], workspace=ws, **kw)

    us = _graph_time(fn, sets, iters)
    flops = 2.0 * m * n * k
    return {"kernel": "nf4_gemm_tc", "n": n, "k": k, "m": m, "epilogue": epilogue, "sets": sets, "us": round(us, 3),
            "bytes": nbytes, "gbs": round(nbytes / (us * 1e-6) / 1e9, 1), "tflops": round(flops / (us * 1e-6) / 1e12, 1)}


def bench_attn(ctx: int, batch: int = 1, q_heads: int = 32, kv_heads: int = 8, window: int = 0, chunk: int = 0,
               sets: int = 0, iters: int = 20, seed: int = 0) -> dict:
    dev = torch.device("cuda")
    d = 128
    max_len = ctx + GROUP_T
    qlen = ctx // GROUP_T * GROUP_T
    written = ctx
    per_set = batch * kv_heads * max_len * 2 * d
    sets = sets or max(2, min(32, (768 << 20) // per_set + 1))
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    span = min(max_len, window + GROUP_T) if window else max_len   # tokens the splits must cover
    if not chunk:
        chunk = pick_chunk(span, batch, kv_heads, q_heads, sms)
    n_splits = -(-span // chunk)
    g = torch.Generator(device=dev).manual_seed(seed)
    ng = -(-max_len // GROUP_T)
    caches = []
    for _ in range(sets):
        kq = torch.randint(0, 256, (batch, kv_heads, max_len, d), generator=g, device=dev, dtype=torch.uint8)
        vq = torch.randint(0, 256, (batch, kv_heads, max_len, d), generator=g, device=dev, dtype=torch.uint8)
        sc = [(torch.rand(batch, kv_heads, ng, d, generator=g, device=dev) * 0.01).half() for _ in range(4)]
        tail = [(torch.randn(batch, kv_heads, GROUP_T, d, generator=g, device=dev)).half() for _ in range(2)]
        caches.append((kq, sc[0], sc[1], vq, sc[2], sc[3], tail))
    q = torch.randn(batch, q_heads, d, generator=g, device=dev).half()
    out = torch.zeros(batch, q_heads, d, dtype=torch.float16, device=dev)
    qlen_t = torch.tensor([qlen], device=dev)
    pg_t = torch.tensor([qlen // GROUP_T], device=dev)
    written_t = torch.tensor([written], device=dev)
    ws = new_workspace(batch, q_heads, kv_heads, n_splits, True, dev)

    def fn(i):
        kq, kmn, kst, vq, vmn, vst, tail = caches[i]
        launch_attention(q, (kq, kmn, kst, vq, vmn, vst), tuple(tail), out, None, qlen_t, pg_t, written_t, None, ws,
                         max_len=max_len, n_splits=n_splits, chunk=chunk, window=window)

    us = _graph_time(fn, sets, iters)
    valid = min(qlen, window) if window else qlen
    ring = min(written - qlen, window) if window else written - qlen
    nbytes = batch * kv_heads * (valid * 272 + ring * 2 * d * 2) + 2 * batch * q_heads * d * 2
    return {"kernel": "attn_decode_int8", "ctx": ctx, "batch": batch, "window": window, "chunk": chunk,
            "n_splits": n_splits, "sets": sets, "us": round(us, 3), "bytes": nbytes,
            "gbs": round(nbytes / (us * 1e-6) / 1e9, 1)}


def bench_append_attn(ctx: int = 4096, batch: int = 1, q_heads: int = 32, kv_heads: int = 8, sets: int = 0,
                      iters: int = 20, seed: int = 0) -> dict:
    """the decode append of the token at position ctx-1
    (nova_kv_append_int8: ring slot write; the token completes a 64-token
    group, so the group is requantized into the int8 cache) followed by the
    decode attention of that token over all ctx positions
    (nova_attn_decode_int8), one pair of launches per layer, rotating over
    ``sets`` layers (more than L2 holds).  Algorithmic bytes: the int8 cache
    read by the attention (272 B per token and KV head), the fp16 ring read by
    the requantization, the group's codes and scales written, the new K/V, q
    and the output."""
    dev = torch.device("cuda")
    d = 128
    if ctx % GROUP_T:
        raise ValueError("ctx must be a multiple of 64")
    per_set = batch * kv_heads * ctx * 272
    sets = sets or max(2, min(64, (320 << 20) // per_set + 1))
    chunk = pick_chunk(ctx, batch, kv_heads, q_heads, torch.cuda.get_device_properties(dev).multi_processor_count)
    n_splits = -(-ctx // chunk)
    g = torch.Generator(device=dev).manual_seed(seed)
    ng = ctx // GROUP_T
    layers = []
    for _ in range(sets):
        kq = torch.randint(0, 256, (batch, kv_heads, ctx, d), generator=g, device=dev, dtype=torch.uint8)
        vq = torch.randint(0, 256, (batch, kv_heads, ctx, d), generator=g, device=dev, dtype=torch.uint8)
        sc = [(torch.rand(batch, kv_heads, ng, d, generator=g, device=dev) * 0.01).half() for _ in range(4)]
        tail = [torch.randn(batch, kv_heads, GROUP_T, d, generator=g, device=dev).half() for _ in range(2)]
        new = [torch.randn(batch, kv_heads, d, generator=g, device=dev).half() for _ in range(2)]
        layers.append((kq, sc[0], sc[1], vq, sc[2], sc[3], tail, new))
    q = torch.randn(batch, q_heads, d, generator=g, device=dev).half()
    out = torch.zeros(batch, q_heads, d, dtype=torch.float16, device=dev)
    pos = torch.tensor([ctx - 1], device=dev)
    written, qlen, pg = (torch.zeros(1, dtype=torch.int64, device=dev) for _ in range(3))
    ws = new_workspace(batch, q_heads, kv_heads, n_splits, True, dev)
    stream = _lib.stream_of(dev)

    def fn(i):
        kq, kmn, kst, vq, vmn, vst, tail, (kn, vn) = layers[i]
        _lib.call("nova_kv_append_int8", kn.data_ptr(), vn.data_ptr(), kn.stride(0), kn.stride(1),
                  tail[0].data_ptr(), tail[1].data_ptr(), kq.data_ptr(), vq.data_ptr(), kmn.data_ptr(), kst.data_ptr(),
                  vmn.data_ptr(), vst.data_ptr(), pos.data_ptr(), written.data_ptr(), qlen.data_ptr(), pg.data_ptr(),
                  batch, kv_heads, ctx, d, GROUP_T, stream)
        launch_attention(q, (kq, kmn, kst, vq, vmn, vst), tuple(tail), out, None, qlen, pg, written, None, ws,
                         max_len=ctx, n_splits=n_splits, chunk=chunk)

    us = _graph_time(fn, sets, iters)
    bh = batch * kv_heads
    nbytes = (bh * (ctx * 272 + 2 * GROUP_T * d * 2 + 2 * GROUP_T * d + 4 * d * 2 + 2 * d * 2)
              + 2 * batch * q_heads * d * 2)
    return {"kernel": "kv_append_int8 + attn_decode_int8", "ctx": ctx, "batch": batch, "sets": sets,
            "us": round(us, 3), "bytes": nbytes, "gbs": round(nbytes / (us * 1e-6) / 1e9, 1)}


def bench_prefill_attn(n: int, prefix: int, batch: int = 1, q_heads: int = 32, kv_heads: int = 8,
                       iters: int = 10, seed: int = 0) -> dict:
    """nova_attn_prefill_int8: a chunk of ``n`` queries at positions [prefix,
    prefix + n) attending causally to an int8 prefix of ``prefix`` tokens
    (read in place) and to the chunk's own fp16 keys.  Algorithmic work: 4 *
    q_heads * 128 FLOPs per (query, key) pair attended (QK and PV); bytes =
    the int8 prefix (272 B per token and KV head) + the chunk's fp16 q/k/v/out."""
    from .kvattn import prefill_attention

    dev = torch.device("cuda")
    d = 128
    g = torch.Generator(device=dev).manual_seed(seed)
    max_len = prefix + n + GROUP_T
    ng = -(-max_len // GROUP_T)
    kq = torch.randint(0, 256, (batch, kv_heads, max_len, d), generator=g, device=dev, dtype=torch.uint8)
    vq = torch.randint(0, 256, (batch, kv_heads, max_len, d), generator=g, device=dev, dtype=torch.uint8)
    sc = [(torch.rand(batch, kv_heads, ng, d, generator=g, device=dev) * 0.01).half() for _ in range(4)]
    q = torch.randn(batch, q_heads, n, d, generator=g, device=dev).half()
    k = torch.randn(batch, kv_heads, n, d, generator=g, device=dev).half()
    v = torch.randn(batch, kv_heads, n, d, generator=g, device=dev).half()
    out = torch.empty(batch, n, q_heads * d, dtype=torch.float16, device=dev)
    int8 = (kq, sc[0], sc[1], vq, sc[2], sc[3])

    def fn(i):
        prefill_attention(q, k, v, prefix=prefix, int8=int8 if prefix else None, int8_len=prefix, out=out)

    us = _graph_time(fn, 1, iters)
    pairs = n * prefix + n * (n + 1) // 2
    flops = 4.0 * batch * q_heads * d * pairs
    nbytes = batch * kv_heads * prefix * 272 + 2 * batch * (q_heads + 2 * kv_heads) * n * d * 2
    return {"kernel": "attn_prefill_int8", "n": n, "prefix": prefix, "batch": batch, "us": round(us, 3),
            "tflops": round(flops / (us * 1e-6) / 1e12, 2), "bytes": nbytes,
            "gbs": round(nbytes / (us * 1e-6) / 1e9, 1)}


def bench_prefill_e2e(prompt: int, chunk: int = 512, seed: int = 0) -> dict:
    """NovaDecoder.prefill of a ``prompt``-token prompt in ``chunk``-token
    chunks (36-layer config, random weights): prompt tokens per second,
    wall time around the call with a device synchronize."""
    import time

    from .decoder import DecoderConfig, DecoderWeights, NovaDecoder

    cfg = DecoderConfig()
    W = DecoderWeights.random_init(cfg, seed=seed)
    dec = NovaDecoder(W, max_len=prompt + 64, batch=1)
    ids = torch.randint(0, cfg.vocab_size, (1, prompt), generator=torch.Generator().manual_seed(seed))
    dec.prefill(ids, chunk=chunk)   # warm-up (and GEMM unit packing)
    torch.cuda.synchronize()
    times = []
    for _ in range(3):
        t0 = time.perf_counter()
        dec.prefill(ids, chunk=chunk)
        torch.cuda.synchronize()
        times.append(time.perf_counter() - t0)
    t = sorted(times)[1]
    return {"kernel": "prefill_e2e", "prompt": prompt, "chunk": chunk, "s": round(t, 4),
            "tok_s": round(prompt / t, 1)}


CONFIG2 = [("q_proj", 4096, 2560), ("k_proj", 1024, 2560), ("v_proj", 1024, 2560), ("o_proj", 2560, 4096),
           ("gate_proj", 9728, 2560), ("up_proj", 9728, 2560), ("down_proj", 2560, 9728),
           ("lm_head", 151936, 2560)]


def main() -> None:
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    a = sub.add_parser("gemv")
    a.add_argument("--n", type=int, required=True)
    a.add_argument("--k", type=int, required=True)
    a.add_argument("--m", type=int, default=1)
    a.add_argument("--epilogue", choices=list(EPI), default="plain")
    a.add_argument("--norm", action="store_true")
    a.add_argument("--sets", type=int, default=0)
    a.add_argument("--iters", type=int, default=20)
    a.add_argument("--layout", choices=["native", "ref"], default="native")
    a.add_argument("--pdl", action="store_true", help="launch with programmatic dependent launch")
    a.add_argument("--variant", choices=["cta", "warp"], default="cta",
                   help="native GEMV split-K at CTA level (default) or warp level")
    a.add_argument("--edges", action="store_true", help="SiLU·mul at M = 1 with CTA edges (edge_out)")
    a.add_argument("--heads", type=int, default=0,
                   help="o_proj over a decode attention's split partials: KV heads (N = output rows, K = all heads)")
    c = sub.add_parser("gemm")
    c.add_argument("--n", type=int, required=True)
    c.add_argument("--k", type=int, required=True)
    c.add_argument("--m", type=int, default=64)
    c.add_argument("--epilogue", choices=list(EPI), default="plain")
    c.add_argument("--sets", type=int, default=0)
    c.add_argument("--iters", type=int, default=20)
    b = sub.add_parser("attn")
    b.add_argument("--ctx", type=int, required=True)
    b.add_argument("--batch", type=int, default=1)
    b.add_argument("--window", type=int, default=0)
    b.add_argument("--chunk", type=int, default=0)
    b.add_argument("--sets", type=int, default=0)
    b.add_argument("--iters", type=int, default=20)
    f = sub.add_parser("prefill")
    f.add_argument("--n", type=int, default=512, help="queries in the chunk")
    f.add_argument("--prefix", type=int, default=8192, help="int8 prefix tokens")
    f.add_argument("--iters", type=int, default=10)
    e = sub.add_parser("prefill_e2e")
    e.add_argument("--prompt", type=int, default=8192)
    e.add_argument("--chunk", type=int, default=512)
    sub.add_parser("all")
    args = ap.parse_args()
    _lib.lib()
    if args.cmd == "gemv":
        _lib.set_launch_flags((_lib.LAUNCH_PDL if args.pdl else 0) |
                              (_lib.LAUNCH_WARP_SPLITK if args.variant == "warp" else 0))
        print(json.dumps(bench_gemv(args.n, args.k, args.m, args.epilogue, args.norm, args.sets, args.iters,
                                    layout=args.layout, edges=args.edges, heads=args.heads)))
    elif args.cmd == "gemm":
        _lib.set_launch_flags(_lib.LAUNCH_PDL)
        print(json.dumps(bench_gemm(args.n, args.k, args.m, args.epilogue, args.sets, args.iters)))
    elif args.cmd == "prefill":
        _lib.set_launch_flags(_lib.LAUNCH_PDL)
        print(json.dumps(bench_prefill_attn(args.n, args.prefix, iters=args.iters)))
    elif args.cmd == "prefill_e2e":
        print(json.dumps(bench_prefill_e2e(args.prompt, args.chunk)))
    elif args.cmd == "attn":
        print(json.dumps(bench_attn(args.ctx, args.batch, window=args.window, chunk=args.chunk, sets=args.sets,
                                    iters=args.iters)))
    else:
        for variant in ("warp", "cta"):
            _lib.set_launch_flags(_lib.LAUNCH_PDL | (_lib.LAUNCH_WARP_SPLITK if variant == "warp" else 0))
            for name, n, k in CONFIG2:
                r = bench_gemv(n, k)
                r["name"], r["variant"] = name, variant
                print(json.dumps(r), flush=True)
            for name, n, k, epi, nrm in (("qkv_fused", 6144, 2560, "plain", True),
                                         ("gate_up_fused", 19456, 2560, "silu", True)):
                r = bench_gemv(n, k, epilogue=epi, norm=nrm)
                r["name"], r["variant"] = name, variant
                print(json.dumps(r), flush=True)
        _lib.set_launch_flags(_lib.LAUNCH_PDL)
        for ctx in (4096, 8192, 32768, 65536, 131072):
            for batch in (1, 4, 16):
                if batch * ctx > 16 * 65536:
                    continue
                print(json.dumps(bench_attn(ctx, batch)), flush=True)
        print(json.dumps(bench_attn(131072, 4, window=4096)), flush=True)


if __name__ == "__main__":
    main()
