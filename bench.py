"""Benchmark: greedy decode tok/s of the full random-init Qwen3-VL-4B text
decoder (36 layers, NF4 weights incl. the 4-bit lm_head, int8 KV cache
prefilled with 8192 uniform-random tokens, batch 1) -- the configuration
BASELINE.json quotes its decode metric on -- with the per-kernel roofline of
the NF4 GEMV and the int8-KV attention measured live.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One step = one decode token for every row (one CUDA-graph replay).  The step
streams ~2.8 GB (weights + KV), far above the 126 MB L2, so no flush is needed
between steps.  N > 1 (torchrun, one process per GPU): by default the same
decode sharded over the N GPUs by tensor parallelism (KV heads / intermediate
columns, NCCL all-reduce after o_proj and down_proj inside the graph; strong
scaling: one sequence, whole-job tok/s); ``--parallel replicas`` runs N
independent copies instead (weak scaling).  The timed region is bracketed by
barriers and the max over ranks is reported.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "decode tok/s (Qwen3-VL-4B text, NF4+int8 KV); int8-KV attn HBM GB/s vs peak"
UNIT = "tok/s"


def _workload(args) -> str:
    """The BASELINE configuration a run measures."""
    which = ("BASELINE config 4" if (args.batch, args.ctx) == (1, 8192) else
             "BASELINE config 5" if (args.batch, args.ctx) == (64, 32768) else "custom")
    return (f"qwen3vl4b-text greedy decode, NF4 weights (blocksize 64, fp16 absmax) incl. 4-bit lm_head, int8 KV "
            f"(int8t64), batch {args.batch}, ctx {args.ctx} ({which})")


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--ctx", type=int, default=8192)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--layers", type=int, default=36, help="36 for the headline config")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the BASELINE config 1/2/3/5 sub-records added to the line")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--kv-fill", choices=["auto", "prefill", "random"], default="auto",
                    help="context: eager prefill of random tokens, or random int8 codes written straight into the "
                         "cache (auto: prefill up to batch*ctx = 65536 tokens)")
    ap.add_argument("--parallel", choices=["tp", "replicas"], default="tp",
                    help="N > 1: tensor parallelism over the N GPUs (default) or N independent replicas")
    return ap.parse_args()


def _peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc = None
        self.samples: list[tuple[float, str]] = []   # (host time, csv line)
        self.t_begin = self.t_end = None
        self._reader = None

    def start(self) -> None:
        """Start nvidia-smi (every 20 ms) and return once its first sample
        arrived (its start-up can take longer than a short timed region)."""
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return

        def read() -> None:
            for line in self.proc.stdout:
                if line.strip():
                    self.samples.append((time.monotonic(), line.strip()))

        self._reader = threading.Thread(target=read, daemon=True)
        self._reader.start()
        t0 = time.monotonic()
        while not self.samples and time.monotonic() - t0 < 5.0 and self.proc.poll() is None:
            time.sleep(0.005)

    def mark_begin(self) -> None:
        self.t_begin = time.monotonic()

    def mark_end(self) -> None:
        self.t_end = time.monotonic()

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        t0 = time.monotonic()   # one more sample after the timed region (the last one may straddle its end)
        while time.monotonic() - t0 < 0.5 and not any(t > (self.t_end or 0.0) for t, _ in self.samples):
            time.sleep(0.005)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self._reader is not None:
            self._reader.join(timeout=5)
        lines = self.samples
        if self.t_begin is not None and self.t_end is not None:   # the samples taken while the steps ran
            inside = [x for x in lines if self.t_begin - 0.005 <= x[0] <= self.t_end + 0.025]
            lines = inside or lines
        rows = [r.split(", ") for _, r in lines]
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows if len(r) >= 9 for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------- reference arm


def run_reference(args, rank: int) -> None:
    """The reference algorithm on the host cores: the CPU oracle port of one
    decode token (the reference's decode path is Python + Triton on CUDA; its
    CPU path is the torch eager model, which the oracle restates in numpy).
    Each step is a bounded sample of the same workload -- one full decoder
    layer at the bench context plus 1/36 of the 4-bit lm_head, every linear
    NF4-dequantized on the call -- and tok/s = 1 / (36 x the median sample),
    the same figure as the B200 arm's ``cpu_baseline``."""
    if rank != 0:
        return
    import numpy as np

    from oracle.baseline import LayerSample, host_threads

    s = LayerSample(ctx=args.ctx, seed=args.seed)
    for _ in range(max(1, args.warmup)):
        s.run()
    times = [s.run() for _ in range(args.steps)]
    sec_tok = float(np.median(times)) * s.layers   # one sequence; the host does B sequences one after another
    v = 1.0 / sec_tok
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": sec_tok * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": _workload(args), "ctx": args.ctx, "global_batch": args.batch, "layers": 36,
                   "parallelism": "host cores"},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": host_threads(), "kind": "port",
                         "sample": f"per step: one full decoder layer at ctx {args.ctx} + 1/36 of the lm_head (NF4 "
                                   "dequant per call + fp32 numpy matmul, int8 KV dequant + fp32 attention); "
                                   "tok/s = 1 / (36 x median step)"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- B200 arm


def _time_kernels(dec, reps: int = 10) -> dict:
    """Per-kernel device time of one decode step's launch families: each
    family is captured as a CUDA graph of one launch per layer (36 distinct
    weight sets / KV caches, so every launch reads HBM, not L2) and replayed
    ``reps`` times between CUDA events on the launching stream."""
    import torch

    from nova_b200 import _lib
    from nova_b200.kernels import nf4_gemv
    from nova_b200.kvattn import launch_attention

    cfg, lut, eps, ws = dec.cfg, dec.lut, dec.cfg.rms_norm_eps, dec.gemv_ws
    B = dec.batch
    out = {}
    stream = torch.cuda.current_stream()

    def bytes_of(w):
        return w.stream_bytes

    scratch = {"qkv": dec.qkv.clone(), "resid": dec.resid.clone(), "act": dec.act.clone(), "attn": dec.attn.clone()}
    layer_index = {id(lw): i for i, lw in enumerate(dec.w.layers)}
    if dec.tp.active:   # row-parallel projections write fp32 partial sums
        part = dec.part32.clone()

        def row_par(x, w, **kw):
            dec._gemv(x, w, part, epilogue=_lib.NF4_F32)
    elif dec.deferred:   # batch 1: fp32 sums per CTA, added by the next GEMV's staging
        slots, r_alt = dec.slots.clone(), scratch["resid"].clone()

        def row_par(x, w, **kw):
            dec._gemv(x, w, slots, epilogue=_lib.NF4_SLOTS, **kw)
    else:
        def row_par(x, w, **kw):
            dec._gemv(x, w, scratch["resid"], epilogue=_lib.NF4_RESIDUAL, residual=scratch["resid"])
    gate_up_add = dict(add=(slots, dec.q_dim), resid_out=r_alt) if (dec.deferred and not dec.tp.active) else {}
    down_edges = {}
    if dec.edges is not None:   # gate|up leaves its CTA-edge row groups to down_proj's staging
        edges = dec.edges.clone()
        gate_up_add["edge_out"] = edges
        down_edges = {"edge_in": (edges, dec.cfg.hidden_size)}
    o_fn = lambda lw: row_par(scratch["attn"], lw.o)
    if dec.heads:   # o_proj over the attention's split partials (those the last step left), per-head sums
        o_fn = lambda lw: dec._o_heads(layer_index[id(lw)])
        gate_up_add.pop("add", None)
        gate_up_add["add_heads"] = dec.y_heads
    fams = {
        # the step's q|k|v launch (with q/k norm + RoPE + ring write; pos does not move, so the same ring slot
        # is rewritten)
        "qkv": (lambda lw: dec._qkv_step(layer_index[id(lw)], lw), lambda lw: bytes_of(lw.qkv)),
        "o_proj": (o_fn, lambda lw: bytes_of(lw.o)),
        "gate_up": (lambda lw: dec._gemv(scratch["resid"], lw.gate_up, scratch["act"], epilogue=_lib.NF4_SILU_MUL,
                                         norm_weight=lw.post_ln, **gate_up_add),
                    lambda lw: bytes_of(lw.gate_up)),
        "down": (lambda lw: row_par(scratch["act"], lw.down, **down_edges), lambda lw: bytes_of(lw.down)),
    }
    from nova_b200.bench_kernels import _graph_time

    layers = dec.w.layers
    for name, (fn, nbytes) in fams.items():
        us = _graph_time(lambda i: fn(layers[i]), len(layers), reps)
        out[name] = {"launches": reps * len(layers), "ms": us * 1e-3, "bytes": nbytes(layers[0]),
                     "gbs": nbytes(layers[0]) / (us * 1e-6) / 1e9}
    # lm_head (a single 207 MB matrix, above L2)
    hw = dec.w.lm_head
    logits = dec.logits.clone()
    slot = torch.zeros_like(dec.argmax_slot)
    us = _graph_time(lambda i: dec._gemv(scratch["resid"], hw, logits, epilogue=_lib.NF4_ARGMAX,
                                         norm_weight=dec.w.final_norm, argmax=slot), 4, reps)
    hb = bytes_of(hw)
    out["lm_head"] = {"launches": reps * 4, "ms": us * 1e-3, "bytes": hb, "gbs": hb / (us * 1e-6) / 1e9}
    # int8-KV attention over every layer's cache at the current context
    c = dec.cache
    q3 = dec.q_rot.view(B, dec.hq, cfg.head_dim)
    a3 = scratch["attn"].view(B, dec.hq, cfg.head_dim)

    def attn(li):
        launch_attention(q3, (c.kq[li], c.kmn[li], c.kst[li], c.vq[li], c.vmn[li], c.vst[li]),
                         (c.tail_k[li], c.tail_v[li]), a3, None, c._qlen, c._pg, c._written, c.first, c.workspace,
                         max_len=dec.max_len, n_splits=c.n_splits, chunk=c.chunk, window=c.window)

    us = _graph_time(attn, cfg.num_hidden_layers, reps)
    n = reps * cfg.num_hidden_layers
    ms = us * 1e-3
    qlen, written = int(c._qlen.item()), int(c._written.item())
    hkv = dec.hkv
    # algorithmic bytes: per cached int8 token and KV head 272 B = K+V codes (2*128 B) + the fp16
    # min/step vectors amortised over 64 tokens (4*128*2/64 B); the fp16 ring slots in use; q in, out
    ab = B * hkv * (qlen * 272 + (written - qlen) * 2 * 128 * 2) + 2 * B * dec.q_dim * 2
    out["attention"] = {"launches": n, "ms": ms, "bytes": ab, "gbs": ab / (ms * 1e-3) / 1e9, "ctx": written}
    return out


def _kernel_configs(peaks: dict, cpu: bool) -> dict:
    """BASELINE configs 1-3 measured in this run on one GPU (device time per
    launch from CUDA-graph replays over weight / KV sets larger than L2), each
    next to its CPU figure (the oracle port on this host's cores)."""
    import torch

    from nova_b200.bench_kernels import CONFIG2, bench_append_attn, bench_attn, bench_gemv

    from oracle.baseline import AttnSlice, Config1Sample, GemvSample, host_threads, median_time

    hbm = peaks["hbm_gbs"]
    out = {}
    # config 1: one layer, batch 1, 32 q / 8 KV heads, ctx 4096: the append of the group-completing token + attention
    r = bench_append_attn(4096, 1)
    c1 = {"workload": "1 layer, batch 1, 32 q / 8 KV heads, ctx 4096: int8 KV append (group requantized) + decode "
                      "attention", "kernel": r["kernel"], "us": r["us"], "bytes": r["bytes"], "gbs": r["gbs"],
          "frac": round(r["gbs"] / hbm, 3)}
    if cpu:
        sec, runs = median_time(Config1Sample().run, budget_s=2.0)
        c1["cpu"] = {"us": round(sec * 1e6, 1), "gbs": round(r["bytes"] / sec / 1e9, 2), "cores": host_threads(),
                     "kind": "port", "sample": f"median of {runs}: ring requantization + int8 dequant + fp32 attention"}
    out["c1"] = c1
    torch.cuda.empty_cache()
    # config 2: the NF4 GEMV shapes at batch 1 (native unit layout, as the decoder streams them)
    shapes = []
    for name, n, k in CONFIG2:
        r = bench_gemv(n, k, iters=10)
        rec = {"name": name, "n": n, "k": k, "us": r["us"], "bytes": r["bytes"], "gbs": r["gbs"],
               "frac": round(r["gbs"] / hbm, 3)}
        if cpu:
            smp = GemvSample(n, k, rows=min(n, 9728))
            sec, runs = median_time(smp.run, budget_s=1.0)
            rec["cpu_us"] = round(sec * smp.scale * 1e6, 1)
            rec["cpu_sample"] = (f"median of {runs}" if smp.scale == 1 else
                                 f"median of {runs} over 9728 of the {n} rows, scaled x{smp.scale:.2f}")
        shapes.append(rec)
        torch.cuda.empty_cache()
    out["c2"] = {"workload": "NF4 GEMV, batch 1, weights N(0,0.02) blocksize 64 fp16 absmax", "kernel": "nf4_gemv",
                 "shapes": shapes, "cpu_cores": host_threads() if cpu else None,
                 "cpu_kind": "port: NF4 dequant + fp32 numpy matmul per call" if cpu else None}
    # config 3: long-context decode attention, full causal and window 4096
    cases = []
    slices = {}
    for batch in (1, 4, 16):
        for ctx in (32768, 65536, 131072):
            for window in (0, 4096):
                r = bench_attn(ctx, batch, window=window, iters=10)
                rec = {"ctx": ctx, "batch": batch, "window": window, "us": r["us"], "bytes": r["bytes"],
                       "gbs": r["gbs"], "frac": round(r["gbs"] / hbm, 3), "chunk": r["chunk"]}
                if cpu:
                    if (ctx, window) not in slices:
                        slices[(ctx, window)] = median_time(AttnSlice(ctx, window).run, budget_s=0.5)[0]
                    rec["cpu_us"] = round(slices[(ctx, window)] * batch * 8 * 1e6, 1)
                cases.append(rec)
                torch.cuda.empty_cache()
    out["c3"] = {"workload": "int8-KV decode attention, 32 q / 8 KV heads", "kernel": "attn_decode_int8",
                 "cases": cases,
                 "basis": "algorithmic bytes (272 B per attended int8 token and KV head + ring + q/out) / CUDA-event "
                          "device time per launch",
                 "cpu_sample": "one batch row x one KV head (4 q heads) timed, x batch x 8" if cpu else None}
    return out


def _config5(args, rank: int, world: int, dev, use_tp: bool, cpu: bool) -> dict:
    """BASELINE config 5 measured in the same run: batch 64, ctx 32768 per
    sequence (random int8 codes written straight into the cache), the batched
    NF4 GEMMs on the tcgen05 tensor cores, tensor-parallel over the job's GPUs
    when the bench runs tensor parallelism.  Every rank takes part."""
    import torch
    import torch.distributed as dist

    from nova_b200.decoder import DecoderConfig, DecoderWeights, NovaDecoder
    from nova_b200.tp import TPContext

    cfg = DecoderConfig()
    batch, ctx, warm = 64, 32768, 2
    steps = max(1, min(args.steps, 16))
    W = DecoderWeights.random_init(cfg, seed=args.seed, device=dev)
    tp = TPContext(rank, world, dist.group.WORLD) if use_tp else None
    dec = NovaDecoder(W, max_len=ctx + warm + steps + 64, batch=batch, device=dev, tp=tp)
    del W
    dec.fill_random(ctx, seed=args.seed + 5)
    dec.capture()
    for _ in range(warm):
        dec.step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        dec.step()
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ar_us = _time_allreduce(dec, reps=3)
    dec.check_errors()
    ms = float(t.item()) / steps
    copies = 1 if use_tp else world
    kv_bytes = batch * dec.hkv * ctx * 272 * cfg.num_hidden_layers    # this GPU's shard
    step_bytes = kv_bytes + dec.w.nbytes_per_token()
    peak = _peaks()["hbm_gbs"]
    rec = {"workload": "batch 64, ctx 32768, random int8 KV, NF4 GEMMs on tcgen05" +
                       (f", tp{world}" if use_tp else ""),
           "value": copies * batch / (ms * 1e-3), "unit": UNIT, "ms_per_step": ms, "steps": steps,
           "n_gpus": world, "step_roofline": {"bytes_per_step": step_bytes, "per": "GPU",
                                              "ms_at_peak": step_bytes / (peak * 1e9) * 1e3,
                                              "frac": step_bytes / (peak * 1e9) / (ms * 1e-3)},
           "gpu_launches_per_step": dec.launches_per_step()}
    if ar_us is not None:
        calls = 2 * cfg.num_hidden_layers
        rec["tp_breakdown"] = {"allreduce_us_per_call": round(ar_us, 2), "calls_per_step": calls,
                               "allreduce_share": round(calls * ar_us * 1e-3 / ms, 3)}
    dec.close()
    del dec
    torch.cuda.empty_cache()
    if cpu and rank == 0:
        from oracle.baseline import LayerSample, host_threads

        smp = LayerSample(ctx=ctx, seed=args.seed, batch=batch, attn_rows=2)
        sec = min(smp.run() for _ in range(2))
        rec["cpu"] = {"value": batch / (sec * smp.layers), "unit": UNIT, "cores": host_threads(), "kind": "port",
                      "sample": "best of 2 x one decoder layer for 64 rows at ctx 32768 (linears for all rows, "
                                "2 rows' attentions timed and scaled to 64) + 1/36 of the lm_head; x 36 layers"}
    return rec


def _time_allreduce(dec, reps: int = 10) -> float | None:
    """Device microseconds per call of the decode step's fused NVLink
    all-reduce + residual add (tensor parallelism, peer-memory path), from a
    graph of one call per layer replayed ``reps`` times on every rank at once
    (every rank makes the same calls in the same order).  None without it."""
    if dec.p2p is None:
        return None
    import torch

    from nova_b200.bench_kernels import _graph_time

    part, resid = torch.zeros_like(dec.part32), dec.resid.clone()
    return _graph_time(lambda i: dec.p2p(part, resid), dec.cfg.num_hidden_layers, reps)


def run_b200(args, rank: int, world: int, local_rank: int) -> None:
    import torch
    import torch.distributed as dist

    from nova_b200 import _lib
    from nova_b200.decoder import DecoderConfig, DecoderWeights, NovaDecoder

    from nova_b200.tp import TPContext

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    _lib.lib()
    cfg = DecoderConfig(num_hidden_layers=args.layers)
    t0 = time.time()
    W = DecoderWeights.random_init(cfg, seed=args.seed, device=dev)
    max_len = args.ctx + 2 * (args.warmup + args.steps) + 64
    use_tp = world > 1 and args.parallel == "tp"
    tp = TPContext(rank, world, dist.group.WORLD) if use_tp else None
    dec = NovaDecoder(W, max_len=max_len, batch=args.batch, device=dev, tp=tp)
    del W
    copies = 1 if use_tp else world   # independent sequences in the job
    g = torch.Generator().manual_seed(args.seed + 1 + (0 if use_tp else rank))
    fill = args.kv_fill if args.kv_fill != "auto" else ("prefill" if args.batch * args.ctx <= 65536 else "random")
    if fill == "prefill":
        prompt = torch.randint(0, cfg.vocab_size, (args.batch, args.ctx), generator=g)
        dec.prefill(prompt)
    else:
        dec.fill_random(args.ctx, seed=args.seed + 1)
    dec.capture()
    torch.cuda.synchronize()
    setup_s = time.time() - t0

    for _ in range(args.warmup):
        dec.step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(torch.cuda.current_device() if "CUDA_VISIBLE_DEVICES" not in os.environ else local_rank)
    clocks.start()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    clocks.mark_begin()
    torch.cuda.nvtx.range_push("timed_steps")   # lets ncu select the timed launches (--nvtx-include timed_steps/)
    e0.record(stream)
    for _ in range(args.steps):
        dec.step()
    e1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    clocks.mark_end()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = copies * args.batch * args.steps / (ms_max * 1e-3)

    # ---- e2e through the public API: pinned host token in, greedy token out, every step
    tok_in = torch.empty(args.batch, dtype=torch.int64, pin_memory=True)
    tok_out = torch.empty(args.batch, dtype=torch.int64, pin_memory=True)
    tok_in.copy_(dec.input_ids.cpu())
    for _ in range(2):
        dec.step_host(tok_in, tok_out)
        tok_in.copy_(tok_out)
    if world > 1:
        dist.barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    f0.record(stream)
    for _ in range(args.steps):
        dec.step_host(tok_in, tok_out)
        tok_in.copy_(tok_out)
    f1.record(stream)
    torch.cuda.synchronize()
    te = torch.tensor([f0.elapsed_time(f1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_v = copies * args.batch * args.steps / (float(te.item()) * 1e-3)

    kern = _time_kernels(dec)
    ar_us = _time_allreduce(dec)
    dec.check_errors()   # a bounded wait that gave up in any launch invalidates the numbers
    if world > 1:
        dist.barrier()
    launches = dec.launches_per_step()
    configs = {}
    if world == 1 and not args.no_configs:
        configs.update(_kernel_configs(_peaks(), cpu=not args.no_cpu_baseline))
    if not args.no_configs and (args.batch, args.ctx) == (1, 8192):
        dec.close()
        del dec
        torch.cuda.empty_cache()
        configs["c5"] = _config5(args, rank, world, dev, use_tp, cpu=world == 1 and not args.no_cpu_baseline)
    if rank != 0:
        return

    peaks = _peaks()
    # DRAM bytes per algorithmic byte from one ncu capture of each kernel (dram__bytes_read.sum +
    # dram__bytes_write.sum): the fused gate/up GEMV moved 26.54 MB for 26.46 MB of codes + absmax;
    # the attention at ctx 32768 moved 71.86 + 1.31 MB for 71.32 MB.  Applied to this run's bytes.
    gemv_traffic_ratio = 26.540288 / 26.460160
    attn_traffic_ratio = (71.857920 + 1.305600) / 71.319552
    gemv = [kern[k] for k in ("qkv", "o_proj", "gate_up", "down", "lm_head")]
    per_tok = {k: kern[k]["ms"] * (1 if k == "lm_head" else cfg.num_hidden_layers) for k in kern}
    gemv_bytes = sum(kern[k]["bytes"] * (1 if k == "lm_head" else cfg.num_hidden_layers)
                     for k in ("qkv", "o_proj", "gate_up", "down", "lm_head"))
    gemv_ms = sum(per_tok[k] for k in ("qkv", "o_proj", "gate_up", "down", "lm_head"))
    gemv_gbs = gemv_bytes / (gemv_ms * 1e-3) / 1e9
    n_launch = sum(k["launches"] for k in gemv)
    att = kern["attention"]
    roofline = {"kernel": "nf4_gemv_kernel (all decode GEMVs of a step)", "bound": "hbm", "achieved": gemv_gbs,
                "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": gemv_gbs / peaks["hbm_gbs"],
                "peak_source": peaks["source"] + " (MEASURED_PEAKS.json hbm_gbs)" if peaks["source"] == "measured"
                else "fallback 6650 GB/s",
                "traffic": gemv_bytes * gemv_traffic_ratio, "traffic_basis": "per step; ncu DRAM bytes of the fused "
                "gate/up launch scaled by algorithmic bytes", "bytes_per_step": gemv_bytes, "ms_per_step": gemv_ms, "launches_timed": n_launch,
                "per_shape_note": "each launch family replayed alone (one launch per layer in its own graph): no "
                                  "overlap with the neighbouring kernels, so these times exceed the family's share "
                                  "of the step",
                "per_shape": {k: {"gbs": round(kern[k]["gbs"], 1), "us": round(kern[k]["ms"] * 1e3, 2),
                                  "bytes": kern[k]["bytes"]} for k in ("qkv", "o_proj", "gate_up", "down", "lm_head")}}
    attn_roof = {"kernel": "attn_decode_int8_kernel", "bound": "hbm", "achieved": att["gbs"], "peak": peaks["hbm_gbs"],
                 "unit": "GB/s", "frac": att["gbs"] / peaks["hbm_gbs"], "ctx": att["ctx"],
                 "bytes_per_launch": att["bytes"], "us_per_launch": att["ms"] * 1e3,
                 "traffic": att["bytes"] * attn_traffic_ratio,
                 "traffic_basis": "per launch; ncu DRAM bytes at ctx 32768 scaled by algorithmic bytes"}
    step_bytes = gemv_bytes + att["bytes"] * cfg.num_hidden_layers
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_max / args.steps, "higher_is_better": True,
        "scaling": "strong" if use_tp else "weak", "vs_baseline": None,
        "dtype": "fp16", "data": "synthetic",
        "config": {"workload": _workload(args),
                   "kv_fill": "random int8 codes" if fill == "random" else "prefill of uniform random tokens",
                   "model": "Qwen3-VL-4B text (random init N(0,0.02))",
                   "global_batch": args.batch * copies, "ctx": args.ctx, "layers": cfg.num_hidden_layers,
                   "parallelism": f"tp{world} (KV-head / column-row split; all-reduce after o_proj and down_proj "
                                  f"as one NVLink peer-memory kernel with the residual add)" if use_tp
                                  else ("replicas" if world > 1 else "single GPU"),
                   "l2": "inputs larger than L2 (>= 2.8 GB streamed per step)", "graph": "one CUDA graph per step"},
        "roofline": roofline,
        "attn_roofline": attn_roof,
        # bytes one GPU streams per step (its shard with tensor parallelism) against one GPU's peak
        "step_roofline": {"bytes_per_token": step_bytes, "per": "GPU",
                          "tok_s_at_peak": peaks["hbm_gbs"] * 1e9 / step_bytes,
                          "frac": (value / copies / args.batch) / (peaks["hbm_gbs"] * 1e9 / step_bytes)},
        "e2e": {"value": e2e_v, "unit": UNIT, "h2d_bytes_per_step": 8 * args.batch, "d2h_bytes_per_step": 8 * args.batch},
        "gpu_launches": launches * args.steps * world,
        "clocks": clk,
        "setup_s": round(setup_s, 1),
    }
    if ar_us is not None:
        calls = 2 * cfg.num_hidden_layers
        step_ms = ms_max / args.steps
        line["tp_breakdown"] = {
            "allreduce_us_per_call": round(ar_us, 2), "calls_per_step": calls,
            "allreduce_ms_per_step": round(calls * ar_us * 1e-3, 3),
            "allreduce_share": round(calls * ar_us * 1e-3 / step_ms, 3),
            "lm_head_ms_per_step": round(kern["lm_head"]["ms"], 3),
            "lm_head_share": round(kern["lm_head"]["ms"] / step_ms, 3),
            "basis": "each family replayed alone (graph of one call per layer), device time; shares of the measured "
                     "step time"}
    line.update(configs)
    if world == 1 and not args.no_cpu_baseline:
        from oracle.baseline import LayerSample, host_threads, median_time

        smp = LayerSample(ctx=args.ctx, seed=args.seed)
        sec, runs = median_time(smp.run, budget_s=20.0, max_runs=20)
        line["cpu_baseline"] = {"value": 1.0 / (sec * smp.layers), "unit": UNIT, "cores": host_threads(),
                                "kind": "port",
                                "sample": f"{runs} x one full decoder layer at ctx {args.ctx} + 1/36 of the lm_head "
                                          "(NF4 dequant per call + fp32 numpy matmul, int8 KV dequant + fp32 "
                                          "attention); tok/s = 1 / (36 x median sample)"}
    print(json.dumps(line), flush=True)


def main() -> None:
    args = _args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    try:
        run_b200(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
