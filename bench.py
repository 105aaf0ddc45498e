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
    ap.add_argument("--no-attn-sweep", action="store_true",
                    help="skip the long-context attention sample (BASELINE config 3) added to the line")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--kv-fill", choices=["auto", "prefill", "random"], default="auto",
                    help="context: eager prefill of random tokens, or random int8 codes written straight into the "
                         "cache (auto: prefill up to batch*ctx = 65536 tokens)")
    ap.add_argument("--qkv-fused", action="store_true",
                    help="q|k|v GEMV and q/k norm + RoPE + append as one launch (one CTA per head)")
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
        self.lines: list[str] = []

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.05)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        rows = [r.split(", ") for r in out.strip().splitlines() if r.strip()]
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows if len(r) >= 9 for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------- reference arm


def run_reference(args, rank: int) -> None:
    """The reference algorithm on the host cores (the CPU oracle port; the
    reference itself is Python/Triton and its CPU path is what the oracle
    restates).  Each step is a bounded sample: one decoder layer with 1/8 of
    every linear's rows and of the KV heads, plus its lm_head share; tok/s
    scales it by 36 * 8."""
    if rank != 0:
        return
    import numpy as np

    from oracle.baseline import LayerSample, host_threads

    s = LayerSample(ctx=args.ctx, slice=8, seed=args.seed)
    for _ in range(max(1, args.warmup)):
        s.run()
    times = [s.run() for _ in range(args.steps)]
    sec_tok = float(np.mean(times)) * s.seconds_scale   # one sequence; the host does B sequences one after another
    v = 1.0 / sec_tok
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": float(np.mean(times)) * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": _workload(args), "ctx": args.ctx, "global_batch": args.batch, "layers": 36,
                   "parallelism": "host cores"},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": host_threads(), "kind": "port",
                         "sample": f"per step: 1 decoder layer at ctx {args.ctx} with 1/8 of each linear's rows and "
                                   "of the KV heads + 1/288 of the lm_head, NF4 dequant per call + fp32 numpy; "
                                   "scaled x288 (one sequence; tok/s of a batch is the same on the host)"},
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

        def row_par(x, w):
            dec._gemv(x, w, part, epilogue=_lib.NF4_F32)
    else:
        def row_par(x, w):
            dec._gemv(x, w, scratch["resid"], epilogue=_lib.NF4_RESIDUAL, residual=scratch["resid"])
    fams = {
        # the step's q|k|v launch (with q/k norm + RoPE + ring write; pos does not move, so the same ring slot
        # is rewritten)
        "qkv": (lambda lw: dec._qkv_step(layer_index[id(lw)], lw), lambda lw: bytes_of(lw.qkv)),
        "o_proj": (lambda lw: row_par(scratch["attn"], lw.o), lambda lw: bytes_of(lw.o)),
        "gate_up": (lambda lw: dec._gemv(scratch["resid"], lw.gate_up, scratch["act"], epilogue=_lib.NF4_SILU_MUL,
                                         norm_weight=lw.post_ln),
                    lambda lw: bytes_of(lw.gate_up)),
        "down": (lambda lw: row_par(scratch["act"], lw.down), lambda lw: bytes_of(lw.down)),
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
    dec = NovaDecoder(W, max_len=max_len, batch=args.batch, device=dev, tp=tp, qkv_fused=args.qkv_fused)
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
    time.sleep(0.1)
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("timed_steps")   # lets ncu select the timed launches (--nvtx-include timed_steps/)
    e0.record(stream)
    for _ in range(args.steps):
        dec.step()
    e1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
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
    if world > 1:
        dist.barrier()
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
        "gpu_launches": dec.launches_per_step() * args.steps * world,
        "clocks": clk,
        "setup_s": round(setup_s, 1),
    }
    if world == 1 and not args.no_attn_sweep:
        # BASELINE config 3 (long-context int8-KV decode attention, 32 q / 8 KV heads), measured live:
        # device time per launch from graph replays over rotating KV caches larger than L2
        from nova_b200.bench_kernels import bench_attn

        del dec
        torch.cuda.empty_cache()
        cases = []
        for ctx_l, b_l in ((32768, 1), (32768, 4), (32768, 16), (131072, 1)):
            r = bench_attn(ctx_l, b_l, iters=10)
            cases.append({"ctx": ctx_l, "batch": b_l, "us": r["us"], "gbs": r["gbs"],
                          "frac": round(r["gbs"] / peaks["hbm_gbs"], 3)})
            torch.cuda.empty_cache()
        line["attn_long_ctx"] = {"kernel": "attn_decode_int8_kernel", "bound": "hbm", "unit": "GB/s",
                                 "peak": peaks["hbm_gbs"], "cases": cases,
                                 "basis": "algorithmic bytes (272 B per cached token and KV head + ring + q/out) "
                                          "/ CUDA-event device time per launch"}
    if world == 1 and not args.no_cpu_baseline:
        from oracle.baseline import LayerSample, host_threads

        s = LayerSample(ctx=args.ctx, slice=1, seed=args.seed)
        s.run()
        times = []
        t_end = time.time() + 20
        while time.time() < t_end and len(times) < 20:
            times.append(s.run())
        tok_s = 1.0 / (statistics.median(times) * s.seconds_scale)
        line["cpu_baseline"] = {"value": tok_s, "unit": UNIT, "cores": host_threads(), "kind": "port",
                                "sample": f"{len(times)} x one full decoder layer at ctx {args.ctx} + 1/36 of the "
                                          "lm_head (NF4 dequant per call + fp32 numpy matmul, int8 KV dequant + fp32 "
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
