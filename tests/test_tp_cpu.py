"""CPU, world size 2 over gloo: the tensor-parallel sharding of the decode step
(nova_b200.tp) reproduces the unsharded projections -- column shards give the
same rows, row shards' partial sums all-reduced give the full product -- with
the reference-layout slicing and the same all-reduce helper the decoder uses.
The arithmetic is the CPU oracle's; no GPU is involved."""

from __future__ import annotations

import os
import socket
from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import nf4 as onf4


def _cfg():
    # small model that splits over 2 ranks the way the real one splits over up to 8
    return SimpleNamespace(num_attention_heads=4, num_key_value_heads=2, head_dim=64, hidden_size=256,
                           intermediate_size=256, q_dim=256, kv_dim=128)


def _weights(seed):
    cfg = _cfg()
    rng = np.random.default_rng(seed)
    code = onf4.nf4_codebook()

    def lin(n, k):
        p, a = onf4.quantize_nf4((rng.standard_normal((n, k)) * 0.02).astype(np.float16), code)
        return SimpleNamespace(packed=torch.from_numpy(p), absmax=torch.from_numpy(a))

    from nova_b200.decoder import interleave_gate_up

    q, k, v = lin(cfg.q_dim, cfg.hidden_size), lin(cfg.kv_dim, cfg.hidden_size), lin(cfg.kv_dim, cfg.hidden_size)
    gate, up = lin(cfg.intermediate_size, cfg.hidden_size), lin(cfg.intermediate_size, cfg.hidden_size)
    gu = interleave_gate_up(gate.packed, gate.absmax, up.packed, up.absmax)
    layer = SimpleNamespace(
        qkv=SimpleNamespace(packed=torch.cat([q.packed, k.packed, v.packed]),
                            absmax=torch.cat([q.absmax, k.absmax, v.absmax], dim=1)),
        o=lin(cfg.hidden_size, cfg.q_dim), gate_up=SimpleNamespace(packed=gu[0], absmax=gu[1]),
        down=lin(cfg.hidden_size, cfg.intermediate_size))
    return cfg, layer, gate, up, code


def _y(x, w, code):
    return onf4.nf4_linear(x, w[0].numpy(), w[1].numpy(), code)


def _rank_main(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from nova_b200.decoder import deinterleave_gate_up
        from nova_b200.tp import TPContext, all_reduce_sum, shard_layer_tensors, shard_ranges

        cfg, layer, gate, up, code = _weights(7)
        tp = TPContext(rank, world, dist.group.WORLD)
        sr = shard_ranges(cfg, rank, world)
        sh = shard_layer_tensors(layer, cfg, sr)
        rng = np.random.default_rng(100)
        x = rng.standard_normal((3, cfg.hidden_size)).astype(np.float32)
        attn = rng.standard_normal((3, cfg.q_dim)).astype(np.float32)
        act = rng.standard_normal((3, cfg.intermediate_size)).astype(np.float32)
        d = cfg.head_dim
        res = {}
        # column-parallel q|k|v: this rank's heads, in q|k|v order
        full = _y(x, (layer.qkv.packed, layer.qkv.absmax), code)
        qh, kh = sr.q_heads, sr.kv_heads
        want = np.concatenate([full[:, qh[0] * d:qh[1] * d],
                               full[:, cfg.q_dim + kh[0] * d:cfg.q_dim + kh[1] * d],
                               full[:, cfg.q_dim + cfg.kv_dim + kh[0] * d:cfg.q_dim + cfg.kv_dim + kh[1] * d]], 1)
        res["qkv"] = float(np.abs(_y(x, sh["qkv"], code) - want).max())
        # column-parallel gate|up, still tile-interleaved
        gp, ga, upp, ua = deinterleave_gate_up(*sh["gate_up"])
        i0, i1 = sr.inter
        res["gate"] = float(np.abs(_y(x, (gp, ga), code) - _y(x, (gate.packed, gate.absmax), code)[:, i0:i1]).max())
        res["up"] = float(np.abs(_y(x, (upp, ua), code) - _y(x, (up.packed, up.absmax), code)[:, i0:i1]).max())
        # row-parallel o_proj / down_proj: partial sums all-reduced over the group
        for name, inp, cols in (("o", attn, (qh[0] * d, qh[1] * d)), ("down", act, sr.inter)):
            part = torch.from_numpy(_y(inp[:, cols[0]:cols[1]], sh[name], code))
            all_reduce_sum(part, tp)
            w = getattr(layer, name)
            full = _y(inp, (w.packed, w.absmax), code)
            res[name] = float(np.abs(part.numpy() - full).max() / np.abs(full).max())
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), np.array([res[k] for k in sorted(res)]))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_projections_match_unsharded(tmp_path):
    mp.spawn(_rank_main, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        errs = np.load(tmp_path / f"rank{r}.npy")   # gate, o, qkv, down, up (sorted keys)
        assert errs.max() < 1e-5, errs


def test_shard_ranges_cover_and_reject():
    from nova_b200.decoder import DecoderConfig
    from nova_b200.tp import shard_ranges

    cfg = DecoderConfig()
    for world in (1, 2, 4, 8):
        rs = [shard_ranges(cfg, r, world) for r in range(world)]
        assert rs[0].q_heads[0] == 0 and rs[-1].q_heads[1] == cfg.num_attention_heads
        assert rs[-1].kv_heads[1] == cfg.num_key_value_heads and rs[-1].inter[1] == cfg.intermediate_size
        for a, b in zip(rs, rs[1:]):
            assert a.q_heads[1] == b.q_heads[0] and a.kv_heads[1] == b.kv_heads[0] and a.inter[1] == b.inter[0]
        # GQA: every q head of a rank maps to one of its KV heads
        gq = cfg.num_attention_heads // cfg.num_key_value_heads
        for r in rs:
            assert r.q_heads[0] // gq == r.kv_heads[0] and (r.q_heads[1] - 1) // gq == r.kv_heads[1] - 1
    with pytest.raises(ValueError):
        shard_ranges(cfg, 0, 3)
    with pytest.raises(ValueError):
        shard_ranges(cfg, 0, 16)
    with pytest.raises(ValueError):
        shard_ranges(cfg, 2, 2)


def test_nf4_col_shards_need_whole_blocks():
    from nova_b200.tp import nf4_cols

    p = torch.zeros(32, 64, dtype=torch.uint8)
    a = torch.zeros(2, 32, dtype=torch.float16)
    nf4_cols(p, a, 0, 64)
    with pytest.raises(ValueError):
        nf4_cols(p, a, 0, 32)


# ---------------------------------------------------------------- failure detection on the host


def _fault_rank(rank, world, port, out_dir, mode):
    """One rank of a 2-rank gloo group: a healthy all-reduce, then rank 1 fails
    before the next collective (``raise``: an exception ends its process;
    ``absent``: it stays alive but never joins) while rank 0 enters it."""
    import datetime
    import json
    import time

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=2))
    from nova_b200.tp import TPContext, all_reduce_sum

    tp = TPContext(rank, world, dist.group.WORLD, allreduce="nccl")
    t = torch.ones(16)
    all_reduce_sum(t, tp)
    if rank == 1:
        if mode == "raise":
            raise RuntimeError("injected fault: rank 1 fails before its next collective")
        time.sleep(10)
        os._exit(0)
    t0 = time.time()
    try:
        all_reduce_sum(t, tp)
        status = "completed"
    except Exception as e:   # noqa: BLE001 -- the point is that it raises instead of hanging
        status = type(e).__name__
    with open(os.path.join(out_dir, "rank0.json"), "w") as f:
        json.dump({"status": status, "seconds": time.time() - t0, "first": float(t[0])}, f)
    os._exit(0)


@pytest.mark.parametrize("mode", ["raise", "absent"])
def test_rank_failure_surfaces_as_an_error(tmp_path, mode):
    """A rank that dies (or never joins) before a collective of the decode
    step: the surviving rank's all-reduce ends with an error within the
    process group's timeout instead of hanging, and the healthy step before it
    was correct."""
    import json

    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_fault_rank, args=(r, 2, port, str(tmp_path), mode)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank did not exit")
    res = json.loads((tmp_path / "rank0.json").read_text())
    assert res["first"] == 2.0                  # the healthy all-reduce summed both ranks
    assert res["status"] != "completed", res
    assert res["seconds"] < 20, res             # bounded by the 2 s process-group timeout
    if mode == "raise":
        assert procs[1].exitcode != 0
