"""Tensor parallelism for the decode step: the model is sharded by KV head
(attention) and by intermediate column / row (MLP) over the ranks of one node,
with one all-reduce after o_proj and one after down_proj per layer (the
north-star sharded configuration; the reference itself runs on one GPU).

Per rank r of W (KV heads Hkv, query heads Hq, intermediate I, head dim D):

    q_proj   rows of q heads  [r*Hq/W, (r+1)*Hq/W)      (column split)
    k/v_proj rows of KV heads [r*Hkv/W, (r+1)*Hkv/W)    (column split)
    o_proj   columns (K) of the same q heads            (row split -> partial sums)
    gate/up  rows [r*I/W, (r+1)*I/W)                    (column split)
    down     columns (K) [r*I/W, (r+1)*I/W)             (row split -> partial sums)

Embedding, norms, the 4-bit lm_head and the greedy argmax are replicated, so
every rank holds the same residual stream and emits the same token.  The KV
cache of a rank holds only its KV heads.  GQA keeps q head h on KV head
h // (Hq/Hkv), which the contiguous split preserves.

The slicing works on the reference NF4 layout (packed ``[N, K/2]``, absmax
``[K/64, N]``) and on any device, so the host logic is testable on the CPU.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class TPContext:
    """This process's place in the tensor-parallel group.  ``allreduce``:
    "p2p" = the fused NVLink peer-memory all-reduce + residual add of this
    library (one kernel), "nccl" = torch.distributed all-reduce + a separate
    residual-add kernel."""

    rank: int = 0
    world: int = 1
    group: object = None     # torch.distributed ProcessGroup (NCCL on GPUs, gloo in CPU tests)
    allreduce: str = "p2p"

    @property
    def active(self) -> bool:
        return self.world > 1


@dataclass(frozen=True)
class ShardRanges:
    q_heads: tuple[int, int]
    kv_heads: tuple[int, int]
    inter: tuple[int, int]


def shard_ranges(cfg, rank: int, world: int) -> ShardRanges:
    """Head and intermediate ranges of ``rank``; raises ValueError when the
    model does not split evenly into whole NF4 blocks and GEMV tiles."""
    hq, hkv, inter = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.intermediate_size
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if hkv % world or hq % world:
        raise ValueError(f"{hkv} KV heads / {hq} q heads do not split over {world} ranks")
    if inter % world or (inter // world) % 64:
        raise ValueError(f"intermediate size {inter} / {world} is not a multiple of 64")
    if (hq // world) * cfg.head_dim % 64:
        raise ValueError("the o_proj K split must be a multiple of 64")
    qh, kh, il = hq // world, hkv // world, inter // world
    return ShardRanges((rank * qh, (rank + 1) * qh), (rank * kh, (rank + 1) * kh), (rank * il, (rank + 1) * il))


def nf4_rows(packed: torch.Tensor, absmax: torch.Tensor, r0: int, r1: int):
    """Output rows [r0, r1) of an NF4 matrix (column-parallel shard)."""
    return packed[r0:r1].contiguous(), absmax[:, r0:r1].contiguous()


def nf4_cols(packed: torch.Tensor, absmax: torch.Tensor, k0: int, k1: int):
    """Input columns [k0, k1) of an NF4 matrix (row-parallel shard); k0 and k1
    must be multiples of the 64-element block."""
    if k0 % 64 or k1 % 64:
        raise ValueError("K shards must cover whole 64-element NF4 blocks")
    return packed[:, k0 // 2:k1 // 2].contiguous(), absmax[k0 // 64:k1 // 64].contiguous()


def shard_qkv(packed, absmax, cfg, sr: ShardRanges):
    """Rows of the concatenated q|k|v weight for this rank's heads, kept in
    q|k|v order."""
    d = cfg.head_dim
    qd, kvd = cfg.q_dim, cfg.kv_dim
    parts = [nf4_rows(packed, absmax, sr.q_heads[0] * d, sr.q_heads[1] * d),
             nf4_rows(packed, absmax, qd + sr.kv_heads[0] * d, qd + sr.kv_heads[1] * d),
             nf4_rows(packed, absmax, qd + kvd + sr.kv_heads[0] * d, qd + kvd + sr.kv_heads[1] * d)]
    return torch.cat([p for p, _ in parts]).contiguous(), torch.cat([a for _, a in parts], dim=1).contiguous()


def shard_gate_up(packed, absmax, sr: ShardRanges):
    """This rank's intermediate rows of the tile-interleaved gate|up weight
    (re-interleaved, so the SiLU*up epilogue still pairs them)."""
    from .decoder import deinterleave_gate_up, interleave_gate_up

    gp, ga, up, ua = deinterleave_gate_up(packed, absmax)
    i0, i1 = sr.inter
    g = nf4_rows(gp, ga, i0, i1)
    u = nf4_rows(up, ua, i0, i1)
    return interleave_gate_up(g[0], g[1], u[0], u[1])


def shard_layer_tensors(lw, cfg, sr: ShardRanges) -> dict:
    """Reference-layout (packed, absmax) shards of one layer's projections."""
    d = cfg.head_dim
    return {
        "qkv": shard_qkv(lw.qkv.packed, lw.qkv.absmax, cfg, sr),
        "o": nf4_cols(lw.o.packed, lw.o.absmax, sr.q_heads[0] * d, sr.q_heads[1] * d),
        "gate_up": shard_gate_up(lw.gate_up.packed, lw.gate_up.absmax, sr),
        "down": nf4_cols(lw.down.packed, lw.down.absmax, sr.inter[0], sr.inter[1]),
    }


def shard_weights(weights, rank: int, world: int):
    """DecoderWeights with every layer's projections cut to this rank's shard
    (native unit streams rebuilt); embedding, norms and lm_head are shared."""
    from .decoder import DecoderWeights, LayerWeights, NF4Weight

    cfg = weights.cfg
    sr = shard_ranges(cfg, rank, world)
    layers = []
    for lw in weights.layers:
        t = shard_layer_tensors(lw, cfg, sr)
        layers.append(LayerWeights(qkv=NF4Weight(*t["qkv"]), o=NF4Weight(*t["o"]), gate_up=NF4Weight(*t["gate_up"]),
                                   down=NF4Weight(*t["down"]), input_ln=lw.input_ln, post_ln=lw.post_ln,
                                   q_norm=lw.q_norm, k_norm=lw.k_norm))
    return DecoderWeights(cfg=cfg, embed=weights.embed, lm_head=weights.lm_head, final_norm=weights.final_norm,
                          layers=layers, code=weights.code)


def all_reduce_sum(t: torch.Tensor, tp: TPContext) -> None:
    """In-place sum over the tensor-parallel group (captured into the decode
    graph with the NCCL backend)."""
    if tp.active:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=tp.group)


class P2PAllReduce:
    """``nova_tp_allreduce_add`` over receive buffers shared by CUDA IPC: one
    per rank, mapped into every rank's process at construction (a collective
    call: every rank of the group must construct it)."""

    def __init__(self, tp: TPContext, rows: int, n: int, device, timeout_s: float = 2.0) -> None:
        import ctypes

        import torch.distributed as dist

        from . import _lib

        self.tp, self.rows, self.n = tp, int(rows), int(n)
        nbytes = ctypes.c_int64(0)
        _lib.call("nova_tp_recv_bytes", tp.world, self.rows, self.n, ctypes.byref(nbytes))
        self.recv = torch.zeros(int(nbytes.value), dtype=torch.uint8, device=device)
        self.epoch = torch.zeros(1, dtype=torch.int64, device=device)
        self.counter = torch.zeros(1, dtype=torch.int32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        handle = ctypes.create_string_buffer(64)
        off = ctypes.c_int64(0)
        _lib.call("nova_ipc_handle", self.recv.data_ptr(), handle, ctypes.byref(off))
        peers: list = [None] * tp.world
        dist.all_gather_object(peers, (bytes(handle.raw[:64]), int(off.value)), group=tp.group)
        self._bases = []
        ptrs = []
        for r, (h, o) in enumerate(peers):
            if r == tp.rank:
                ptrs.append(self.recv.data_ptr())
                continue
            ptr, base = ctypes.c_void_p(), ctypes.c_void_p()
            _lib.call("nova_ipc_open", ctypes.create_string_buffer(h, 64), o, ctypes.byref(ptr), ctypes.byref(base))
            self._bases.append(base.value)
            ptrs.append(ptr.value)
        dist.barrier(group=tp.group)
        a = _lib.TPAllReduceArgs()
        for r, ptr in enumerate(ptrs):
            a.recv[r] = ptr
        a.epoch, a.counter, a.err = self.epoch.data_ptr(), self.counter.data_ptr(), self.err.data_ptr()
        a.rows, a.n, a.rank, a.world = self.rows, self.n, tp.rank, tp.world
        a.timeout_ns = int(timeout_s * 1e9)
        self.args = a

    def __call__(self, partial: torch.Tensor, residual: torch.Tensor) -> None:
        """residual += all-reduced partial (fp16 rounding as in the decoder)."""
        import ctypes

        from . import _lib

        if partial.dtype != torch.float32 or not partial.is_contiguous() or partial.shape != (self.rows, self.n):
            raise ValueError("partial must be contiguous fp32 [rows, n]")
        a = self.args
        a.partial, a.residual, a.res_stride = partial.data_ptr(), residual.data_ptr(), residual.stride(0)
        _lib.check(_lib.lib().nova_tp_allreduce_add(ctypes.byref(a), _lib.stream_of(partial.device)),
                   "nova_tp_allreduce_add")

    def error(self) -> int:
        """Non-zero when a wait for a peer gave up (synchronizes)."""
        return int(self.err.item())

    def close(self) -> None:
        from . import _lib

        for b in self._bases:
            _lib.call("nova_ipc_close", b)
        self._bases = []


__all__ = ["TPContext", "ShardRanges", "shard_ranges", "nf4_rows", "nf4_cols", "shard_qkv", "shard_gate_up",
           "shard_layer_tensors", "shard_weights", "all_reduce_sum", "P2PAllReduce"]
