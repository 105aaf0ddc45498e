"""Next-token sampling on the logits buffer, outside the decode graph -- the
chat CLI's ``sample_next`` (src/chat.py:46-75) on ``nova_sample_topk``.

    tok = sample_next(dec.logits, args, seen_mask, gen)   # args: temperature, top_k, top_p, repetition_penalty

The graph keeps its in-graph argmax; sampling after the replay overwrites the
next step's input token (and here also its embedding row), as the reference's
CLI does with ``dec.input_ids.copy_(nxt)``.  The draw is one uniform number per
row from ``gen`` and an inverse-CDF pick from the same probabilities the
reference hands to ``torch.multinomial``.
"""

from __future__ import annotations

import torch

from . import _lib


def sample_topk(logits: torch.Tensor, *, temperature: float, top_k: int, top_p: float = 1.0,
                repetition_penalty: float = 1.0, seen: torch.Tensor | None = None,
                uniform: torch.Tensor | None = None, token_out: torch.Tensor | None = None,
                embed: torch.Tensor | None = None, embed_out: torch.Tensor | None = None,
                seen_mark: torch.Tensor | None = None, probs_out: torch.Tensor | None = None,
                idx_out: torch.Tensor | None = None) -> torch.Tensor:
    """``nova_sample_topk`` on fp16 logits ``[rows, vocab]``; returns the int64
    tokens ``[rows]``.  ``seen``/``seen_mark``: uint8 or bool ``[rows, vocab]``
    (or ``[vocab]`` for one row); ``uniform``: fp32 ``[rows]`` in [0, 1)."""
    if logits.dim() == 1:
        logits = logits.view(1, -1)
    rows, vocab = logits.shape
    if logits.dtype != torch.float16 or logits.stride(1) != 1:
        raise ValueError("logits must be float16 with a contiguous last dimension")
    k = int(top_k) if top_k > 0 else 64
    tok = token_out if token_out is not None else torch.empty(rows, dtype=torch.int64, device=logits.device)

    def u8(t):
        if t is None:
            return None
        t = t.view(-1, vocab) if t.dim() == 1 else t
        return t.view(torch.uint8) if t.dtype == torch.bool else t

    seen8, mark8 = u8(seen), u8(seen_mark)
    a = _lib.SampleArgs()
    a.logits, a.logits_stride = logits.data_ptr(), logits.stride(0)
    a.seen, a.seen_stride = (_lib.ptr(seen8), seen8.stride(0) if seen8 is not None and seen8.shape[0] > 1 else 0)
    a.uniform = _lib.ptr(uniform)
    a.token_out = tok.data_ptr()
    a.embed = _lib.ptr(embed)
    a.embed_out = _lib.ptr(embed_out)
    a.embed_out_stride = embed_out.stride(0) if embed_out is not None else 0
    a.embed_dim = embed.shape[1] if embed is not None else 0
    a.probs_out, a.idx_out = _lib.ptr(probs_out), _lib.ptr(idx_out)
    a.seen_mark = _lib.ptr(mark8)
    a.seen_mark_stride = mark8.stride(0) if mark8 is not None and mark8.shape[0] > 1 else 0
    a.rows, a.vocab, a.top_k = rows, vocab, min(k, vocab)
    a.temperature, a.top_p, a.repetition_penalty = float(temperature), float(top_p), float(repetition_penalty)
    _lib.check(_lib.lib().nova_sample_topk(_lib.ctypes.byref(a), _lib.stream_of(logits.device)), "nova_sample_topk")
    return tok


def sample_next(logits: torch.Tensor, args, seen_mask: torch.Tensor | None, gen: torch.Generator | None = None
                ) -> torch.Tensor:
    """Drop-in for the chat CLI's ``sample_next(logits [1, vocab], args,
    seen_mask, gen) -> [1, 1]`` (src/chat.py:46-75)."""
    _lib.require_cuda(logits, names=("logits",))
    rows = logits.shape[0] if logits.dim() == 2 else 1
    u = None
    if args.temperature > 0:
        u = torch.rand(rows, generator=gen, device=logits.device if gen is None else gen.device)
        u = u.to(logits.device, torch.float32)
    lg = logits if logits.dtype == torch.float16 else logits.to(torch.float16)
    tok = sample_topk(lg, temperature=args.temperature, top_k=args.top_k, top_p=args.top_p,
                      repetition_penalty=args.repetition_penalty,
                      seen=seen_mask if args.repetition_penalty != 1.0 else None, uniform=u)
    return tok.view(rows, 1)
