"""CPU restatement of the chat CLI's next-token sampling (test infrastructure;
only tests/, smoke() and bench.py's CPU legs may use it).

Follows sample_next, src/chat.py:46-75: greedy argmax at temperature <= 0;
otherwise fp32 logits, repetition penalty on seen tokens (l < 0 ? l * rp :
l / rp), the top_k largest (64 when top_k <= 0), softmax(vals / temperature),
tokens whose exclusive cumulative probability exceeds top_p dropped,
renormalized.  The reference then draws with torch.multinomial; the restatement
(and nova_sample_topk) pick by inverse CDF from a given uniform number.  Ties at
the top-k boundary are broken by lowest index (torch.topk leaves that order
unspecified).  Pinned by tests/golden/sampling.npz, produced by the reference's
own sample_next.
"""

from __future__ import annotations

import numpy as np


def sample_probs(logits: np.ndarray, seen: np.ndarray | None, temperature: float, top_k: int, top_p: float,
                 repetition_penalty: float) -> tuple[np.ndarray, np.ndarray]:
    """(candidate token ids in descending order, final probabilities) for one
    row of fp16 logits; the probabilities past the top-p cut are 0."""
    l = np.asarray(logits).astype(np.float32)
    if repetition_penalty != 1.0 and seen is not None:
        rp = np.float32(repetition_penalty)
        pen = np.where(l < 0, l * rp, l / rp).astype(np.float32)
        l = np.where(np.asarray(seen, dtype=bool), pen, l)
    k = min(top_k if top_k > 0 else 64, l.shape[0])
    order = np.lexsort((np.arange(l.shape[0]), -l.astype(np.float64)))[:k]   # value desc, index asc
    x = (l[order] / np.float32(temperature)).astype(np.float32)
    e = np.exp((x - x[0]).astype(np.float32)).astype(np.float32)
    p = (e / e.sum(dtype=np.float32)).astype(np.float32)
    if top_p < 1.0:
        drop = (np.cumsum(p, dtype=np.float32) - p) > np.float32(top_p)
        p = np.where(drop, np.float32(0), p)
        p = (p / p.sum(dtype=np.float32)).astype(np.float32)
    return order.astype(np.int64), p


def sample_token(logits: np.ndarray, seen: np.ndarray | None, temperature: float, top_k: int, top_p: float,
                 repetition_penalty: float, u: float) -> int:
    """The token for uniform draw u in [0, 1): greedy at temperature <= 0, else
    the first candidate whose cumulative probability exceeds u."""
    if temperature <= 0:
        lf = np.asarray(logits).astype(np.float32)
        return int(np.argmax(lf))   # first index of the maximum
    idx, p = sample_probs(logits, seen, temperature, top_k, top_p, repetition_penalty)
    c = np.cumsum(p, dtype=np.float32)
    kept = int(np.count_nonzero(p))
    i = int(np.searchsorted(c[:kept], np.float32(u), side="right"))
    return int(idx[min(i, kept - 1)])
