"""Lightning-indexer scores and the stable top-k rule, in numpy.
TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

``indexer_scores`` is ``cirrus/model/layers.py:282-288``
(``s = sum_h w_h * relu(q_h . k_s)``) evaluated in one fixed float32 order,
the order the CUDA scorer uses, so that equal inputs give bit-identical
scores and therefore bit-identical selections:

* per head, eight running sums ``p[r] = sum_i q[8i+r] * k[8i+r]`` (i ascending),
  then ``((p0+p1)+(p2+p3)) + ((p4+p5)+(p6+p7))``;
* ``relu(d) = d if d > 0 else +0``;
* ``score = w0*r0``, then ``score = score + w_h*r_h`` for h = 1, 2, ...

Every product and sum is rounded to float32 on its own (no fused multiply-add).

``topk_select`` is ``topk_mask`` (``layers.py:291-309``) for one query row:
keep the k causally visible keys with the largest score, ties broken towards
the most recent key (the reference sorts the flipped row stably), always keep
the query's own position, and keep every visible key when there are at most k.
"""

from __future__ import annotations

import numpy as np


def indexer_scores(iq: np.ndarray, iw: np.ndarray, ik: np.ndarray) -> np.ndarray:
    """iq float32 [Hi, Di], iw float32 [Hi], ik float32 [n, Di] -> float32 [n]."""
    iq = np.asarray(iq, dtype=np.float32)
    iw = np.asarray(iw, dtype=np.float32)
    ik = np.asarray(ik, dtype=np.float32)
    Hi, Di = iq.shape
    if Di % 8:
        raise ValueError("indexer_dim must be a multiple of 8")
    score = None
    for h in range(Hi):
        p = [ik[:, r] * iq[h, r] for r in range(8)]
        for i in range(1, Di // 8):
            for r in range(8):
                p[r] = p[r] + ik[:, 8 * i + r] * iq[h, 8 * i + r]
        d = ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]))
        rl = np.where(d > 0, d, np.float32(0.0)).astype(np.float32)
        term = rl * iw[h]
        score = term if score is None else score + term
    return score.astype(np.float32)


def topk_select(scores: np.ndarray, k: int) -> np.ndarray:
    """Selected key indices (ascending) for a query at position ``len(scores) - 1``
    that sees keys ``0 .. len(scores) - 1``."""
    s = np.asarray(scores, dtype=np.float32) + np.float32(0.0)  # -0 sorts with +0
    n = len(s)
    if n <= k:
        return np.arange(n, dtype=np.int64)
    idx = np.arange(n)
    order = np.lexsort((-idx, -s.astype(np.float64)))  # score desc, then most recent first
    sel = set(order[:k].tolist())
    sel.add(n - 1)  # the diagonal
    return np.array(sorted(sel), dtype=np.int64)
