"""MoE router: logits projection and softmax top-k, restated in numpy (test oracle).

* ``router_logits``: x . W^T (+ bias) of bf16 inputs, fp32 result without rounding
  (kernels/sglang/srt/layers/moe/router_gemv.py:10-45: tl.dot with fp32 accumulation,
  bias added in fp32, fp32 store), computed here in fp64.
* ``softmax_topk``: the packed-key softmax top-k router
  (patches/sglang/series/0110-moe-router-packed-key-softmax-top-k-SGLANG_ROUTER_FA.patch:
  60-130, as changed by 0111): biased = score + bias; weights exp(b - max) / sum over
  the row; the topk largest biased values in descending order, the lowest expert id
  winning ties, a NaN ranked as the -1e30 floor and -0.0 as +0.0 (it is +0.0 after the
  zero bias); with renormalize the picked weights are divided by their sum when it is
  positive.  A NaN anywhere in a row makes its sum, so all its weights, NaN.
"""

from __future__ import annotations

import numpy as np


def router_logits(x_bf16: np.ndarray, w_bf16: np.ndarray, bias=None) -> np.ndarray:
    y = np.asarray(x_bf16, np.float64) @ np.asarray(w_bf16, np.float64).T
    if bias is not None:
        y = y + np.asarray(bias, np.float64)[None, :]
    return y


def softmax_topk(scores: np.ndarray, topk: int, renormalize: bool, bias=None):
    """(weights float64 [M, topk], ids int32 [M, topk]) of fp32/bf16 scores [M, N]."""
    s = np.asarray(scores, np.float32).astype(np.float64)
    if bias is not None:
        s = s + np.asarray(bias, np.float64)[None, :]
    M, N = s.shape
    w = np.zeros((M, topk))
    ids = np.zeros((M, topk), np.int32)
    for m in range(M):
        row = s[m]
        rank = np.where(np.isnan(row), -1e30, row) + 0.0  # -0.0 -> +0.0
        order = np.lexsort((np.arange(N), -rank))[:topk]  # value desc, then id asc
        valid = row[~np.isnan(row)]
        mx = valid.max() if valid.size else np.nan
        with np.errstate(invalid="ignore", over="ignore"):
            den = np.exp(row - mx).sum()
            picked = np.exp(rank[order] - mx) / den
        if renormalize:
            tot = picked.sum()
            picked = picked / (tot if tot > 0 else 1.0)
        w[m] = picked
        ids[m] = order
    return w, ids
