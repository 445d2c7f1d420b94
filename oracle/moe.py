"""Routed NVFP4 MoE layer, restated in numpy (test oracle).

Follows the reference's per-route dequantised reference
(bench/bench/moe_smallm/refs.py:50-78, and the "dqb" variant of
bench/bench/dg1/layer.py:57-73 that rounds the activation to bf16 between the two
GEMVs, which is the arithmetic of the kernels in
patches/sglang/series/0112-DG1-one-token-draft-MoE-as-a-W4A16-NVFP4-Triton-GEMV.patch:182-287):

    for each token t and route r with e = ids[t, r] >= 0:
        h    = dequant(w13[e]) @ x[t]            (both halves scaled by g13[e, 0])
        act  = silu(gate) * up                    (optionally rounded to bf16)
        out += w[t, r] * (dequant(w2[e]) @ act)
    out += shared expert (weight 1.0), if given
    out  -> bf16

Row order: "server" = w13 rows [up(I); gate(I)] (0112-...patch:68-75); "checkpoint" =
[gate; up] (refs.py:73-74).  Block scales are passed in the linear [rows, K/16] layout;
``nvfp4.unswizzle_blockscale`` recovers it from the server's swizzled tensor.
"""

from __future__ import annotations

import numpy as np

from . import nvfp4
from .numerics import bf16_round_from_f64


class _ExpertCache:
    def __init__(self, w13, s13, g13, w2, s2, g2):
        self.w13, self.s13, self.g13 = w13, s13, np.asarray(g13, dtype=np.float32)
        self.w2, self.s2, self.g2 = w2, s2, np.asarray(g2, dtype=np.float32)
        self._cache = {}

    def get(self, e: int):
        hit = self._cache.get(e)
        if hit is None:
            g13 = self.g13.reshape(self.g13.shape[0], -1)[e, 0]
            g2 = self.g2.reshape(-1)[e]
            w13 = nvfp4.dequantize(self.w13[e], self.s13[e], g13).astype(np.float64)
            w2 = nvfp4.dequantize(self.w2[e], self.s2[e], g2).astype(np.float64)
            hit = (w13, w2)
            self._cache[e] = hit
        return hit


def _expert(x64: np.ndarray, w13: np.ndarray, w2: np.ndarray, order: str, act_round: bool):
    I = w13.shape[0] // 2
    h = w13 @ x64
    if order == "server":
        up, gate = h[:I], h[I:]
    elif order == "checkpoint":
        gate, up = h[:I], h[I:]
    else:
        raise ValueError(order)
    act = gate / (1.0 + np.exp(-gate)) * up
    if act_round:
        act = bf16_round_from_f64(act).astype(np.float64)
    return w2 @ act


def moe_f64(x_bf16, ids, wts, w13, s13, g13, w2, s2, g2, shared=None, order="server",
            act_round=True, expert_offset=0, num_local=None):
    """Unrounded fp64 layer output [M, H].

    ``shared``: optional dict with keys w13, s13, g13 (scalar), w2, s2, g2 (scalar) of one
    always-on expert (weight 1.0).  ``expert_offset`` / ``num_local`` restrict the sum to
    one expert-parallel shard (ids outside it are skipped, like ids < 0).
    """
    x = np.asarray(x_bf16, dtype=np.float64)
    ids = np.asarray(ids)
    wts = np.asarray(wts, dtype=np.float32)
    M, H = x.shape
    E = np.asarray(w13).shape[0] if num_local is None else num_local
    bank = _ExpertCache(w13, s13, g13, w2, s2, g2)
    sh = None
    if shared is not None:
        sh = (
            nvfp4.dequantize(shared["w13"], shared["s13"], shared["g13"]).astype(np.float64),
            nvfp4.dequantize(shared["w2"], shared["s2"], shared["g2"]).astype(np.float64),
        )
    out = np.zeros((M, H), dtype=np.float64)
    for t in range(M):
        acc = np.zeros(H, dtype=np.float64)
        for r in range(ids.shape[1]):
            e = int(ids[t, r]) - expert_offset
            if int(ids[t, r]) < 0 or e < 0 or e >= E:
                continue
            a13, a2 = bank.get(e)
            acc += _expert(x[t], a13, a2, order, act_round) * np.float64(wts[t, r])
        if sh is not None:
            acc += _expert(x[t], sh[0], sh[1], order, act_round)
        out[t] = acc
    return out


def moe(*args, **kwargs) -> np.ndarray:
    """bf16-rounded layer output (fp32 values) [M, H]."""
    return bf16_round_from_f64(moe_f64(*args, **kwargs))


def distinct_experts(ids: np.ndarray, num_experts: int) -> int:
    ids = np.asarray(ids).reshape(-1)
    return int(np.unique(ids[(ids >= 0) & (ids < num_experts)]).size)
