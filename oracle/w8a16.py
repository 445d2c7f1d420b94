"""W8A16 GEMV, fused gate_up SiLU and greedy argmax, restated in numpy (test oracle).

Semantics (kernels/sglang/srt/layers/quantization/w8a16_gemv.py):
* y[m, n] = (sum_k w[n, k] * x[m, k]) * s[n]; one-byte weights (fp8 e4m3 or int8) are
  widened exactly; the scale is applied once per output after the k sum (:266-270); the
  result is rounded to bf16 and only then widened when the destination is fp32 (:92-95).
* scales: [N], [N, 1] or a scalar, fp32 or bf16 (the host upcasts to fp32, :660-662).
* fused gate_up: silu(g) * u with g = x.w[j] * s[j], u = x.w[H + j] * s[H + j], the
  activation evaluated on the unrounded fp32 values (:1009-1018, :930-935).
* greedy argmax over the bf16-rounded logits, lowest index on ties (torch.argmax).
"""

from __future__ import annotations

import numpy as np

from .numerics import bf16_round, bf16_round_from_f64, e4m3_to_f32


def weight_values(w: np.ndarray, kind: str) -> np.ndarray:
    """Exact fp64 values of a weight stored as 'int8', 'fp8' (e4m3 bytes) or 'bf16' (fp32 values)."""
    if kind == "int8":
        return np.asarray(w, dtype=np.int8).astype(np.float64)
    if kind == "fp8":
        return e4m3_to_f32(np.asarray(w, dtype=np.uint8)).astype(np.float64)
    if kind == "bf16":
        return np.asarray(w, dtype=np.float64)
    raise ValueError(kind)


def gemv_f64(x_bf16: np.ndarray, w: np.ndarray, kind: str, scale,
             row_chunk: int = 16384) -> np.ndarray:
    """Unrounded fp64 logits (x @ w^T) * s (rows in chunks to bound memory)."""
    x = np.asarray(x_bf16, dtype=np.float64)
    s = np.asarray(scale, dtype=np.float64).reshape(-1)
    N = np.asarray(w).shape[0]
    y = np.empty((x.shape[0], N), dtype=np.float64)
    for r0 in range(0, N, row_chunk):
        r1 = min(N, r0 + row_chunk)
        y[:, r0:r1] = x @ weight_values(w[r0:r1], kind).T
    return y * (s[None, :] if s.size > 1 else s[0])


def gemv(x_bf16: np.ndarray, w: np.ndarray, kind: str, scale) -> np.ndarray:
    """bf16-rounded logits (as fp32 values)."""
    return bf16_round_from_f64(gemv_f64(x_bf16, w, kind, scale))


def argmax_lowest(logits: np.ndarray) -> np.ndarray:
    """Row-wise argmax, lowest index among equal maxima (torch.argmax semantics)."""
    logits = np.asarray(logits)
    return np.argmax(logits, axis=-1).astype(np.int64)  # numpy also returns the first max


def top2_gap(logits_f64: np.ndarray) -> np.ndarray:
    """Gap between the largest and second-largest exact logit of each row."""
    part = np.partition(np.asarray(logits_f64, dtype=np.float64), -2, axis=-1)
    return part[..., -1] - part[..., -2]


def silu_mul(x_bf16: np.ndarray, w: np.ndarray, kind: str, scale) -> np.ndarray:
    """bf16(silu(g) * u) of the fused gate_up form, evaluated in fp64."""
    y = gemv_f64(x_bf16, w, kind, scale)
    h = y.shape[1] // 2
    g, u = y[:, :h], y[:, h:]
    return bf16_round_from_f64(g / (1.0 + np.exp(-g)) * u)


def silu_mul_two_step(x_bf16: np.ndarray, w: np.ndarray, kind: str, scale) -> np.ndarray:
    """The unfused reference path: bf16 gate_up, then act_and_mul in fp32 -> bf16."""
    y = gemv(x_bf16, w, kind, scale).astype(np.float32)
    h = y.shape[1] // 2
    g, u = y[:, :h], y[:, h:]
    return bf16_round((g / (np.float32(1) + np.exp(-g))) * u)


def reference_cpu_path(x: np.ndarray, w: np.ndarray, kind: str, scale):
    """The reference's torch CPU path in fp32, restated: W = w.float() * s[:, None];
    logits = bf16(x.float() @ W^T); token = argmax (used as the timed CPU baseline)."""
    wf = weight_values(w, kind).astype(np.float32) if kind != "int8" else np.asarray(w, np.float32)
    s = np.asarray(scale, dtype=np.float32).reshape(-1)
    W = wf * (s[:, None] if s.size > 1 else s[0])
    logits = bf16_round(np.asarray(x, dtype=np.float32) @ W.T)
    return logits, argmax_lowest(logits)


def gated_rmsnorm(x_bf16: np.ndarray, z_bf16: np.ndarray, norm_weight: np.ndarray,
                  group_size: int, eps: float, sigmoid_gate: bool = False,
                  bf16_cast=bf16_round) -> np.ndarray:
    """The fused norm prologue of w8a16_gemv_norm_gated (w8a16_gemv.py:186-190, :220-233,
    :246-255), in fp32: every contiguous group_size slice of a row is its own RMS group,
    y = x * rsqrt(mean(x^2) + eps) * w[k % G] * gate(z) with gate = z * sigmoid(z)
    (silu) or sigmoid(z), cast to bf16 before the dot.  bf16_cast is round-to-nearest-even
    (the GPU's cast); a test may pass a truncating cast to emulate the Triton CPU
    interpreter."""
    x = np.asarray(x_bf16, dtype=np.float32)
    z = np.asarray(z_bf16, dtype=np.float32)
    M, K = x.shape
    G = group_size
    xg = x.reshape(M, K // G, G)
    var = (xg * xg).sum(axis=-1, dtype=np.float32) / np.float32(G)
    rstd = (np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)
    yn = xg * rstd[..., None] * np.asarray(norm_weight, dtype=np.float32)[None, None, :]
    zg = z.reshape(M, K // G, G)
    sig = (np.float32(1.0) / (np.float32(1.0) + np.exp(-zg))).astype(np.float32)
    yn = yn * (sig if sigmoid_gate else zg * sig)
    return bf16_cast(yn.reshape(M, K).astype(np.float32))


def gemv_norm_gated(x_bf16, z_bf16, norm_weight, group_size, eps, w, kind, scale,
                    sigmoid_gate: bool = False) -> np.ndarray:
    """bf16 logits of (gated_rmsnorm(x, z) @ w^T) * s (w8a16_gemv.py:780-823)."""
    xn = gated_rmsnorm(x_bf16, z_bf16, norm_weight, group_size, eps, sigmoid_gate)
    return gemv(xn, w, kind, scale)


def draft_topk1(logits: np.ndarray, positions: np.ndarray, draft_tokens=None,
                draft_token_column: int = 0, hot_token_id=None):
    """draft_topk1_postprocess (patches/sglang/series/0016-…patch:46-73): the argmax of
    each row (lowest column on ties), mapped through hot_token_id; returns (topk_p ones
    [B, 1], topk_index [B, 1], new positions, new draft_tokens)."""
    idx = argmax_lowest(np.asarray(logits, np.float64))
    tok = idx if hot_token_id is None else np.asarray(hot_token_id)[idx]
    dt = None
    if draft_tokens is not None:
        dt = np.array(draft_tokens, copy=True)
        dt[:, draft_token_column] = tok
    return (np.ones((len(idx), 1), np.float32), tok.reshape(-1, 1).astype(np.int64),
            np.asarray(positions) + 1, dt)
