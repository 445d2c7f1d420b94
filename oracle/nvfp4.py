"""NVFP4 codec and GEMV, restated in numpy (test oracle).

Format (kernels/sglang/srt/layers/quantization/w4a16_nvfp4_gemv.py:3-9):
    W[n, k] = e2m1(code[n, k]) * e4m3(bs[n, k // 16]) * gscale
``wq[N, K/2]`` uint8 holds two codes per byte, low nibble = even k; ``bs[N, K/16]`` holds
e4m3 bit patterns; ``gscale`` is an fp32 scalar or ``[N]``.
"""

from __future__ import annotations

import numpy as np

from .numerics import (
    E2M1_MAX,
    E4M3_MAX,
    bf16_round_from_f64,
    e2m1_to_f32,
    e4m3_to_f32,
    f32_to_e4m3,
    round_e2m1,
)

BLOCK = 16


def unpack_codes(wq: np.ndarray) -> np.ndarray:
    """[..., K/2] uint8 -> [..., K] codes, low nibble first (bench/bench/moe_smallm/refs.py:30-36)."""
    wq = np.asarray(wq, dtype=np.uint8)
    out = np.empty(wq.shape[:-1] + (wq.shape[-1] * 2,), dtype=np.uint8)
    out[..., 0::2] = wq & 0x0F
    out[..., 1::2] = wq >> 4
    return out


def pack_codes(codes: np.ndarray) -> np.ndarray:
    """[..., K] codes -> [..., K/2] bytes (inverse of unpack_codes)."""
    codes = np.asarray(codes, dtype=np.uint8)
    return (codes[..., 0::2] | (codes[..., 1::2] << 4)).astype(np.uint8)


def dequantize(wq: np.ndarray, bs: np.ndarray, gscale) -> np.ndarray:
    """fp32 [N, K] weight (w4a16_nvfp4_gemv.py:489-510): val * (e4m3(bs) * g) per 16-block."""
    val = e2m1_to_f32(unpack_codes(wq))
    g = np.asarray(gscale, dtype=np.float32).reshape(-1)
    g = g.reshape(-1, 1) if g.size > 1 else g.reshape(1, 1)
    s = (e4m3_to_f32(bs) * g).astype(np.float32)
    return (val * np.repeat(s, BLOCK, axis=1)).astype(np.float32)


def quantize(w: np.ndarray):
    """[N, K] weight -> (wq uint8 [N, K/2], bs uint8 [N, K/16], gscale fp32 [1]).

    The ModelOpt convention of w4a16_nvfp4_gemv.py:426-472, step for step in fp32:
    gscale = amax / (448 * 6) (clamped to 1e-30); enc = 1 / gscale; per 16-block
    sb = clamp(amax_b / 6 * enc, 0, 448) -> e4m3; eff = e4m3(sb) / enc;
    code = round_e2m1(|w / eff|) | sign (a block whose eff is 0 encodes to 0).
    """
    w = np.asarray(w, dtype=np.float32)
    N, K = w.shape
    assert K % BLOCK == 0
    gmax = np.float32(np.abs(w).max()) if w.size else np.float32(0)
    gscale = np.float32(max(np.float32(gmax / np.float32(E4M3_MAX * E2M1_MAX)), np.float32(1e-30)))
    enc = np.float32(np.float32(1.0) / gscale)
    blk = w.reshape(N, K // BLOCK, BLOCK)
    amax = np.abs(blk).max(axis=-1).astype(np.float32)
    sb = np.clip((amax / np.float32(E2M1_MAX)).astype(np.float32) * enc, 0.0, E4M3_MAX).astype(np.float32)
    bs = f32_to_e4m3(sb)
    eff = (e4m3_to_f32(bs) / enc).astype(np.float32)[..., None]
    with np.errstate(divide="ignore", invalid="ignore"):
        a = np.where(eff > 0, blk / np.maximum(eff, np.float32(1e-38)), np.float32(0)).astype(np.float32)
    code = round_e2m1(np.abs(a)) | ((a < 0).astype(np.uint8) * 8)
    wq = pack_codes(code.reshape(N, K))
    return wq, bs, np.array([gscale], dtype=np.float32)


def swizzle_blockscale(sf: np.ndarray) -> np.ndarray:
    """128x4 block-scale swizzle with zero padding (bench/bench/moe_smallm/weights.py:156-175).

    [.., M, K] -> [.., Mp, Kp] with Mp = ceil(M/128)*128, Kp = ceil(K/4)*4:
    reshape to [B, Mp/128, 4, 32, Kp/4, 4] and permute to [B, Mp/128, Kp/4, 32, 4, 4].
    """
    sf = np.asarray(sf)
    two_d = sf.ndim == 2
    if two_d:
        sf = sf[None]
    B, M, K = sf.shape
    Mp, Kp = (M + 127) // 128 * 128, (K + 3) // 4 * 4
    pad = np.zeros((B, Mp, Kp), dtype=sf.dtype)
    pad[:, :M, :K] = sf
    sw = pad.reshape(B, Mp // 128, 4, 32, Kp // 4, 4).transpose(0, 1, 4, 3, 2, 5)
    sw = np.ascontiguousarray(sw).reshape(B, Mp, Kp)
    return sw[0] if two_d else sw


def swizzled_offset(m: int, kb: int, kp: int) -> int:
    """Byte offset of scale (m, kb) in one swizzled [M, KP] block (0112-...patch:165-177)."""
    return (m // 128) * 128 * kp + (kb // 4) * 512 + (m % 32) * 16 + ((m % 128) // 32) * 4 + kb % 4


def unswizzle_blockscale(sw: np.ndarray, M: int, K: int) -> np.ndarray:
    """Inverse of swizzle_blockscale for M % 128 == 0 and K % 4 == 0."""
    sw = np.asarray(sw)
    two_d = sw.ndim == 2
    if two_d:
        sw = sw[None]
    B = sw.shape[0]
    x = sw.reshape(B, M // 128, K // 4, 32, 4, 4).transpose(0, 1, 4, 3, 2, 5)
    x = np.ascontiguousarray(x).reshape(B, M, K)
    return x[0] if two_d else x


def gemv(x_bf16: np.ndarray, wq: np.ndarray, bs: np.ndarray, gscale) -> np.ndarray:
    """y = bf16(x @ dequant(W)^T), fp64 accumulation (the north star's oracle path)."""
    w = dequantize(wq, bs, gscale).astype(np.float64)
    y = np.asarray(x_bf16, dtype=np.float64) @ w.T
    return bf16_round_from_f64(y)
