"""W4A16 NVFP4 skinny GEMV (M <= 16) and the NVFP4 codec, on the sm_100a library.

Host-side mirror of ``kernels/sglang/srt/layers/quantization/w4a16_nvfp4_gemv.py``:

    W[n, k] = e2m1(code[n, k]) * e4m3(bs[n, k // 16]) * gscale

``wq[N, K/2]`` uint8 holds two codes per byte, low nibble = even k; ``bs[N, K/16]`` holds
e4m3 bit patterns (uint8 or float8_e4m3fn); ``gscale`` is the plain fp32 global scale,
scalar or ``[N]``.  The kernel decodes e2m1 natively (``cvt.rn.f16x2.e2m1x2``), so no
2^14 factor appears anywhere.

``quantize_nvfp4`` / ``dequantize_nvfp4`` are the load-time codec (ModelOpt convention,
w4a16_nvfp4_gemv.py:426-510), written here with torch tensor ops on the weight's device;
they are not on the decode path.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from ._lib import check, ptr
from .w8a16_gemv import (
    PDL,
    _activation,
    _argmax_dest,
    _cfg,
    _split_dests,
    _stream,
    _workspace,
)

FP4_SCALE_BLOCK = 16
E4M3_MAX = 448.0
E2M1_MAX = 6.0
_E2M1_LEVELS = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
_E2M1_MID = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)
_TIE_UP = (0.75, 1.75, 3.5)


def w4a16_nvfp4_gemv(
    x: torch.Tensor,
    wq: torch.Tensor,
    bs: torch.Tensor,
    gscale: torch.Tensor,
    cfg=None,
    out: Optional[torch.Tensor] = None,
    out2: Optional[torch.Tensor] = None,
    split_n: int = 0,
    argmax_out: Optional[torch.Tensor] = None,
    pdl: Optional[bool] = None,
):
    """x: [M,K] bf16; wq: [N,K//2] uint8; bs: [N,K//16] e4m3; gscale: fp32 scalar or [N]."""
    M, K = x.shape
    N = wq.shape[0]
    assert wq.shape[1] == K // 2 and bs.shape == (N, K // FP4_SCALE_BLOCK)
    assert M <= 16 and wq.stride(1) == 1 and bs.stride(1) == 1
    y, y2, split_n = _split_dests(out, out2, split_n, M, N, x.device)
    g = gscale.reshape(-1)
    if g.dtype != torch.float32 or not g.is_contiguous():
        g = g.contiguous().float()
    if g.numel() not in (1, N):
        raise ValueError(f"gscale must be a scalar or [{N}]")
    x = _activation(x)
    am = _argmax_dest(argmax_out, M, x.device)
    ws = _workspace(x.device)
    c = _cfg(cfg)
    rc = _lib.lib().fnx_w4a16_nvfp4_gemv(
        ptr(x), x.stride(0), ptr(wq), wq.stride(0), ptr(bs), bs.stride(0), ptr(g), int(g.numel() > 1),
        ptr(y), y.stride(0), ptr(y2), 0 if y2 is None else y2.stride(0), split_n,
        int(y.dtype == torch.float32), ptr(am), None, 0, M, N, K,
        None if c is None else ctypes.byref(c), ctypes.byref(ws.c), int(PDL if pdl is None else pdl),
        _stream(x))
    check(rc, "w4a16_nvfp4_gemv")
    return y if y2 is None else (y, y2)


def _round_e2m1(a: torch.Tensor) -> torch.Tensor:
    """|a| in block-scale units -> magnitude code 0..7, nearest level, ties to the even code."""
    mids = torch.tensor(_E2M1_MID, dtype=torch.float32, device=a.device)
    idx = torch.bucketize(a, mids, right=False)
    tie = (a == _TIE_UP[0]) | (a == _TIE_UP[1]) | (a == _TIE_UP[2])
    return (idx + tie).clamp_(0, 7).to(torch.uint8)


def quantize_nvfp4(w: torch.Tensor, block: int = FP4_SCALE_BLOCK, row_chunk: int = 4096):
    """[N, K] weight -> (wq [N, K//2] uint8, bs [N, K//16] uint8 e4m3 bits, gscale fp32 [1]).

    gscale = amax(|W|) / (448 * 6); per 16-block scale amax_b / 6 * (1 / gscale) rounded
    to e4m3; codes = round_e2m1(W / (e4m3(bs) / (1 / gscale))).  Chunked over rows so the
    transient is row_chunk * K fp32.
    """
    assert w.dim() == 2 and w.shape[1] % block == 0
    N, K = w.shape
    gmax = torch.zeros((), dtype=torch.float32, device=w.device)
    for r0 in range(0, N, row_chunk):
        gmax = torch.maximum(gmax, w[r0:r0 + row_chunk].float().abs().amax())
    gscale = (gmax / (E4M3_MAX * E2M1_MAX)).clamp_(min=1e-30)
    enc = 1.0 / gscale
    wq = torch.empty((N, K // 2), dtype=torch.uint8, device=w.device)
    bs = torch.empty((N, K // block), dtype=torch.uint8, device=w.device)
    for r0 in range(0, N, row_chunk):
        r1 = min(N, r0 + row_chunk)
        blk = w[r0:r1].float().view(r1 - r0, K // block, block)
        amax = blk.abs().amax(dim=-1)
        sb8 = (amax / E2M1_MAX * enc).clamp_(min=0.0, max=E4M3_MAX).to(torch.float8_e4m3fn)
        bs[r0:r1] = sb8.view(torch.uint8)
        eff = (sb8.float() / enc).unsqueeze(-1)
        a = torch.where(eff > 0, blk / eff.clamp(min=1e-38), torch.zeros_like(blk))
        code = (_round_e2m1(a.abs()) | (a < 0).to(torch.uint8) * 8).reshape(r1 - r0, K)
        wq[r0:r1] = code[:, 0::2] | (code[:, 1::2] << 4)
    return wq, bs, gscale.reshape(1)


_LEVELS: dict = {}


def dequantize_nvfp4(wq: torch.Tensor, bs: torch.Tensor, gscale: torch.Tensor,
                     block: int = FP4_SCALE_BLOCK) -> torch.Tensor:
    """fp32 [N, K] weight (the wide-M fallback and the numerics reference).  The level
    table is cached per device so the call is graph-capture safe."""
    N, KH = wq.shape
    K = KH * 2
    lvl = _LEVELS.get(wq.device)
    if lvl is None:
        lvl = torch.tensor(_E2M1_LEVELS, dtype=torch.float32, device=wq.device)
        _LEVELS[wq.device] = lvl
    code = torch.empty((N, K), dtype=torch.uint8, device=wq.device)
    code[:, 0::2] = wq & 0x0F
    code[:, 1::2] = wq >> 4
    mag = lvl[(code & 0x07).long()]
    val = torch.where((code & 0x08) > 0, -mag, mag)
    g = gscale.to(wq.device, torch.float32).reshape(-1)
    g = g.reshape(-1, 1) if g.numel() > 1 else g.reshape(1, 1)
    s = bs.view(torch.float8_e4m3fn).float() * g
    return val * s.repeat_interleave(block, dim=1)


def swizzle_blockscale(scale: torch.Tensor) -> torch.Tensor:
    """The 128x4 block-scale layout the MoE runner expects (zero padded):
    [B, M, K] -> reshape [B, M/128, 4, 32, K/4, 4] -> permute (0, 1, 4, 3, 2, 5)."""
    two_d = scale.dim() == 2
    if two_d:
        scale = scale.unsqueeze(0)
    B, M, K = scale.shape
    Mp, Kp = (M + 127) // 128 * 128, (K + 3) // 4 * 4
    pad = torch.zeros((B, Mp, Kp), dtype=scale.dtype, device=scale.device)
    pad[:, :M, :K] = scale
    sw = pad.reshape(B, Mp // 128, 4, 32, Kp // 4, 4).permute(0, 1, 4, 3, 2, 5).contiguous()
    sw = sw.reshape(B, Mp, Kp)
    return sw[0] if two_d else sw
