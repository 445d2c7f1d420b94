"""W4A16 NVFP4 skinny GEMV (M <= 16) and the NVFP4 codec, on the sm_100a library.

Host-side mirror of ``kernels/sglang/srt/layers/quantization/w4a16_nvfp4_gemv.py``:

    W[n, k] = e2m1(code[n, k]) * e4m3(bs[n, k // 16]) * gscale

``wq[N, K/2]`` uint8 holds two codes per byte, low nibble = even k; ``bs[N, K/16]`` holds
e4m3 bit patterns (uint8 or float8_e4m3fn); ``gscale`` is the plain fp32 global scale,
scalar or ``[N]``.  The kernel decodes e2m1 natively (``cvt.rn.f16x2.e2m1x2``), so no
2^14 factor appears anywhere.

``quantize_nvfp4`` / ``dequantize_nvfp4`` are the load-time codec (ModelOpt convention,
w4a16_nvfp4_gemv.py:426-510), run by the library's codec kernels on the GPU; they are not
on the decode path.
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


_SCRATCH: dict = {}


def quantize_nvfp4(w: torch.Tensor, block: int = FP4_SCALE_BLOCK):
    """[N, K] bf16 / fp32 CUDA weight -> (wq [N, K//2] uint8, bs [N, K//16] uint8 e4m3 bits,
    gscale fp32 [1]), computed by the library's codec kernels on the weight's device.

    The ModelOpt convention (w4a16_nvfp4_gemv.py:426-472): gscale = max|W| / (448 * 6);
    each 16-block's scale amax_b / 6 / gscale rounded to e4m3; codes = W / (e4m3 scale *
    gscale) rounded to e2m1 with ties to even.  The codes equal the reference's bit for bit.
    """
    if block != FP4_SCALE_BLOCK:
        raise NotImplementedError("NVFP4 blocks are 16 values")
    if not w.is_cuda:
        raise NotImplementedError("quantize_nvfp4 runs on the GPU; move the weight to CUDA first")
    assert w.dim() == 2 and w.shape[1] % block == 0
    if w.dtype not in (torch.bfloat16, torch.float32):
        w = w.float()
    if w.stride(1) != 1:
        w = w.contiguous()
    N, K = w.shape
    wq = torch.empty((N, K // 2), dtype=torch.uint8, device=w.device)
    bs = torch.empty((N, K // block), dtype=torch.uint8, device=w.device)
    gscale = torch.empty(1, dtype=torch.float32, device=w.device)
    scratch = _SCRATCH.get(w.device)
    if scratch is None:
        scratch = torch.zeros(1, dtype=torch.int32, device=w.device)
        _SCRATCH[w.device] = scratch
    with torch.cuda.device(w.device):
        rc = _lib.lib().fnx_nvfp4_quantize(
            ptr(w), w.stride(0), int(w.dtype == torch.float32), N, K, ptr(wq), wq.stride(0),
            ptr(bs), bs.stride(0), ptr(gscale), ptr(scratch),
            torch.cuda.current_stream(w.device).cuda_stream)
    check(rc, "quantize_nvfp4")
    return wq, bs, gscale


def dequantize_nvfp4(wq: torch.Tensor, bs: torch.Tensor, gscale: torch.Tensor,
                     block: int = FP4_SCALE_BLOCK, dtype: torch.dtype = torch.float32,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """[N, K] weight (fp32 by default, or bf16) from CUDA NVFP4 tensors, by the library's
    codec kernel: e2m1(code) * (e4m3(bs) * gscale), gscale scalar or [N]
    (w4a16_nvfp4_gemv.py:489-510).  No host synchronisation (graph-capture safe)."""
    if block != FP4_SCALE_BLOCK:
        raise NotImplementedError("NVFP4 blocks are 16 values")
    if not wq.is_cuda:
        raise NotImplementedError("dequantize_nvfp4 runs on the GPU")
    N, KH = wq.shape
    K = KH * 2
    if dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("dtype must be float32 or bfloat16")
    bs = bs.view(torch.uint8) if bs.dtype != torch.uint8 else bs
    g = gscale.reshape(-1)
    if g.dtype != torch.float32 or not g.is_contiguous():
        g = g.float().contiguous()
    if g.numel() not in (1, N):
        raise ValueError(f"gscale must be a scalar or [{N}]")
    if wq.stride(1) != 1 or wq.stride(0) % 8 or wq.data_ptr() % 8:
        wq = wq.contiguous()
    if bs.stride(1) != 1:
        bs = bs.contiguous()
    y = torch.empty((N, K), dtype=dtype, device=wq.device) if out is None else out
    if tuple(y.shape) != (N, K) or y.dtype != dtype or y.stride(1) != 1:
        raise ValueError(f"out must be a row-contiguous {dtype} [{N}, {K}] tensor")
    with torch.cuda.device(wq.device):
        rc = _lib.lib().fnx_nvfp4_dequantize(
            ptr(wq), wq.stride(0), ptr(bs), bs.stride(0), ptr(g), int(g.numel() > 1), ptr(y),
            y.stride(0), int(dtype == torch.float32), N, K,
            torch.cuda.current_stream(wq.device).cuda_stream)
    check(rc, "dequantize_nvfp4")
    return y


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
