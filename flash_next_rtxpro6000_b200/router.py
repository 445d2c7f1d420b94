"""MoE router on B200: the logits projection and the softmax top-k routing table.

Host mirrors of the reference's operators, computed by ``_fnx.so`` (csrc/router.cu):

* ``router_gemv(x, weight, bias=None)`` -- kernels/sglang/srt/layers/moe/router_gemv.py:
  49-93: ``x @ weight.T + bias`` into fp32 logits, M <= 16, same checks and errors;
* ``covered`` / ``route_softmax_fast`` -- the packed-key softmax top-k router of
  patches/sglang/series/0110-…patch and 0111-…patch
  (python/sglang/kernels/ops/moe/moe_router_softmax_fast.py): same arguments and
  results (ids exact; weights to fp32 rounding), fp32 logits accepted too;
* ``router_topk(x, weight, bias, topk, renormalize)`` -- both in one launch: the last CTA
  of the projection computes the routing table, so the MoE prologue loses a launch.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import check, ptr
from .w8a16_gemv import PDL, _stream, _workspace


def _check_router_args(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor]):
    """The reference's validation (router_gemv.py:54-80), in its order."""
    if x.dim() != 2 or weight.dim() != 2:
        raise ValueError("x and weight must be 2-D")
    m, k = x.shape
    n, weight_k = weight.shape
    if not 1 <= m <= 16:
        raise ValueError("router GEMV requires 1 <= M <= 16")
    if k != weight_k or k % 128 != 0 or n % 32 != 0:
        raise ValueError("router GEMV requires matching K % 128 == 0 and N % 32 == 0")
    tensors = (x, weight) if bias is None else (x, weight, bias)
    if any(not t.is_cuda for t in tensors):
        raise ValueError("router GEMV requires CUDA tensors")
    if any(t.device != x.device for t in tensors):
        raise ValueError("all router GEMV tensors must be on the same device")
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise ValueError("router GEMV supports BF16 inputs and weights only")
    if not x.is_contiguous() or not weight.is_contiguous():
        raise ValueError("router GEMV inputs and weights must be contiguous")
    if bias is not None:
        if bias.shape != (n,) or bias.dtype != torch.bfloat16:
            raise ValueError("router GEMV bias must be contiguous BF16 with shape [N]")
        if not bias.is_contiguous():
            raise ValueError("router GEMV bias must be contiguous")
    return m, n, k


def _launch_router(x, weight, bias, logits, out_w, out_i, topk, renormalize, pdl):
    m, k = x.shape
    n = weight.shape[0]
    ws = _workspace(x.device)
    rc = _lib.lib().fnx_router_gemv_topk(
        ptr(x), x.stride(0), ptr(weight), weight.stride(0), ptr(bias), ptr(logits),
        0 if logits is None else logits.stride(0), ptr(out_w), ptr(out_i),
        0 if out_w is None else out_w.stride(0), m, n, k, topk, int(bool(renormalize)),
        ctypes.byref(ws.c), int(PDL if pdl is None else pdl), _stream(x))
    check(rc, "router_gemv")


def router_gemv(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
                pdl: Optional[bool] = None) -> torch.Tensor:
    """Compute ``x @ weight.T + bias`` into an FP32 router-logit tensor."""
    m, n, _ = _check_router_args(x, weight, bias)
    out = torch.empty((m, n), dtype=torch.float32, device=x.device)
    _launch_router(x, weight, bias, out, None, None, 0, False, pdl)
    return out


def covered(scores: torch.Tensor, bias: torch.Tensor, topk: int) -> bool:
    """bf16 logits, fp32 bias, at most 512 experts (the reference's predicate, 0111);
    topk is also limited to 32 here."""
    return (
        scores.dim() == 2
        and scores.dtype == torch.bfloat16
        and bias.dim() == 1
        and bias.dtype == torch.float32
        and scores.size(1) == bias.size(0)
        and scores.size(1) <= 512
        and 0 < int(topk) <= min(scores.size(1), 32)
    )


def route_softmax_fast(scores: torch.Tensor, zero_bias: Optional[torch.Tensor], topk: int,
                       renormalize: bool, pdl: Optional[bool] = None
                       ) -> Tuple[torch.Tensor, torch.Tensor]:
    """(topk_weights fp32 [M, topk], topk_ids int32 [M, topk]) of bf16 (or fp32) logits;
    the caller checks covered() (fp32 scores are accepted here as well)."""
    if scores.dtype not in (torch.bfloat16, torch.float32) or scores.stride(1) != 1:
        raise ValueError("scores must be row-contiguous bf16 or fp32")
    M, N = scores.shape
    weights = torch.empty((M, topk), dtype=torch.float32, device=scores.device)
    indices = torch.empty((M, topk), dtype=torch.int32, device=scores.device)
    b = zero_bias
    if b is not None and (b.dtype != torch.float32 or not b.is_contiguous()):
        b = b.float().contiguous()
    rc = _lib.lib().fnx_softmax_topk(
        ptr(scores), scores.stride(0), int(scores.dtype == torch.float32), ptr(b),
        ptr(weights), ptr(indices), weights.stride(0), M, N, int(topk),
        int(bool(renormalize)), int(PDL if pdl is None else pdl), _stream(scores))
    check(rc, "route_softmax_fast")
    return weights, indices


def router_topk(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
                topk: int = 10, renormalize: bool = True,
                logits_out: Optional[torch.Tensor] = None, pdl: Optional[bool] = None
                ) -> Tuple[torch.Tensor, torch.Tensor]:
    """router_gemv followed by the softmax top-k, in one launch: returns (topk_weights
    fp32 [M, topk], topk_ids int32 [M, topk]), the routing table ``draft_moe_gemv``
    reads.  ``logits_out`` (fp32 [M, N]) also receives the logits."""
    m, n, _ = _check_router_args(x, weight, bias)
    if logits_out is not None and (tuple(logits_out.shape) != (m, n) or
                                   logits_out.dtype != torch.float32 or
                                   logits_out.stride(1) != 1):
        raise ValueError(f"logits_out must be a row-contiguous fp32 [{m}, {n}] tensor")
    weights = torch.empty((m, topk), dtype=torch.float32, device=x.device)
    ids = torch.empty((m, topk), dtype=torch.int32, device=x.device)
    _launch_router(x, weight, bias, logits_out, weights, ids, int(topk), renormalize, pdl)
    return weights, ids
