"""Greedy (topk = 1) draft step on B200, with the hot-vocabulary token map.

Host mirrors of the reference's operator, computed by ``_fnx.so`` (csrc/topk1.cu and the
dense GEMV's argmax):

* ``draft_topk1_postprocess(next_token_logits, positions, draft_tokens=None,
  draft_token_column=0, hot_token_id=None)`` -- patches/sglang/series/0016-spec-remove-
  per-draft-step-glue-in-the-topk-1-chain-.patch:46-73 (python/sglang/kernels/ops/
  speculative/topk1.py): argmax of each row (lowest column on ties), mapped through
  ``hot_token_id`` to a full-vocabulary token, stored in ``topk_index`` and in
  ``draft_tokens[:, draft_token_column]``; ``topk_p`` = 1; ``positions`` += 1 in place.
* ``draft_head_topk1(x, w, scale, positions, ...)`` -- the draft head GEMV with that step
  fused into its argmax: one launch from hidden state to the next draft token.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import check, ptr
from .w8a16_gemv import (PDL, _activation, _cfg, _k_major, _out_or_new, _scale_kind, _stream,
                         _weight_kind, _workspace)


def _check_chain(B: int, V: int, device, positions, draft_tokens, draft_token_column,
                 hot_token_id):
    """The reference's asserts (0016-…patch, draft_topk1_postprocess)."""
    assert positions.is_contiguous()
    assert positions.shape[0] == B
    assert positions.device == device
    assert positions.dtype == torch.int64
    if hot_token_id is not None:
        assert hot_token_id.ndim == 1
        assert hot_token_id.dtype == torch.int64
        assert hot_token_id.is_contiguous()
        assert hot_token_id.device == device
        assert hot_token_id.shape[0] == V
    if draft_tokens is not None:
        assert draft_tokens.ndim == 2
        assert draft_tokens.dtype == torch.int64
        assert draft_tokens.device == device
        assert draft_tokens.shape[0] == B
        assert draft_tokens.stride(1) == 1
        assert 0 <= draft_token_column < draft_tokens.shape[1]


def draft_topk1_postprocess(
    next_token_logits: torch.Tensor,
    positions: torch.Tensor,
    draft_tokens: Optional[torch.Tensor] = None,
    draft_token_column: int = 0,
    hot_token_id: Optional[torch.Tensor] = None,
    pdl: Optional[bool] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Argmax draft logits for topk=1 and advance positions; returns (topk_p [B, 1] fp32,
    all 1.0, topk_index [B, 1] int64).  ``hot_token_id`` maps the argmax to a
    full-vocabulary token; ``draft_tokens[:, draft_token_column]`` receives it."""
    assert next_token_logits.ndim == 2
    assert next_token_logits.stride(1) == 1
    B, V = next_token_logits.shape
    if next_token_logits.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("next_token_logits must be fp32 or bf16")
    _check_chain(B, V, next_token_logits.device, positions, draft_tokens, draft_token_column,
                 hot_token_id)
    topk_p = torch.empty((B, 1), dtype=torch.float32, device=next_token_logits.device)
    topk_index = torch.empty((B, 1), dtype=torch.int64, device=next_token_logits.device)
    ws = _workspace(next_token_logits.device)
    rc = _lib.lib().fnx_draft_topk1(
        ptr(next_token_logits), next_token_logits.stride(0),
        int(next_token_logits.dtype == torch.float32), B, V, ptr(hot_token_id), ptr(positions),
        ptr(draft_tokens), 0 if draft_tokens is None else draft_tokens.stride(0),
        int(draft_token_column), ptr(topk_index), ptr(topk_p), ctypes.byref(ws.c),
        int(PDL if pdl is None else pdl), _stream(next_token_logits))
    check(rc, "draft_topk1_postprocess")
    return topk_p, topk_index


def draft_head_topk1(
    x: torch.Tensor,
    w: torch.Tensor,
    scale: torch.Tensor,
    positions: torch.Tensor,
    draft_tokens: Optional[torch.Tensor] = None,
    draft_token_column: int = 0,
    hot_token_id: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
    cfg=None,
    pdl: Optional[bool] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """The draft head ``w8a16_gemv(x, w, scale)`` and ``draft_topk1_postprocess`` on its
    bf16-rounded logits, in one launch.  ``out`` (bf16 or fp32 [M, N]) receives the
    logits.  Returns (topk_p [M, 1], topk_index [M, 1])."""
    M, K = x.shape
    N = w.shape[0]
    assert w.shape[1] == K and M <= 16
    _k_major(w, "draft_head_topk1")
    _check_chain(M, N, x.device, positions, draft_tokens, draft_token_column, hot_token_id)
    y = _out_or_new(out, M, N, x.device)
    x = _activation(x)
    s, skind = _scale_kind(scale, N)
    topk_p = torch.empty((M, 1), dtype=torch.float32, device=x.device)
    topk_index = torch.empty((M, 1), dtype=torch.int64, device=x.device)
    ws = _workspace(x.device)
    c = _cfg(cfg)
    rc = _lib.lib().fnx_draft_head_topk1(
        ptr(x), x.stride(0), ptr(w), w.stride(0) * w.element_size(), _weight_kind(w), ptr(s),
        skind, ptr(y), y.stride(0), int(y.dtype == torch.float32), M, N, K, ptr(hot_token_id),
        ptr(positions), ptr(draft_tokens), 0 if draft_tokens is None else draft_tokens.stride(0),
        int(draft_token_column), ptr(topk_index), ptr(topk_p),
        None if c is None else ctypes.byref(c), ctypes.byref(ws.c),
        int(PDL if pdl is None else pdl), _stream(x))
    check(rc, "draft_head_topk1")
    return topk_p, topk_index
