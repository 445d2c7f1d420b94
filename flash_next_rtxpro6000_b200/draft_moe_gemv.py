"""Routed NVFP4 MoE GEMV for decode and verify widths (M <= 16), on the sm_100a library.

Host-side mirror of the reference's ``python/sglang/srt/layers/moe/draft_moe_gemv.py``
(added by patches/sglang/series/0112-DG1-one-token-draft-MoE-as-a-W4A16-NVFP4-Triton-
GEMV.patch): ``draft_moe_gemv``, ``make_workspace``, ``unsupported_reason``,
``DraftMoeGemvRunner.maybe_apply`` and ``enable_draft_moe_gemv`` keep their names,
keyword arguments and decline-by-returning-None behaviour.  What changes:

* one launch pair serves M = 1..16 tokens (the reference handles only M = 1 and leaves
  M >= 2 to FlashInfer's CUTLASS W4A4 chain); each distinct expert is streamed once for
  all tokens routed to it, with bf16 activations (W4A16);
* an optional always-on shared expert in the same NVFP4 format joins the route sum with
  weight 1.0;
* ``out_f32`` returns the fp32 partial sum of one expert slice for a cross-rank SUM.
"""

from __future__ import annotations

import ctypes
import logging
from dataclasses import dataclass
from types import SimpleNamespace
from typing import Optional

import torch

from . import _lib, errors
from ._lib import FnxMoeWeights, FnxMoeWorkspace, FnxMoeWorkspaceSizes, check, ptr
from .w8a16_gemv import _activation, _stream

logger = logging.getLogger(__name__)

_SF_TILE_ROWS = 128
_SF_COL_GROUP = 4
_FP4_BLOCK = 16


@dataclass(frozen=True)
class DraftMoeGemvConfig:
    """Launch options.  The tiling itself is fixed by (H, I) inside the library."""

    pdl: bool = False          # let k1 overlap the previous kernel's tail
    max_tokens: int = 16       # workspace capacity


DEFAULT_CONFIG = DraftMoeGemvConfig()


@dataclass(frozen=True)
class DraftMoeWorkspace:
    """Scratch of one MoE layer call.  Every buffer is fully rewritten before it is read
    within a call, so nothing is cleared per call or graph replay."""

    act: torch.Tensor              # uint8 rows of 2I + 64 B: bf16 act in the down
                                   # projection's B-operand order, one row per route slot
    partials: torch.Tensor         # [P, H] fp32 route partials of the down projection
    error_flag: torch.Tensor       # [1] int32 device error code (0 = none)
    max_tokens: int
    num_routes: int
    counters: Optional[torch.Tensor] = None  # int32, zero between calls: the one-launch form

    def to_c(self) -> FnxMoeWorkspace:
        n = 0 if self.counters is None else self.counters.numel()
        return FnxMoeWorkspace(ptr(self.act), ptr(self.partials), ptr(self.error_flag),
                               self.max_tokens, self.num_routes, ptr(self.counters), n)


@dataclass
class SharedExpert:
    """An always-on expert in the routed experts' NVFP4 format (weight 1.0)."""

    w13_weight: torch.Tensor               # [1, 2I, H/2] or [2I, H/2]
    w13_blockscale_swizzled: torch.Tensor  # [1, 2I, H/16] (or linear, see scales_swizzled)
    w13_weight_scale_2: torch.Tensor       # fp32 scalar (or [1, 2] / [1])
    w2_weight: torch.Tensor                # [1, H, I/2]
    w2_blockscale_swizzled: torch.Tensor
    w2_weight_scale_2: torch.Tensor


def unsupported_reason(*, hidden_size: int, intermediate_size: int,
                       cfg: DraftMoeGemvConfig = DEFAULT_CONFIG, num_routes: int = 10,
                       num_experts: int = 512) -> Optional[str]:
    """Why these shapes cannot take the GEMV, or None (0112-...patch:289-304).

    The structural checks below are the library's; the last one asks the library
    whether both kernels fit in shared memory at ``cfg.max_tokens`` tokens."""
    if hidden_size % _SF_TILE_ROWS or intermediate_size % _SF_TILE_ROWS:
        return "H and I must be multiples of 128 (no swizzle padding)"
    if (hidden_size // _FP4_BLOCK) % _SF_COL_GROUP or (intermediate_size // _FP4_BLOCK) % _SF_COL_GROUP:
        return "H/16 and I/16 must be multiples of 4 (no swizzle padding)"
    ch1, ch2 = hidden_size // 128, intermediate_size // 128
    # gate/up: the consumer warps split H into ch1 chunks of 128 (4..11 warps x 1..4 chunks)
    if not any(ch1 % c == 0 and 4 <= ch1 // c <= 11 for c in (1, 2, 4)):
        return f"H={hidden_size}: no gate/up tiling (H/128 must be 4..11 warps x 1, 2 or 4 chunks)"
    # down: rt row tiles (4, 2 or 1 quadrants of a 128-row block) x (ch2 / c) k slices
    # <= 16 warps
    if not any(ch2 % c == 0 and rt * (ch2 // c) <= 16 for rt in (1, 2, 4) for c in (1, 2, 4)):
        return f"I={intermediate_size}: no down tiling (I/128 must split into <= 16 slices)"
    if cfg.max_tokens < 1 or cfg.max_tokens > _lib.MAX_M:
        return "max_tokens must be in [1, 16]"
    sz = FnxMoeWorkspaceSizes()
    if _lib.lib().fnx_moe_workspace_bytes(cfg.max_tokens, num_routes, num_experts, hidden_size,
                                          intermediate_size, ctypes.byref(sz)) != _lib.FNX_OK:
        return _lib.last_error()
    return None


def make_workspace(*, num_routes: int, hidden_size: int, intermediate_size: int,
                   device: torch.device, cfg: DraftMoeGemvConfig = DEFAULT_CONFIG,
                   max_tokens: Optional[int] = None,
                   num_experts: int = 4096, fused: bool = True) -> DraftMoeWorkspace:
    """Scratch of one MoE layer call (0112-...patch:307-325), sized for max_tokens.

    ``fused`` (default) adds the counters of the one-launch layer; without them the layer
    runs as three launches (gate/up, down, route sum)."""
    m = cfg.max_tokens if max_tokens is None else max_tokens
    sz = FnxMoeWorkspaceSizes()
    check(_lib.lib().fnx_moe_workspace_bytes(m, num_routes, num_experts, hidden_size,
                                             intermediate_size, ctypes.byref(sz)),
          "make_workspace")
    pairs = m * (num_routes + 1)
    u8 = dict(dtype=torch.uint8, device=device)
    ws = DraftMoeWorkspace(
        act=torch.empty(sz.act, **u8),
        partials=torch.empty((pairs, hidden_size), dtype=torch.float32, device=device),
        error_flag=torch.zeros(1, dtype=torch.int32, device=device),
        max_tokens=m, num_routes=num_routes,
        counters=torch.zeros(sz.counters, dtype=torch.int32, device=device) if fused else None,
    )
    errors.register(ws.error_flag, f"MoE workspace ({m} tokens x {num_routes} routes) on {device}")
    return ws


def _u8(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.uint8) if t.dtype != torch.uint8 else t


def _expert_bank(w13, s13, g13, w2, s2, g2, hidden: int, inter: int, swizzled: bool,
                 expert_offset: int = 0) -> FnxMoeWeights:
    E = w13.shape[0] if w13.dim() == 3 else 1
    g13 = g13 if g13.dtype == torch.float32 else g13.float()
    g2 = g2 if g2.dtype == torch.float32 else g2.float()
    g13_stride = g13.stride(0) if g13.dim() >= 1 and g13.numel() > 1 else 0
    g2_stride = g2.stride(0) if g2.dim() >= 1 and g2.numel() > 1 else 0
    for t in (w13, s13, w2, s2):
        if not t.is_contiguous():
            raise ValueError("expert weights and scales must be contiguous")
    return FnxMoeWeights(ptr(w13), ptr(s13), ptr(g13), g13_stride, ptr(w2), ptr(s2), ptr(g2),
                         g2_stride, E, expert_offset, hidden, inter, int(swizzled))


def draft_moe_gemv(
    *,
    hidden_states: torch.Tensor,
    topk_ids: torch.Tensor,
    topk_weights: torch.Tensor,
    w13_weight: torch.Tensor,
    w13_blockscale_swizzled: torch.Tensor,
    w13_weight_scale_2: torch.Tensor,
    w2_weight: torch.Tensor,
    w2_blockscale_swizzled: torch.Tensor,
    w2_weight_scale_2: torch.Tensor,
    workspace: DraftMoeWorkspace,
    cfg: DraftMoeGemvConfig = DEFAULT_CONFIG,
    shared_expert: Optional[SharedExpert] = None,
    scales_swizzled: bool = True,
    expert_offset: int = 0,
    out: Optional[torch.Tensor] = None,
    out_f32: bool = False,
) -> torch.Tensor:
    """MoE layer: hidden_states [M, H] bf16 (M <= 16), topk_* [M, R] -> [M, H] bf16.

    ``expert_offset``: global id of the first expert held by w13/w2 (expert-parallel
    shards); routes to experts outside the slice are skipped.  ``out_f32`` returns the
    fp32 partial sum of this slice instead of the bf16 result.
    """
    x = _activation(hidden_states)
    M, H = x.shape
    inter = w13_weight.shape[1] // 2
    hidden = w13_weight.shape[2] * 2
    if hidden != H:
        raise ValueError(f"hidden_states width {H} != expert hidden size {hidden}")
    R = topk_ids.shape[1]
    if M > workspace.max_tokens or R > workspace.num_routes:
        raise ValueError("workspace too small for this call")
    ids = topk_ids if topk_ids.dtype == torch.int32 else topk_ids.to(torch.int32)
    wts = topk_weights if topk_weights.dtype == torch.float32 else topk_weights.float()
    ids, wts = ids.contiguous(), wts.contiguous()
    bank = _expert_bank(_u8(w13_weight), _u8(w13_blockscale_swizzled), w13_weight_scale_2,
                        _u8(w2_weight), _u8(w2_blockscale_swizzled), w2_weight_scale_2,
                        hidden, inter, scales_swizzled, expert_offset)
    sh = None
    if shared_expert is not None:
        se = shared_expert
        sh = _expert_bank(_u8(se.w13_weight), _u8(se.w13_blockscale_swizzled),
                          se.w13_weight_scale_2.reshape(-1)[:1], _u8(se.w2_weight),
                          _u8(se.w2_blockscale_swizzled), se.w2_weight_scale_2.reshape(-1)[:1],
                          hidden, inter, scales_swizzled)
    if out is None:
        out = torch.empty((M, H), dtype=torch.float32 if out_f32 else torch.bfloat16,
                          device=x.device)
    elif (tuple(out.shape) != (M, H) or out.stride(1) != 1 or
          out.dtype != (torch.float32 if out_f32 else torch.bfloat16)):
        raise ValueError("out= has the wrong shape, dtype or layout")
    wsc = workspace.to_c()
    rc = _lib.lib().fnx_moe_gemv(
        ptr(x), x.stride(0), ptr(ids), ptr(wts), M, R, ctypes.byref(bank),
        None if sh is None else ctypes.byref(sh), ptr(out), out.stride(0), int(out_f32),
        ctypes.byref(wsc), int(cfg.pdl), _stream(x))
    check(rc, "draft_moe_gemv")
    return out


#: The M <= 16 entry point under a width-neutral name.
moe_gemv = draft_moe_gemv


_FUSED_TILINGS = ((2048, 512), (2560, 640), (1024, 256), (2048, 1024))  # (H, I)


def fused_tiling(hidden_size: int, intermediate_size: int) -> bool:
    """Whether the one-launch layer is compiled for this (H, I)."""
    return (hidden_size, intermediate_size) in _FUSED_TILINGS


_MOE_PATHS = {"auto": 0, "fused": 1}


def set_moe_path(path: str) -> str:
    """Select the one-launch MoE layer (process-wide): ``"auto"`` (the decode-width
    kernel for M = 1 with swizzled scales, the general one-launch kernel otherwise) or
    ``"fused"`` (the general one-launch kernel at every M).  Returns the previous
    setting."""
    if path not in _MOE_PATHS:
        raise ValueError(f"MoE path must be one of {sorted(_MOE_PATHS)}, got {path!r}")
    prev = ctypes.c_int(0)
    check(_lib.lib().fnx_set_moe_path(_MOE_PATHS[path], ctypes.byref(prev)), "set_moe_path")
    return {v: k for k, v in _MOE_PATHS.items()}[prev.value]


class moe_path:
    """Context manager running the calls inside it with ``set_moe_path(path)``."""

    def __init__(self, path: str):
        self.path = path
        self.prev = "auto"

    def __enter__(self):
        self.prev = set_moe_path(self.path)
        return self

    def __exit__(self, *exc):
        set_moe_path(self.prev)
        return False


_FORMS = {0: "three", 1: "fused", 2: "lean"}


def moe_plan(num_tokens: int, top_k: int, num_experts: int, hidden_size: int,
             intermediate_size: int) -> dict:
    """The form a call with a fused workspace and swizzled scales takes
    (``fnx_plan_moe``): ``form`` ("lean": the decode-width one-launch layer, "fused": the
    general one-launch layer, "three": three launches), ``fused`` (one launch) and, for a
    one-launch layer, its weight-ring ``stages``, consumer ``groups`` and dynamic shared
    memory ``smem_bytes``."""
    f, ns, ng = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    sm = ctypes.c_int64()
    check(_lib.lib().fnx_plan_moe(num_tokens, top_k, num_experts, hidden_size, intermediate_size,
                                  ctypes.byref(f), ctypes.byref(ns), ctypes.byref(ng),
                                  ctypes.byref(sm)), "fnx_plan_moe")
    return {"form": _FORMS[f.value], "fused": f.value > 0, "stages": ns.value,
            "groups": ng.value, "smem_bytes": sm.value}


def _form(hidden_size, intermediate_size, fused, num_tokens, top_k, num_experts) -> str:
    if not fused:
        return "three"
    if num_tokens is None:
        return "fused" if fused_tiling(hidden_size, intermediate_size) else "three"
    form = moe_plan(num_tokens, top_k, num_experts, hidden_size, intermediate_size)["form"]
    if form == "fused" and not fused_tiling(hidden_size, intermediate_size):
        return "three"
    return form


def _one_launch(hidden_size, intermediate_size, fused, num_tokens, top_k, num_experts) -> bool:
    return _form(hidden_size, intermediate_size, fused, num_tokens, top_k, num_experts) != "three"


def moe_launches_per_call(hidden_size: int, intermediate_size: int, fused: bool = True,
                          num_tokens: Optional[int] = None, top_k: int = 10,
                          num_experts: int = 512) -> int:
    """Kernel launches of one draft_moe_gemv call with a workspace made with ``fused``
    (for ``num_tokens`` tokens when given: the one-launch layer needs its shared memory
    to fit, else the call takes the three-launch form)."""
    one = _one_launch(hidden_size, intermediate_size, fused, num_tokens, top_k, num_experts)
    return 1 if one else 3


def moe_kernel_name(hidden_size: int, intermediate_size: int, fused: bool = True,
                    num_tokens: Optional[int] = None, top_k: int = 10,
                    num_experts: int = 512) -> str:
    """The kernel(s) one draft_moe_gemv call (swizzled scales) runs."""
    form = _form(hidden_size, intermediate_size, fused, num_tokens, top_k, num_experts)
    if form == "lean":
        return "moe_lean_kernel"
    if form == "fused":
        return "moe_fused_kernel"
    return "moe_up_kernel + moe_down_kernel + moe_sum_kernel"


def _is_small_batch_call(dispatch_output, max_tokens: int = 16) -> bool:
    x = dispatch_output.hidden_states
    topk_output = dispatch_output.topk_output
    return (
        1 <= x.shape[0] <= max_tokens
        and x.dtype == torch.bfloat16
        and x.is_contiguous()
        and getattr(dispatch_output, "hidden_states_scale", None) is None
        and topk_output.topk_ids.is_contiguous()
        and topk_output.topk_weights.is_contiguous()
    )


class DraftMoeGemvRunner:
    """The small-batch path of one MoE layer; owns that layer's scratch
    (0112-...patch:402-461).  maybe_apply returns None to keep the caller's fallback."""

    def __init__(self, cfg: DraftMoeGemvConfig = DEFAULT_CONFIG,
                 shared_expert: Optional[SharedExpert] = None) -> None:
        self._cfg = cfg
        self._workspace: Optional[DraftMoeWorkspace] = None
        self._warned_capture = False
        self.shared_expert = shared_expert

    def maybe_apply(self, *, layer, dispatch_output):
        if not _is_small_batch_call(dispatch_output, self._cfg.max_tokens):
            return None
        workspace = self._get_workspace(layer=layer, dispatch_output=dispatch_output)
        if workspace is None:
            return None
        topk_output = dispatch_output.topk_output
        if topk_output.topk_ids.shape[1] > workspace.num_routes:
            return None
        out = draft_moe_gemv(
            hidden_states=dispatch_output.hidden_states,
            topk_ids=topk_output.topk_ids,
            topk_weights=topk_output.topk_weights,
            w13_weight=layer.w13_weight,
            w13_blockscale_swizzled=layer.w13_blockscale_swizzled,
            w13_weight_scale_2=layer.w13_weight_scale_2,
            w2_weight=layer.w2_weight,
            w2_blockscale_swizzled=layer.w2_blockscale_swizzled,
            w2_weight_scale_2=layer.w2_weight_scale_2,
            workspace=workspace,
            cfg=self._cfg,
            shared_expert=self.shared_expert,
        )
        return SimpleNamespace(hidden_states=out)

    def _get_workspace(self, *, layer, dispatch_output) -> Optional[DraftMoeWorkspace]:
        if self._workspace is not None:
            return self._workspace
        # Allocating inside a capture would put the scratch in the graph's private pool.
        if torch.cuda.is_current_stream_capturing():
            if not self._warned_capture:
                logger.warning("MoE GEMV: first call is inside a CUDA graph capture; layer %s "
                               "keeps its fallback for this graph", getattr(layer, "layer_id", "?"))
                self._warned_capture = True
            return None
        self._workspace = make_workspace(
            num_routes=dispatch_output.topk_output.topk_ids.shape[1],
            hidden_size=layer.w13_weight.shape[2] * 2,
            intermediate_size=layer.w13_weight.shape[1] // 2,
            device=dispatch_output.hidden_states.device,
            cfg=self._cfg,
        )
        return self._workspace


def _layer_unsupported_reason(experts) -> Optional[str]:
    rc = getattr(experts, "moe_runner_config", None)
    if getattr(experts, "moe_ep_size", 1) != 1 or getattr(experts, "moe_tp_size", 1) != 1:
        return "needs moe_ep_size == moe_tp_size == 1"
    if rc is not None:
        if not (getattr(rc, "activation", "silu") == "silu" and getattr(rc, "is_gated", True)):
            return "needs gated silu"
        if (getattr(rc, "apply_router_weight_on_input", False)
                or getattr(rc, "gemm1_alpha", None) is not None
                or getattr(rc, "gemm1_beta", None) is not None
                or getattr(rc, "gemm1_clamp_limit", None) is not None
                or getattr(rc, "swiglu_limit", None) is not None):
            return "needs plain silu(gate) * up with router weights on the output"
    return unsupported_reason(hidden_size=experts.w13_weight.shape[2] * 2,
                              intermediate_size=experts.w13_weight.shape[1] // 2)


def enable_draft_moe_gemv(experts, shared_expert: Optional[SharedExpert] = None) -> bool:
    """Attach a runner to one NVFP4 MoE layer's quant method (0112-...patch:484-512)."""
    qm = getattr(experts, "quant_method", None)
    if qm is None or not hasattr(experts, "w13_weight"):
        return False
    reason = _layer_unsupported_reason(experts)
    if reason is not None:
        logger.warning("MoE GEMV not enabled for layer %s: %s",
                       getattr(experts, "layer_id", "?"), reason)
        return False
    qm.draft_moe_gemv = DraftMoeGemvRunner(shared_expert=shared_expert)
    return True
