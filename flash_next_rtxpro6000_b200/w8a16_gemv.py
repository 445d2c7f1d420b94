"""W8A16 skinny GEMV for decode / verify widths (M <= 16), on the sm_100a library.

Host-side mirror of the reference operator module
``kernels/sglang/srt/layers/quantization/w8a16_gemv.py``: the same function names,
argument meaning, destination rules (``out=`` fp32 or bf16, two-destination
``out2=``/``split_n``), exceptions and per-device / per-slot scratch
(``prealloc``, ``scratch_slot``).  Every call goes to ``_fnx.so``; there is no torch or
CPU fallback.

Additions over the reference: int8 weights and bf16 scales are read natively (no
per-call fp32 copy of the scale, w8a16_gemv.py:660-662), and ``argmax_out=`` fuses the
greedy top-1 of the bf16-rounded logits (lowest row on ties) into the same launch.
"""

from __future__ import annotations

import logging
import os
from dataclasses import dataclass
from typing import Optional, Tuple, Union

import torch

from . import _lib, errors
from ._lib import FnxGemvCfg, FnxWorkspace, check, ptr

logger = logging.getLogger(__name__)

# Split-K scratch sizes (the reference's w8a16_gemv.py:329-331).
_WS_FLOATS = 1 << 21
_WS_COUNTERS = 4096
_N_SLOTS = 2
_SLOT = 0
_WS: dict = {}
_ONES: dict = {}


def _env_flag(name: str, default: str = "0") -> bool:
    return os.environ.get(name, default).lower() in ("1", "true", "yes", "on")


#: Programmatic dependent launch for the dense GEMVs (the reference's SGLANG_TRITON_PDL,
#: kernels/sglang/kernels/triton_pdl.py:40-52).  Off by default: with PDL the kernel
#: streams its weights before the previous kernel has finished, which is only correct
#: when no earlier kernel in the stream is still writing those weights.
PDL = _env_flag("FNX_PDL")


@dataclass(frozen=True)
class GemvConfig:
    """Launch geometry (see include/fnx_gemv.h fnx_gemv_cfg): `warps` consumer warps,
    each streaming `chunks_per_warp` 64-byte chunks of every row of one of `groups`
    16-row tiles per unit; `ksplit` k splits; `grid` CTAs (0 = one persistent wave)."""

    warps: int
    chunks_per_warp: int
    groups: int = 1
    ksplit: int = 1
    grid: int = 0

    def to_c(self) -> FnxGemvCfg:
        return FnxGemvCfg(self.warps, self.chunks_per_warp, self.groups, self.ksplit, self.grid)


class Workspace:
    """Split-K partials + counters and argmax keys of one (device, slot)."""

    def __init__(self, device: torch.device):
        self.device = device
        self.partials = torch.empty(_WS_FLOATS, dtype=torch.float32, device=device)
        self.counters = torch.zeros(_WS_COUNTERS, dtype=torch.int32, device=device)
        self.argmax_keys = torch.zeros(_lib.MAX_M, dtype=torch.int64, device=device)
        self.argmax_count = torch.zeros(1, dtype=torch.int32, device=device)
        self.error_flag = torch.zeros(1, dtype=torch.int32, device=device)
        errors.register(self.error_flag, f"dense GEMV scratch on {device}")
        self.c = FnxWorkspace(ptr(self.partials), _WS_FLOATS, ptr(self.counters), _WS_COUNTERS,
                              ptr(self.argmax_keys), ptr(self.argmax_count),
                              ptr(self.error_flag))


class scratch_slot:
    """Context manager selecting the scratch slot for launches inside it
    (w8a16_gemv.py:347-364): concurrent streams must use different slots."""

    def __init__(self, slot: int):
        assert 0 <= slot < _N_SLOTS
        self.slot = slot
        self.prev = 0

    def __enter__(self):
        global _SLOT
        self.prev = _SLOT
        _SLOT = self.slot
        return self

    def __exit__(self, *exc):
        global _SLOT
        _SLOT = self.prev
        return False


def _norm_device(device) -> torch.device:
    d = torch.device(device)
    if d.type == "cuda" and d.index is None:
        d = torch.device("cuda", torch.cuda.current_device())
    return d


def _workspace_slot(device, slot: int) -> Workspace:
    key = (_norm_device(device), slot)
    ws = _WS.get(key)
    if ws is None:
        ws = Workspace(key[0])
        _WS[key] = ws
    return ws


def _workspace(device) -> Workspace:
    return _workspace_slot(device, _SLOT)


def prealloc(device) -> None:
    """Materialise every slot's scratch before any CUDA graph is captured
    (w8a16_gemv.py:383-395)."""
    for slot in range(_N_SLOTS):
        _workspace_slot(device, slot)
    d = _norm_device(device)
    if d not in _ONES:
        _ONES[d] = torch.ones(1, dtype=torch.float32, device=d)
    _lib.lib()


def _stream(t: torch.Tensor) -> int:
    if t.device.index != torch.cuda.current_device():
        raise ValueError(
            f"tensor on {t.device} but the current device is cuda:{torch.cuda.current_device()}")
    return torch.cuda.current_stream(t.device).cuda_stream


def _out_or_new(out, M: int, N: int, device):
    """Validate an optional destination, else allocate the bf16 one (w8a16_gemv.py:599-618)."""
    if out is None:
        return torch.empty((M, N), dtype=torch.bfloat16, device=device)
    if (
        tuple(out.shape) != (M, N)
        or out.dtype not in (torch.bfloat16, torch.float32)
        or out.device != device
        or out.stride(1) != 1
    ):
        raise ValueError(
            f"w8a16 gemv out= must be a [{M}, {N}] row-contiguous bf16/fp32 CUDA "
            f"tensor on {device}; got {tuple(out.shape)} {out.dtype} {out.device}"
        )
    return out


def _split_dests(out, out2, split_n: int, M: int, N: int, device):
    """Two-destination column split (w8a16_gemv.py:621-639)."""
    if out2 is None:
        return _out_or_new(out, M, N, device), None, 0
    if not (0 < split_n < N):
        raise ValueError(f"w8a16 gemv split_n must be in (0, {N}); got {split_n}")
    y = _out_or_new(out, M, split_n, device)
    y2 = _out_or_new(out2, M, N - split_n, device)
    if y.dtype != y2.dtype or y.stride(1) != 1 or y2.stride(1) != 1:
        raise ValueError("w8a16 gemv out/out2 must share a dtype and be row-contiguous")
    return y, y2, split_n


def _activation(x: torch.Tensor) -> torch.Tensor:
    if x.dtype != torch.bfloat16:
        raise ValueError(f"activations must be bf16, got {x.dtype}")
    if x.stride(1) != 1 or (x.stride(0) * 2) % 16 or x.data_ptr() % 16:
        x = x.contiguous()
    return x


def _weight_kind(w: torch.Tensor) -> int:
    if w.dtype == torch.int8:
        return _lib.W_INT8
    if w.dtype == torch.float8_e4m3fn:
        return _lib.W_FP8_E4M3
    if w.dtype == torch.bfloat16:
        return _lib.W_BF16
    raise ValueError(f"unsupported weight dtype {w.dtype} (int8, float8_e4m3fn or bfloat16)")


def _scale_kind(s: torch.Tensor, N: int) -> Tuple[torch.Tensor, int]:
    s = s.reshape(-1)
    if s.dtype not in (torch.float32, torch.bfloat16):
        s = s.float()
    if not s.is_contiguous():
        s = s.contiguous()
    if s.numel() == 1:
        return s, _lib.SCALE_F32_SCALAR if s.dtype == torch.float32 else _lib.SCALE_BF16_SCALAR
    if s.numel() != N:
        raise ValueError(f"scale has {s.numel()} entries, expected 1 or {N}")
    return s, _lib.SCALE_F32_ROW if s.dtype == torch.float32 else _lib.SCALE_BF16_ROW


_REF_CFG_NOTED = [False]


def _cfg(cfg) -> Optional[FnxGemvCfg]:
    """Our geometry (GemvConfig or its 2..5-tuple); None = planner.

    The reference's own 7-tuple ``(BLOCK_N, BLOCK_K, SPLITS, use_dot, w_kn, warps,
    stages)`` (w8a16_gemv.py:522-538) describes a Triton tiling with no counterpart in
    this kernel; it is accepted and ignored (the planner chooses), noted once in the log.
    """
    if cfg is None:
        return None
    if isinstance(cfg, GemvConfig):
        return cfg.to_c()
    if isinstance(cfg, (tuple, list)) and len(cfg) == 7:
        if not _REF_CFG_NOTED[0]:
            logger.info("w8a16 gemv: ignoring the Triton tile config %r; this library plans "
                        "its own launch geometry", tuple(cfg))
            _REF_CFG_NOTED[0] = True
        return None
    if isinstance(cfg, (tuple, list)) and len(cfg) in (2, 3, 4, 5):
        return GemvConfig(*cfg).to_c()
    raise ValueError(f"cfg must be a GemvConfig, (warps, chunks_per_warp[, groups, ksplit, "
                     f"grid]) or the reference's 7-tuple; got {cfg!r}")


def _k_major(w: torch.Tensor, what: str) -> None:
    """The kernels stream K-contiguous weight rows.  An N-contiguous view (the reference's
    W_KN case, w8a16_gemv.py:586) is declined with NotImplementedError, like every other
    shape this library does not tile, so the caller keeps its own path."""
    if w.stride(1) != 1:
        raise NotImplementedError(
            f"{what}: only K-contiguous [N, K] weights (stride(1) == 1) are supported; got "
            f"strides {tuple(w.stride())}")


def _argmax_dest(argmax_out, M: int, device):
    if argmax_out is None:
        return None
    if (argmax_out.dtype != torch.int64 or argmax_out.numel() != M or
            not argmax_out.is_contiguous() or argmax_out.device != device):
        raise ValueError(f"argmax_out must be a contiguous int64 [{M}] tensor on {device}")
    return argmax_out


def w8a16_gemv(
    x: torch.Tensor,
    w: torch.Tensor,
    scale: torch.Tensor,
    cfg=None,
    out: Optional[torch.Tensor] = None,
    out2: Optional[torch.Tensor] = None,
    split_n: int = 0,
    argmax_out: Optional[torch.Tensor] = None,
    pdl: Optional[bool] = None,
) -> Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]]:
    """x: [M,K] bf16; w: [N,K] int8 / fp8_e4m3 / bf16 (K contiguous); scale: [N], [N,1]
    or scalar, fp32 or bf16.  Returns y [M, N] (or (y, y2) with ``out2``).

    ``argmax_out`` (int64 [M]) receives the greedy top-1 row of the bf16-rounded logits.
    """
    M, K = x.shape
    N = w.shape[0]
    assert w.shape[1] == K and M <= 16
    y, y2, split_n = _split_dests(out, out2, split_n, M, N, x.device)
    _k_major(w, "w8a16_gemv")
    x = _activation(x)
    s, skind = _scale_kind(scale, N)
    am = _argmax_dest(argmax_out, M, x.device)
    ws = _workspace(x.device)
    c = _cfg(cfg)
    rc = _lib.lib().fnx_w8a16_gemv(
        ptr(x), x.stride(0), ptr(w), w.stride(0) * w.element_size(), _weight_kind(w), ptr(s), skind,
        ptr(y), y.stride(0), ptr(y2), 0 if y2 is None else y2.stride(0), split_n,
        int(y.dtype == torch.float32), ptr(am), None, 0, M, N, K,
        None if c is None else ctypes_byref(c), ctypes_byref(ws.c), int(PDL if pdl is None else pdl),
        _stream(x))
    check(rc, "w8a16_gemv")
    return y if y2 is None else (y, y2)


def bf16_gemv(
    x: torch.Tensor,
    w: torch.Tensor,
    cfg=None,
    out: Optional[torch.Tensor] = None,
    out2: Optional[torch.Tensor] = None,
    split_n: int = 0,
):
    """Skinny bf16 GEMM y = x @ w^T (w8a16_gemv.py:826-847)."""
    if w.dtype != torch.bfloat16:
        raise ValueError("bf16_gemv needs a bf16 weight")
    d = _norm_device(x.device)
    one = _ONES.get(d)
    if one is None:
        one = torch.ones(1, dtype=torch.float32, device=d)
        _ONES[d] = one
    return w8a16_gemv(x, w, one, cfg=cfg, out=out, out2=out2, split_n=split_n)


def w8a16_gemv_silu_mul(x: torch.Tensor, w: torch.Tensor, scale: torch.Tensor, cfg=None,
                        out: Optional[torch.Tensor] = None,
                        pdl: Optional[bool] = None) -> torch.Tensor:
    """silu(x @ w[:H].T * s[:H]) * (x @ w[H:].T * s[H:]) in one launch
    (w8a16_gemv.py:1009-1061).  w: [2H, K], gate half first; scale per channel."""
    M, K = x.shape
    N = w.shape[0]
    assert w.shape[1] == K and M <= 16 and N % 2 == 0
    H = N // 2
    y = torch.empty((M, H), dtype=torch.bfloat16, device=x.device) if out is None else out
    if tuple(y.shape) != (M, H) or y.dtype != torch.bfloat16 or y.stride(1) != 1:
        raise ValueError(f"out= must be a row-contiguous bf16 [{M}, {H}] tensor")
    s, skind = _scale_kind(scale, N)
    assert s.numel() == N, "fused gate_up needs a per-channel scale"
    _k_major(w, "w8a16_gemv_silu_mul")
    x = _activation(x)
    ws = _workspace(x.device)
    c = _cfg(cfg)
    rc = _lib.lib().fnx_w8a16_gemv_silu_mul(
        ptr(x), x.stride(0), ptr(w), w.stride(0) * w.element_size(), _weight_kind(w), ptr(s), skind,
        ptr(y), y.stride(0), M, H, K, None if c is None else ctypes_byref(c), ctypes_byref(ws.c),
        int(PDL if pdl is None else pdl), _stream(x))
    check(rc, "w8a16_gemv_silu_mul")
    return y


def w8a16_gemv_silu_mul_supported(x: torch.Tensor, w: torch.Tensor, scale: torch.Tensor,
                                  max_m: int = 16) -> bool:
    """Whether this call can take the fused path (w8a16_gemv.py:1064-1079); int8 weights
    are accepted too."""
    return (
        x.is_cuda
        and x.dim() == 2
        and x.dtype == torch.bfloat16
        and 1 <= x.shape[0] <= max_m
        and w.dtype in (torch.float8_e4m3fn, torch.int8)
        and w.dim() == 2
        and w.shape[1] == x.shape[1]
        and w.shape[0] % 2 == 0
        and w.stride(1) == 1
        and scale.numel() == w.shape[0]
    )


#: The fused gated-RMSNorm prologue (the reference's SGLANG_NORM_INTO_GEMV switch,
#: w8a16_gemv.py:670-691, off by default there); on by default here.
NORM_INTO_GEMV = _env_flag("FNX_NORM_INTO_GEMV", "1")


def _norm_group_ok(G: int) -> bool:
    return 8 <= G <= 256 and (G & (G - 1)) == 0


def w8a16_gemv_norm_gated_supported(x: torch.Tensor, w: torch.Tensor, scale: torch.Tensor,
                                    z: torch.Tensor, norm_weight: torch.Tensor,
                                    group_size: int) -> bool:
    """Whether this call can take the fused gated-RMSNorm + GEMV path
    (w8a16_gemv.py:748-777); the group is also a power of two in [8, 256] here, the
    reference's BLOCK_K == group_size tiles."""
    K = x.shape[-1] if x.dim() == 2 else -1
    return bool(
        NORM_INTO_GEMV
        and x.is_cuda
        and x.dim() == 2
        and x.dtype == torch.bfloat16
        and z.dtype == torch.bfloat16
        and 1 <= x.shape[0] <= 16
        and tuple(z.shape) == tuple(x.shape)
        and x.stride(1) == 1
        and z.stride(1) == 1
        and group_size > 0
        and K % group_size == 0
        and _norm_group_ok(group_size)
        and norm_weight.dtype in (torch.bfloat16, torch.float32)
        and norm_weight.numel() == group_size
        and norm_weight.is_contiguous()
        and w.dim() == 2
        and w.dtype in (torch.int8, torch.float8_e4m3fn, torch.bfloat16)
        and w.shape[1] == K
        and w.stride(1) == 1
        and scale.numel() == w.shape[0]
    )


def w8a16_gemv_norm_gated(
    x: torch.Tensor,
    w: torch.Tensor,
    scale: torch.Tensor,
    z: torch.Tensor,
    norm_weight: torch.Tensor,
    group_size: int,
    eps: float,
    sigmoid_gate: bool = False,
    out: Optional[torch.Tensor] = None,
    cfg=None,
    pdl: Optional[bool] = None,
) -> torch.Tensor:
    """``(gated_rms_norm(x, z) @ w^T) * scale`` in one launch (w8a16_gemv.py:780-823).

    ``x``/``z`` are [M, K] bf16 with K a multiple of ``group_size``; each contiguous
    ``group_size`` slice of a row is its own RMS group (RMSNormGated(group_size,
    norm_before_gate=True) on the [M * K / group_size, group_size] reshape), the gate is
    z * sigmoid(z), or sigmoid(z) with ``sigmoid_gate``; the normalised row is rounded to
    bf16 before the dot.  ``norm_weight``: [group_size] bf16 or fp32, passed untouched.
    """
    M, K = x.shape
    N = w.shape[0]
    assert w.shape[1] == K and M <= 16
    if tuple(z.shape) != (M, K) or z.dtype != torch.bfloat16:
        raise ValueError(f"z must be a bf16 [{M}, {K}] tensor; got {tuple(z.shape)} {z.dtype}")
    if norm_weight.dtype not in (torch.bfloat16, torch.float32) or \
            norm_weight.numel() != group_size:
        raise ValueError(f"norm_weight must be a bf16/fp32 [{group_size}] vector")
    _k_major(w, "w8a16_gemv_norm_gated")
    y = _out_or_new(out, M, N, x.device)
    x = _activation(x)
    z = _activation(z)
    nw = norm_weight.reshape(-1)
    if not nw.is_contiguous() or nw.data_ptr() % 16:
        nw = nw.contiguous().clone()
    s, skind = _scale_kind(scale, N)
    ws = _workspace(x.device)
    c = _cfg(cfg)
    rc = _lib.lib().fnx_w8a16_gemv_norm_gated(
        ptr(x), x.stride(0), ptr(z), z.stride(0), ptr(nw), int(nw.dtype == torch.float32),
        int(group_size), float(eps), int(bool(sigmoid_gate)), ptr(w),
        w.stride(0) * w.element_size(), _weight_kind(w), ptr(s), skind, ptr(y), y.stride(0),
        int(y.dtype == torch.float32), M, N, K, None if c is None else ctypes_byref(c),
        ctypes_byref(ws.c), int(PDL if pdl is None else pdl), _stream(x))
    check(rc, "w8a16_gemv_norm_gated")
    return y


_DENSE_PATHS = {"auto": 0, "mma": 1, "tcgen05": 2}


def set_dense_path(path: str) -> str:
    """Select the contraction of the dense GEMV calls made without ``cfg`` (process-wide):
    ``"auto"`` (tcgen05 tensor cores for int8 / fp8 weights at M > 8, mma.sync otherwise),
    ``"mma"`` or ``"tcgen05"`` (wherever it applies, at every M).  Returns the previous
    setting."""
    if path not in _DENSE_PATHS:
        raise ValueError(f"dense path must be one of {sorted(_DENSE_PATHS)}, got {path!r}")
    import ctypes

    prev = ctypes.c_int(0)
    check(_lib.lib().fnx_set_dense_path(_DENSE_PATHS[path], ctypes.byref(prev)), "set_dense_path")
    return {v: k for k, v in _DENSE_PATHS.items()}[prev.value]


class dense_path:
    """Context manager running the calls inside it with ``set_dense_path(path)``."""

    def __init__(self, path: str):
        self.path = path
        self.prev = "auto"

    def __enter__(self):
        self.prev = set_dense_path(self.path)
        return self

    def __exit__(self, *exc):
        set_dense_path(self.prev)
        return False


def plan(M: int, N: int, K: int, w_dtype: torch.dtype, fused_silu: bool = False) -> GemvConfig:
    """The geometry the library's planner picks for a call."""
    c = FnxGemvCfg()
    kind = {torch.int8: _lib.W_INT8, torch.float8_e4m3fn: _lib.W_FP8_E4M3,
            torch.bfloat16: _lib.W_BF16, torch.uint8: _lib.W_NVFP4}[w_dtype]
    check(_lib.lib().fnx_plan_gemv(M, N, K, kind, int(fused_silu), 0, ctypes_byref(c)), "plan")
    return GemvConfig(c.warps, c.chunks_per_warp, c.groups, c.ksplit, c.grid)


def ctypes_byref(obj):
    import ctypes

    return ctypes.byref(obj)
