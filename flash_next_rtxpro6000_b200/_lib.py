"""ctypes binding of the C ABI in include/fnx_gemv.h.

The library is the product: there is no Python or torch fallback.  If ``_fnx.so`` is
missing, importing an operator raises, naming the build command.
"""

from __future__ import annotations

import ctypes
import threading
from ctypes import POINTER, c_char_p, c_float, c_int, c_int64, c_void_p

from .build import LIB_PATH

FNX_OK, FNX_EINVAL, FNX_ECUDA, FNX_EUNSUPPORTED = 0, 1, 2, 3
W_INT8, W_FP8_E4M3, W_BF16, W_NVFP4 = 0, 1, 2, 3
SCALE_NONE, SCALE_F32_SCALAR, SCALE_F32_ROW, SCALE_BF16_SCALAR, SCALE_BF16_ROW = 0, 1, 2, 3, 4
MAX_M = 16
STATIC_PARTIAL_FLOATS, STATIC_COUNTERS = 256 * 1024, 2048  # fnx_w8a16_gemv_static_ws limits
PEER_BUFFER_BYTES, IPC_HANDLE_BYTES, MAX_PEERS = 4096, 64, 8
# device error codes (FNX_DEVERR_* in include/fnx_gemv.h)
DEVICE_ERRORS = {
    1: "WAIT_FULL: a consumer waited for a weight stage",
    2: "WAIT_EMPTY: the producer waited for a free stage",
    3: "WAIT_RED: an epilogue waited for consumer partials",
    4: "WAIT_RFREE: a consumer waited for a free reduction slot",
    5: "DRAIN: in-flight copies did not land before exit",
    6: "WAIT_X: the activation rows did not arrive",
    7: "WAIT_PEER: another rank did not publish its greedy key",
    8: "PEER_DESYNC: another rank is two or more calls ahead",
    9: "ROUTES: a routing table the kernel cannot hold",
    10: "WAIT_EXPERT: a down projection waited for its expert's activations",
    11: "RING: a launch whose ring stages the waits cannot order",
}

EXPORTED = (
    "fnx_set_dense_path",
    "fnx_set_moe_path",
    "fnx_plan_gemv",
    "fnx_gemv_workspace_need",
    "fnx_w8a16_gemv",
    "fnx_w8a16_gemv_static_ws",
    "fnx_w8a16_gemv_silu_mul",
    "fnx_w8a16_gemv_norm_gated",
    "fnx_router_gemv_topk",
    "fnx_softmax_topk",
    "fnx_draft_topk1",
    "fnx_draft_head_topk1",
    "fnx_peer_alloc",
    "fnx_peer_free",
    "fnx_ipc_get_handle",
    "fnx_ipc_open",
    "fnx_ipc_close",
    "fnx_peer_setup",
    "fnx_peer_set_wait_limit",
    "fnx_w8a16_gemv_vocab_sharded",
    "fnx_w4a16_nvfp4_gemv",
    "fnx_nvfp4_quantize",
    "fnx_nvfp4_dequantize",
    "fnx_moe_workspace_bytes",
    "fnx_plan_moe",
    "fnx_moe_gemv",
    "fnx_argmax_decode",
    "fnx_static_ws_error",
    "fnx_last_error",
    "fnx_version",
)


class FnxWorkspace(ctypes.Structure):
    _fields_ = [
        ("partials", c_void_p),
        ("partial_floats", c_int64),
        ("counters", c_void_p),
        ("n_counters", c_int64),
        ("argmax_keys", c_void_p),
        ("argmax_count", c_void_p),
        ("error_flag", c_void_p),
    ]


class FnxGemvCfg(ctypes.Structure):
    _fields_ = [
        ("warps", c_int),
        ("chunks_per_warp", c_int),
        ("groups", c_int),
        ("ksplit", c_int),
        ("grid", c_int),
    ]


class FnxMoeWeights(ctypes.Structure):
    _fields_ = [
        ("w13", c_void_p),
        ("w13_scale", c_void_p),
        ("w13_gscale", c_void_p),
        ("w13_gscale_stride", c_int64),
        ("w2", c_void_p),
        ("w2_scale", c_void_p),
        ("w2_gscale", c_void_p),
        ("w2_gscale_stride", c_int64),
        ("num_experts", c_int),
        ("expert_offset", c_int),
        ("hidden", c_int),
        ("inter", c_int),
        ("scales_swizzled", c_int),
    ]


class FnxMoeWorkspace(ctypes.Structure):
    _fields_ = [
        ("act", c_void_p),
        ("partials", c_void_p),
        ("error_flag", c_void_p),
        ("max_m", c_int),
        ("max_routes", c_int),
        ("counters", c_void_p),
        ("n_counters", c_int64),
    ]


class FnxMoeWorkspaceSizes(ctypes.Structure):
    _fields_ = [
        ("act", c_int64),
        ("partials", c_int64),
        ("counters", c_int64),
    ]


_lock = threading.Lock()
_lib = None

_P = c_void_p
_I64P = POINTER(c_int64)


def _declare(lib):
    lib.fnx_set_dense_path.argtypes = [c_int, POINTER(c_int)]
    lib.fnx_set_moe_path.argtypes = [c_int, POINTER(c_int)]
    lib.fnx_plan_gemv.argtypes = [c_int, c_int, c_int, c_int, c_int, c_int, POINTER(FnxGemvCfg)]
    lib.fnx_gemv_workspace_need.argtypes = [c_int, c_int, c_int, c_int, c_int,
                                            POINTER(FnxGemvCfg), _I64P, _I64P]
    lib.fnx_w8a16_gemv.argtypes = [
        _P, c_int64, _P, c_int64, c_int, _P, c_int, _P, c_int64, _P, c_int64, c_int64, c_int,
        _P, _P, c_int64, c_int, c_int, c_int, POINTER(FnxGemvCfg), POINTER(FnxWorkspace), c_int,
        _P]
    lib.fnx_w8a16_gemv_static_ws.argtypes = [
        _P, c_int64, _P, c_int64, c_int, _P, c_int, _P, c_int64, _P, c_int64, c_int64, c_int,
        _P, _P, c_int64, c_int, c_int, c_int, POINTER(FnxGemvCfg), c_int, _P]
    lib.fnx_w8a16_gemv_silu_mul.argtypes = [
        _P, c_int64, _P, c_int64, c_int, _P, c_int, _P, c_int64, c_int, c_int, c_int,
        POINTER(FnxGemvCfg), POINTER(FnxWorkspace), c_int, _P]
    lib.fnx_w8a16_gemv_norm_gated.argtypes = [
        _P, c_int64, _P, c_int64, _P, c_int, c_int, c_float, c_int, _P, c_int64, c_int, _P,
        c_int, _P, c_int64, c_int, c_int, c_int, c_int, POINTER(FnxGemvCfg),
        POINTER(FnxWorkspace), c_int, _P]
    lib.fnx_router_gemv_topk.argtypes = [
        _P, c_int64, _P, c_int64, _P, _P, c_int64, _P, _P, c_int64, c_int, c_int, c_int, c_int,
        c_int, POINTER(FnxWorkspace), c_int, _P]
    lib.fnx_softmax_topk.argtypes = [
        _P, c_int64, c_int, _P, _P, _P, c_int64, c_int, c_int, c_int, c_int, c_int, _P]
    lib.fnx_draft_topk1.argtypes = [
        _P, c_int64, c_int, c_int, c_int, _P, _P, _P, c_int64, c_int, _P, _P,
        POINTER(FnxWorkspace), c_int, _P]
    lib.fnx_draft_head_topk1.argtypes = [
        _P, c_int64, _P, c_int64, c_int, _P, c_int, _P, c_int64, c_int, c_int, c_int, c_int,
        _P, _P, _P, c_int64, c_int, _P, _P, POINTER(FnxGemvCfg), POINTER(FnxWorkspace), c_int,
        _P]
    lib.fnx_peer_alloc.argtypes = [POINTER(c_void_p)]
    lib.fnx_peer_free.argtypes = [_P]
    lib.fnx_ipc_get_handle.argtypes = [_P, _P]
    lib.fnx_ipc_open.argtypes = [_P, POINTER(c_void_p)]
    lib.fnx_ipc_close.argtypes = [_P]
    lib.fnx_peer_setup.argtypes = [_P, POINTER(c_void_p), c_int, c_int]
    lib.fnx_w8a16_gemv_vocab_sharded.argtypes = [
        _P, c_int64, _P, c_int64, c_int, _P, c_int, _P, c_int64, c_int, _P, c_int64, c_int,
        c_int, c_int, _P, POINTER(FnxGemvCfg), POINTER(FnxWorkspace), c_int, _P]
    lib.fnx_w4a16_nvfp4_gemv.argtypes = [
        _P, c_int64, _P, c_int64, _P, c_int64, _P, c_int, _P, c_int64, _P, c_int64, c_int64,
        c_int, _P, _P, c_int64, c_int, c_int, c_int, POINTER(FnxGemvCfg),
        POINTER(FnxWorkspace), c_int, _P]
    lib.fnx_nvfp4_quantize.argtypes = [_P, c_int64, c_int, c_int, c_int, _P, c_int64, _P, c_int64,
                                       _P, _P, _P]
    lib.fnx_nvfp4_dequantize.argtypes = [_P, c_int64, _P, c_int64, _P, c_int, _P, c_int64, c_int,
                                         c_int, c_int, _P]
    lib.fnx_moe_workspace_bytes.argtypes = [c_int, c_int, c_int, c_int, c_int,
                                            POINTER(FnxMoeWorkspaceSizes)]
    lib.fnx_plan_moe.argtypes = [c_int, c_int, c_int, c_int, c_int, POINTER(c_int), POINTER(c_int),
                                 POINTER(c_int), POINTER(c_int64)]
    lib.fnx_moe_gemv.argtypes = [
        _P, c_int64, _P, _P, c_int, c_int, POINTER(FnxMoeWeights), POINTER(FnxMoeWeights), _P,
        c_int64, c_int, POINTER(FnxMoeWorkspace), c_int, _P]
    lib.fnx_argmax_decode.argtypes = [_P, _P, c_int, _P]
    lib.fnx_peer_set_wait_limit.argtypes = [_P, c_int64]
    lib.fnx_static_ws_error.argtypes = [c_int, _P, POINTER(c_int)]
    lib.fnx_last_error.restype = c_char_p
    lib.fnx_version.restype = c_char_p
    for name in EXPORTED:
        if name not in ("fnx_last_error", "fnx_version"):
            getattr(lib, name).restype = c_int


def lib():
    """The loaded library (built on first use when nvcc is available)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                try:
                    from .build import build

                    build()
                except Exception as e:  # pragma: no cover - depends on the toolchain
                    raise ImportError(
                        f"{LIB_PATH.name} is missing and could not be built ({e}); run "
                        "`python -m flash_next_rtxpro6000_b200.build` on a machine with nvcc"
                    ) from e
            handle = ctypes.CDLL(str(LIB_PATH))
            _declare(handle)
            _lib = handle
    return _lib


def last_error() -> str:
    return lib().fnx_last_error().decode("utf-8", "replace")


def check(rc: int, what: str) -> None:
    """Raise the Python exception the reference raises for the same condition."""
    if rc == FNX_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc == FNX_EINVAL:
        raise ValueError(msg)
    if rc == FNX_EUNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(msg)


def ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())
