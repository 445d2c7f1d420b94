"""The C-ABI library on a machine without a GPU: it loads, exports every entry point
include/fnx_gemv.h declares, plans every benchmark shape sensibly, and rejects invalid
arguments (the reference's asserts / ValueErrors) before any launch."""

import ctypes
import os
import re

import pytest

from flash_next_rtxpro6000_b200 import _lib
from flash_next_rtxpro6000_b200._lib import (FnxGemvCfg, FnxMoeWeights, FnxMoeWorkspace,
                                             FnxMoeWorkspaceSizes)

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "fnx_gemv.h")


def declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(fnx_\w+)\(", src, re.M)))


def test_header_declares_the_binding_surface():
    assert declared() == sorted(_lib.EXPORTED)


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    for name in declared():
        assert hasattr(lib, name), name
    assert lib.fnx_version().decode().startswith("fnx-b200")


@pytest.mark.parametrize("M", [1, 4, 16])
@pytest.mark.parametrize("N,K,wt", [
    (151936, 2048, _lib.W_INT8), (49152, 2048, _lib.W_INT8), (4096, 2048, _lib.W_NVFP4),
    (1024, 2048, _lib.W_FP8_E4M3), (2048, 512, _lib.W_INT8), (1000, 2560, _lib.W_FP8_E4M3),
    (32768, 2048, _lib.W_NVFP4), (700, 1024, _lib.W_BF16)])
def test_planner_invariants(M, N, K, wt):
    c = FnxGemvCfg()
    assert _lib.lib().fnx_plan_gemv(M, N, K, wt, 0, 0, ctypes.byref(c)) == 0
    ch = {_lib.W_INT8: 64, _lib.W_FP8_E4M3: 64, _lib.W_BF16: 32, _lib.W_NVFP4: 128}[wt]
    # groups = 16-row tiles per unit; warps / groups consumer warps share each tile's k
    assert 1 <= c.groups <= 4 and c.warps % c.groups == 0 and c.warps <= 16
    assert (c.warps // c.groups) * c.chunks_per_warp * c.ksplit == K // ch
    assert c.chunks_per_warp in (1, 2, 4, 8)
    if N >= 49152:
        assert c.ksplit == 1  # the wide heads fill the machine on N alone


def _gemv(**kw):
    args = dict(x=16, ldx=2048, w=16, ldw=2048, wt=_lib.W_INT8, s=16, sk=_lib.SCALE_F32_ROW,
                y=16, ldy=1024, y2=None, ldy2=0, split=0, f32=0, am=None, key=None, off=0,
                M=1, N=1024, K=2048, cfg=None, ws=None, pdl=0, stream=None)
    args.update(kw)
    return _lib.lib().fnx_w8a16_gemv(*args.values())


@pytest.mark.parametrize("kw,code", [
    (dict(M=17), _lib.FNX_EINVAL),
    (dict(x=None), _lib.FNX_EINVAL),
    (dict(x=8), _lib.FNX_EINVAL),               # misaligned activation rows
    (dict(ldw=2040), _lib.FNX_EINVAL),          # row stride below K / not 16-byte
    (dict(K=2000, ldx=2000, ldw=2000), _lib.FNX_EUNSUPPORTED),
    (dict(K=2016, ldx=2016, ldw=2016), _lib.FNX_EUNSUPPORTED),
    (dict(sk=9), _lib.FNX_EINVAL),
    (dict(y2=16, ldy2=1024, split=0), _lib.FNX_EINVAL),
    (dict(y2=16, ldy2=1024, split=1024), _lib.FNX_EINVAL),
    (dict(am=16), _lib.FNX_EINVAL),             # argmax without a workspace
    (dict(wt=_lib.W_NVFP4), _lib.FNX_EINVAL),   # NVFP4 has its own entry point
])
def test_invalid_arguments_are_rejected(kw, code):
    assert _gemv(**kw) == code
    assert _lib.last_error()


def test_zero_tokens_returns_ok_without_launch():
    assert _gemv(M=0) == _lib.FNX_OK


def test_moe_validation():
    lib = _lib.lib()
    w = FnxMoeWeights(16, 16, 16, 2, 16, 16, 16, 1, 512, 0, 2000, 512, 1)
    ws = FnxMoeWorkspace(16, 16, 16, 16, 10)
    rc = lib.fnx_moe_gemv(16, 2000, 16, 16, 1, 10, ctypes.byref(w), None, 16, 2000, 0,
                          ctypes.byref(ws), 0, None)
    assert rc == _lib.FNX_EUNSUPPORTED
    w.hidden = 2048
    rc = lib.fnx_moe_gemv(16, 2048, 16, 16, 17, 10, ctypes.byref(w), None, 16, 2048, 0,
                          ctypes.byref(ws), 0, None)
    assert rc == _lib.FNX_EINVAL
    ws.max_m = 1
    rc = lib.fnx_moe_gemv(16, 2048, 16, 16, 2, 10, ctypes.byref(w), None, 16, 2048, 0,
                          ctypes.byref(ws), 0, None)
    assert rc == _lib.FNX_EINVAL


def test_moe_workspace_bytes():
    z = FnxMoeWorkspaceSizes()
    assert _lib.lib().fnx_moe_workspace_bytes(16, 10, 512, 2048, 512, ctypes.byref(z)) == 0
    P = 16 * 11
    assert (z.act, z.partials) == (161 * 16 * (2 * 512 + 64), P * 2048 * 4)


def _norm_gated(**kw):
    args = dict(x=16, ldx=2048, z=16, ldz=2048, nw=16, nw32=0, G=128, eps=1e-6, sig=0, w=16,
                ldw=2048, wt=_lib.W_FP8_E4M3, s=16, sk=_lib.SCALE_F32_ROW, y=16, ldy=1024,
                f32=0, M=1, N=1024, K=2048, cfg=None, ws=None, pdl=0, stream=None)
    args.update(kw)
    return _lib.lib().fnx_w8a16_gemv_norm_gated(*args.values())


@pytest.mark.parametrize("kw,code", [
    (dict(G=96, K=384, ldx=384, ldz=384, ldw=384), _lib.FNX_EUNSUPPORTED),
    (dict(G=512), _lib.FNX_EUNSUPPORTED),
    (dict(G=4), _lib.FNX_EUNSUPPORTED),
    (dict(G=0), _lib.FNX_EINVAL),
    (dict(G=128, K=2000, ldx=2000, ldz=2000, ldw=2000), _lib.FNX_EINVAL),
    (dict(z=None), _lib.FNX_EINVAL),
    (dict(z=8), _lib.FNX_EINVAL),                # misaligned gate rows
    (dict(ldz=1024), _lib.FNX_EINVAL),
    (dict(nw=None), _lib.FNX_EINVAL),
    (dict(eps=-1.0), _lib.FNX_EINVAL),
    (dict(wt=_lib.W_NVFP4), _lib.FNX_EINVAL),
    (dict(M=17), _lib.FNX_EINVAL),
])
def test_norm_gated_invalid_arguments_are_rejected(kw, code):
    assert _norm_gated(**kw) == code
    assert _lib.last_error()


def _router(**kw):
    args = dict(x=16, ldx=2048, w=16, ldw=2048, bias=None, logits=16, ldl=512, tw=16, ti=16,
                ldk=10, M=1, N=512, K=2048, topk=10, renorm=1, ws=None, pdl=0, stream=None)
    args.update(kw)
    return _lib.lib().fnx_router_gemv_topk(*args.values())


@pytest.mark.parametrize("kw,code", [
    (dict(M=0), _lib.FNX_EINVAL),
    (dict(M=17), _lib.FNX_EINVAL),
    (dict(K=2000, ldx=2000, ldw=2000), _lib.FNX_EINVAL),   # K % 128
    (dict(N=500), _lib.FNX_EINVAL),                         # N % 32
    (dict(x=8), _lib.FNX_EINVAL),                           # misaligned rows
    (dict(topk=33, N=1024, ldl=1024), _lib.FNX_EUNSUPPORTED),
    (dict(topk=10, N=1024, ldl=1024), _lib.FNX_EUNSUPPORTED),  # > 512 experts for the top-k
    (dict(topk=10, ws=None), _lib.FNX_EINVAL),              # the top-k needs the counter
    (dict(topk=0, logits=None), _lib.FNX_EINVAL),
    (dict(ldk=4), _lib.FNX_EINVAL),
])
def test_router_invalid_arguments_are_rejected(kw, code):
    assert _router(**kw) == code
    assert _lib.last_error()


@pytest.mark.parametrize("kw,code", [
    (dict(N=513), _lib.FNX_EUNSUPPORTED),
    (dict(topk=0), _lib.FNX_EINVAL),
    (dict(topk=40, N=64), _lib.FNX_EUNSUPPORTED),
    (dict(topk=65, N=64), _lib.FNX_EINVAL),
    (dict(lds=10), _lib.FNX_EINVAL),
])
def test_softmax_topk_invalid_arguments_are_rejected(kw, code):
    args = dict(s=16, lds=512, f32=0, bias=None, tw=16, ti=16, ldk=32, M=2, N=512, topk=10,
                renorm=1, pdl=0, stream=None)
    args.update(kw)
    if "N" in kw and "lds" not in kw:
        args["lds"] = max(args["N"], 1)
    assert _lib.lib().fnx_softmax_topk(*args.values()) == code


@pytest.mark.parametrize("kw,code", [
    (dict(M=17), _lib.FNX_EUNSUPPORTED),
    (dict(V=0), _lib.FNX_EINVAL),
    (dict(ldl=10), _lib.FNX_EINVAL),
    (dict(dt=16, ldd=3, col=3), _lib.FNX_EINVAL),   # column outside the row
    (dict(ti=None, tp=None), _lib.FNX_EINVAL),      # nothing to write
    (dict(ws=None), _lib.FNX_EINVAL),               # keys and counter live in the workspace
])
def test_draft_topk1_invalid_arguments_are_rejected(kw, code):
    from flash_next_rtxpro6000_b200._lib import FnxWorkspace

    fake = FnxWorkspace(16, 0, 16, 0, 16, 16, 16)  # checked for presence only, never read
    args = dict(lg=16, ldl=1000, f32=1, M=2, V=1000, hot=None, pos=None, dt=None, ldd=0, col=0,
                ti=16, tp=16, ws=ctypes.byref(fake), pdl=0, stream=None)
    args.update(kw)
    assert _lib.lib().fnx_draft_topk1(*args.values()) == code
    assert _lib.last_error()
