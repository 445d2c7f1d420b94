"""fnx_w8a16_gemv_static_ws (scratch in the library's static device array, no
allocation) against fnx_w8a16_gemv with a caller workspace, through the C ABI.

Two consecutive calls each must match the workspace entry point: the second call
only agrees if the first left the argmax keys and split-K counters at zero.  The file
name sorts last so the test also runs after every other GPU test in one session."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import w8a16 as ow8
from tests.gpu_util import REL_TOL, dev, rel_err, to_np

pytestmark = pytest.mark.gpu


def _case(N, K, M, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).bfloat16()
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    s = (torch.randn(N, generator=g).abs() / 127).bfloat16()
    return x, w, s


def _call(fn, x, w, s, y, am, keys, M, N, K, ws=None):
    from flash_next_rtxpro6000_b200 import _lib

    p = _lib.ptr
    args = [p(x), x.stride(0), p(w), w.stride(0), _lib.W_INT8, p(s), _lib.SCALE_BF16_ROW, p(y),
            y.stride(0), None, 0, 0, 0, p(am), p(keys), 0, M, N, K, None]
    if ws is not None:
        args.append(ctypes.byref(ws))
    args += [0, torch.cuda.current_stream().cuda_stream]
    return fn(*args)


# draft head, lm_head, and a split-K shape (4 k splits: partials and counters in use)
@pytest.mark.parametrize("M,N,K", [(1, 49152, 2048), (16, 151936, 2048), (4, 1024, 8192)])
def test_static_ws_matches_workspace_entry(M, N, K):
    import flash_next_rtxpro6000_b200 as fx
    from flash_next_rtxpro6000_b200 import _lib
    from flash_next_rtxpro6000_b200.w8a16_gemv import _workspace

    lib = _lib.lib()
    x, w, s = _case(N, K, M, seed=N + K + M)
    x, w, s = x.to(dev()), w.to(dev()), s.to(dev())
    need_f, need_c = ctypes.c_int64(), ctypes.c_int64()
    assert lib.fnx_gemv_workspace_need(M, N, K, _lib.W_INT8, 0, None, ctypes.byref(need_f),
                                       ctypes.byref(need_c)) == 0
    assert need_f.value <= _lib.STATIC_PARTIAL_FLOATS and need_c.value <= _lib.STATIC_COUNTERS

    y_ref = torch.empty(M, N, dtype=torch.bfloat16, device=dev())
    am_ref = torch.empty(M, dtype=torch.int64, device=dev())
    k_ref = torch.empty(M, dtype=torch.int64, device=dev())
    ws = _workspace(dev()).c
    # the static-scratch entry has no room for the tensor-core form's partial sums and
    # always runs the mma.sync form; the workspace entry is held to the same form, so the
    # greedy keys can be compared bit for bit
    with fx.dense_path("mma"):
        _lib.check(_call(lib.fnx_w8a16_gemv, x, w, s, y_ref, am_ref, k_ref, M, N, K, ws),
                   "fnx_w8a16_gemv")
    torch.cuda.synchronize()
    ref = ow8.gemv(x.float().cpu().numpy(), w.cpu().numpy(), "int8", s.float().cpu().numpy())
    assert rel_err(to_np(y_ref), ref) <= REL_TOL

    for _ in range(2):
        y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev())
        am = torch.full((M,), -1, dtype=torch.int64, device=dev())
        keys = torch.zeros(M, dtype=torch.int64, device=dev())
        _lib.check(_call(lib.fnx_w8a16_gemv_static_ws, x, w, s, y, am, keys, M, N, K),
                   "fnx_w8a16_gemv_static_ws")
        torch.cuda.synchronize()
        assert rel_err(to_np(y), to_np(y_ref)) <= REL_TOL
        assert torch.equal(am, am_ref) and torch.equal(keys, k_ref)
        assert np.array_equal(am.cpu().numpy(), np.argmax(to_np(y), axis=1))


def test_static_ws_rejects_oversized_plan():
    from flash_next_rtxpro6000_b200 import _lib

    lib = _lib.lib()
    M, N, K = 1, 2048, 32768  # split-K plan larger than the static partial buffer
    cfg = _lib.FnxGemvCfg(16, 1, 1, 32, 0)
    need_f = ctypes.c_int64()
    rc = lib.fnx_gemv_workspace_need(M, N, K, _lib.W_INT8, 0, ctypes.byref(cfg),
                                     ctypes.byref(need_f), None)
    if rc != 0:
        pytest.skip(_lib.last_error())
    assert need_f.value > _lib.STATIC_PARTIAL_FLOATS
    x = torch.zeros(M, K, dtype=torch.bfloat16, device=dev())
    w = torch.zeros(N, K, dtype=torch.int8, device=dev())
    s = torch.ones(N, dtype=torch.bfloat16, device=dev())
    y = torch.empty(M, N, dtype=torch.bfloat16, device=dev())
    p = _lib.ptr
    rc = lib.fnx_w8a16_gemv_static_ws(p(x), K, p(w), K, _lib.W_INT8, p(s), _lib.SCALE_BF16_ROW,
                                      p(y), N, None, 0, 0, 0, None, None, 0, M, N, K,
                                      ctypes.byref(cfg), 0, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.FNX_EUNSUPPORTED
    assert "static scratch too small" in _lib.last_error()
