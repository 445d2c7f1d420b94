"""The tcgen05 (tensor-memory) form of the dense GEMV against the CPU oracle and against
the mma.sync form: every token count, ragged and tiny row counts, K down to one chunk,
both 8-bit weight formats, both scale formats, fp32 and two-destination stores, the fused
greedy argmax (bit-exact on the lm_head), bitwise graph replay with the stream-K counters
back at zero."""

import numpy as np
import pytest
import torch

from oracle import numerics, w8a16 as ow8
from tests.gpu_util import REL_TOL, dev, rel_err, to_np, ulps

pytestmark = pytest.mark.gpu


def _fx():
    import flash_next_rtxpro6000_b200 as fx

    return fx


def _case(N, K, M, kind, sdtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).bfloat16()
    if kind == "int8":
        w = torch.randint(-128, 128, (N, K), generator=g, dtype=torch.int8)
        w_np = w.numpy()
    else:
        w = (torch.randn(N, K, generator=g) * 64).to(torch.float8_e4m3fn)
        w_np = w.view(torch.uint8).numpy()
    s = (torch.randn(N, generator=g).abs() / 127).to(sdtype)
    return x, w, s, w_np


def _check(got, ref):
    assert rel_err(got, ref) <= REL_TOL
    u = ulps(got, ref)
    big = np.abs(ref) >= 1e-2 * np.abs(ref).max()
    assert u[big].max() <= 2 and (u == 0).mean() > 0.97


@pytest.mark.parametrize("kind", ["int8", "fp8"])
@pytest.mark.parametrize("M", [1, 3, 8, 9, 16])
@pytest.mark.parametrize("N,K", [(1000, 2048), (128, 128), (100, 256), (1, 384), (4096, 512),
                                 (3000, 1024), (777, 4096)])
def test_tcgen05_matches_oracle(kind, M, N, K):
    fx = _fx()
    x, w, s, w_np = _case(N, K, M, kind, torch.float32, seed=N * 7 + K + M)
    with fx.dense_path("tcgen05"):
        y = fx.w8a16_gemv(x.to(dev()), w.to(dev()), s.to(dev()))
    torch.cuda.synchronize()
    ref = ow8.gemv(x.float().numpy(), w_np, kind, s.float().numpy())
    assert y.shape == (M, N)
    _check(to_np(y), ref)


@pytest.mark.parametrize("M", [2, 12, 16])
def test_tcgen05_agrees_with_mma_sync(M):
    fx = _fx()
    x, w, s, w_np = _case(5000, 2048, M, "int8", torch.bfloat16, seed=31 + M)
    x, w, s = x.to(dev()), w.to(dev()), s.to(dev())
    with fx.dense_path("tcgen05"):
        a = fx.w8a16_gemv(x, w, s)
    with fx.dense_path("mma"):
        b = fx.w8a16_gemv(x, w, s)
    ref = ow8.gemv(x.float().cpu().numpy(), w_np, "int8", s.float().cpu().numpy())
    _check(to_np(a), ref)
    _check(to_np(b), ref)
    # the two forms sum k in different orders: outside heavy cancellation they agree to
    # a bf16 step or two
    u = ulps(to_np(a), to_np(b))
    big = np.abs(ref) >= 1e-2 * np.abs(ref).max()
    assert u[big].max() <= 2 and (u == 0).mean() > 0.97


@pytest.mark.parametrize("M", [1, 9, 16])
def test_tcgen05_fp32_out_and_two_destinations(M):
    fx = _fx()
    x, w, s, _ = _case(1200, 1024, M, "fp8", torch.float32, seed=5)
    x, w, s = x.to(dev()), w.to(dev()), s.to(dev())
    with fx.dense_path("tcgen05"):
        y16 = fx.w8a16_gemv(x, w, s)
        buf = torch.full((M, 1200), float("nan"), device=dev())
        y32 = fx.w8a16_gemv(x, w, s, out=buf)
        a = torch.empty(M, 700, device=dev(), dtype=torch.bfloat16)
        b = torch.empty(M, 500, device=dev(), dtype=torch.bfloat16)
        y, y2 = fx.w8a16_gemv(x, w, s, out=a, out2=b, split_n=700)
    assert torch.equal(y32, y16.float())
    assert torch.equal(torch.cat([y, y2], dim=1), y16)


def test_tcgen05_scalar_scale():
    fx = _fx()
    x, w, _, w_np = _case(640, 768, 16, "int8", torch.float32, seed=8)
    s = torch.tensor([0.0123], dtype=torch.float32)
    with fx.dense_path("tcgen05"):
        y = fx.w8a16_gemv(x.to(dev()), w.to(dev()), s.to(dev()))
    ref = ow8.gemv(x.float().numpy(), w_np, "int8", np.full(640, 0.0123, np.float32))
    _check(to_np(y), ref)


@pytest.mark.parametrize("M", [1, 4, 9, 16])
def test_tcgen05_lm_head_argmax_bit_exact(M):
    """Config 1 (int8 [151936, 2048] lm_head, bf16 per-row scales) on the tensor-core form:
    the fused greedy argmax equals the oracle's (fp64 logits rounded to bf16, lowest row
    on ties) and torch.argmax of the kernel's own logits."""
    fx = _fx()
    from flash_next_rtxpro6000_b200 import synthetic as syn

    head = syn.w8_head(151936, syn.HIDDEN, seed=0)
    x = syn.activations(M, seed=1)
    w, s = head.w.to(dev()), head.scale.to(dev())
    am = torch.empty(M, dtype=torch.int64, device=dev())
    with fx.dense_path("tcgen05"):
        y = fx.w8a16_gemv(x.to(dev()), w, s, argmax_out=am)
    torch.cuda.synchronize()
    exact = ow8.gemv_f64(x.float().numpy(), head.w.numpy(), "int8", head.scale.float().numpy())
    ref = numerics.bf16_round_from_f64(exact)
    assert rel_err(to_np(y), ref) <= REL_TOL
    assert am.cpu().numpy().tolist() == ow8.argmax_lowest(ref).tolist()
    assert am.cpu().tolist() == torch.argmax(y.float(), dim=-1).cpu().tolist()


@pytest.mark.parametrize("M", [9, 16])
def test_tcgen05_graph_replay_bitwise_and_counters_reset(M):
    fx = _fx()
    from flash_next_rtxpro6000_b200.w8a16_gemv import _workspace

    N, K = 20000, 2048
    x, w, s, w_np = _case(N, K, M, "int8", torch.bfloat16, seed=12)
    w, s = w.to(dev()), s.to(dev())
    xs = x.to(dev()).clone()
    am = torch.empty(M, dtype=torch.int64, device=dev())
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            fx.w8a16_gemv(xs, w, s, argmax_out=am)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        yg = fx.w8a16_gemv(xs, w, s, argmax_out=am)
    g.replay()
    torch.cuda.synchronize()
    a1, am1 = yg.clone(), am.clone()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(a1, yg) and torch.equal(am1, am)
    ref = ow8.gemv(x.float().numpy(), w_np, "int8", s.float().cpu().numpy())
    _check(to_np(a1), ref)
    assert am.cpu().tolist() == torch.argmax(yg.float(), dim=-1).cpu().tolist()
    ws = _workspace(dev())
    assert int(ws.counters.abs().sum()) == 0
    assert int(ws.argmax_keys.abs().sum()) == 0 and int(ws.argmax_count.sum()) == 0
    assert int(ws.error_flag.item()) == 0
    del g
