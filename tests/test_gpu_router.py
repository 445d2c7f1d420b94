"""MoE router on the GPU against the CPU oracle (the oracle is pinned to the reference's
top-k kernel by tests/test_oracle_golden.py): router_gemv logits (router_gemv.py:10-93),
route_softmax_fast on the reference's own golden inputs and on random bf16 / fp32 logits
with ties, the fused router_topk (ids exact and weights to fp32 rounding against the
oracle's top-k of the kernel's own logits; the arrival counter left at zero; graph replay
bitwise), its routing table driving the MoE, and the reference's ValueErrors."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import router as orouter
from tests.gpu_util import dev, to_np

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _fx():
    import flash_next_rtxpro6000_b200 as fx

    return fx


def _case(M, N, K, seed, bias=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).bfloat16()
    w = (torch.randn(N, K, generator=g) * 0.05).bfloat16()
    b = (torch.randn(N, generator=g) * 0.1).bfloat16() if bias else None
    return x, w, b


def _logit_err(got, ref):
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


@pytest.mark.parametrize("bias", [False, True])
@pytest.mark.parametrize("M", [1, 3, 8, 9, 16])
@pytest.mark.parametrize("N,K", [(512, 2048), (256, 1024), (128, 384)])
def test_router_gemv_matches_oracle(N, K, M, bias):
    fx = _fx()
    x, w, b = _case(M, N, K, seed=N + K + M, bias=bias)
    d = dev()
    y = fx.router_gemv(x.to(d), w.to(d), None if b is None else b.to(d))
    assert y.dtype == torch.float32 and y.shape == (M, N)
    ref = orouter.router_logits(x.float().numpy(), w.float().numpy(),
                                None if b is None else b.float().numpy())
    assert _logit_err(to_np(y), ref) <= 1e-5  # fp32 sums of exact bf16 products


@pytest.mark.parametrize("case", ["a", "b", "c", "d"])
def test_route_softmax_fast_matches_reference_golden(case):
    fx = _fx()
    g = np.load(GOLDEN / "router_topk.npz")
    k, renorm = (int(v) for v in g[f"topk_{case}"])
    scores = torch.from_numpy(g[f"scores_{case}"]).bfloat16().to(dev())
    zero = torch.zeros(scores.shape[1], dtype=torch.float32, device=dev())
    assert fx.covered(scores, zero, k)
    w, ids = fx.route_softmax_fast(scores, zero, k, bool(renorm))
    assert w.dtype == torch.float32 and ids.dtype == torch.int32
    assert np.array_equal(ids.cpu().numpy(), g[f"ids_{case}"])
    ref = g[f"w_{case}"]
    got = w.cpu().numpy()
    nan = np.isnan(ref)
    assert np.array_equal(nan, np.isnan(got))
    assert np.allclose(got[~nan], ref[~nan], rtol=2e-6, atol=1e-9)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("N,k", [(512, 10), (64, 8), (96, 32), (32, 1)])
def test_route_softmax_fast_matches_oracle(dtype, N, k):
    fx = _fx()
    g = torch.Generator().manual_seed(N * 31 + k)
    s = torch.randint(-6, 7, (13, N), generator=g).float() * 0.25  # many ties
    s[::2] = torch.randn(7, N, generator=g) * 3
    s = s.to(dtype)
    bias = torch.randn(N, generator=g) * 0.01
    for b in (None, bias):
        for renorm in (True, False):
            w, ids = fx.route_softmax_fast(s.to(dev()), None if b is None else b.to(dev()), k,
                                           renorm)
            ow, oids = orouter.softmax_topk(s.float().numpy(), k, renorm,
                                            None if b is None else b.float().numpy())
            assert np.array_equal(ids.cpu().numpy(), oids)
            assert np.allclose(w.cpu().numpy(), ow, rtol=2e-6, atol=1e-9)


@pytest.mark.parametrize("M", [1, 4, 16])
@pytest.mark.parametrize("bias", [False, True])
def test_router_topk_fused(M, bias):
    fx = _fx()
    from flash_next_rtxpro6000_b200.w8a16_gemv import _workspace

    N, K, k = 512, 2048, 10
    x, w, b = _case(M, N, K, seed=M + 100, bias=bias)
    d = dev()
    xd, wd, bd = x.to(d), w.to(d), None if b is None else b.to(d)
    logits = torch.empty(M, N, dtype=torch.float32, device=d)
    tw, tids = fx.router_topk(xd, wd, bd, k, True, logits_out=logits)
    torch.cuda.synchronize()
    ref = orouter.router_logits(x.float().numpy(), w.float().numpy(),
                                None if b is None else b.float().numpy())
    lg = to_np(logits)
    assert _logit_err(lg, ref) <= 1e-5
    ow, oids = orouter.softmax_topk(lg, k, True)
    assert np.array_equal(tids.cpu().numpy(), oids)
    assert np.allclose(tw.cpu().numpy(), ow, rtol=2e-6, atol=1e-9)
    assert int(_workspace(d).counters[0]) == 0
    # same table from the unfused pair, and from the internal logits buffer
    w2, i2 = fx.route_softmax_fast(fx.router_gemv(xd, wd, bd), None, k, True)
    assert torch.equal(i2, tids) and torch.equal(w2, tw)
    w3, i3 = fx.router_topk(xd, wd, bd, k, True)
    assert torch.equal(i3, tids) and torch.equal(w3, tw)


def test_router_topk_graph_replay_bitwise():
    fx = _fx()
    M, N, K, k = 4, 512, 2048, 10
    x, w, _ = _case(M, N, K, seed=5)
    d = dev()
    xd, wd = x.to(d), w.to(d)
    tw, tids = fx.router_topk(xd, wd, None, k, True)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fx.router_topk(xd, wd, None, k, True)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        gw, gids = fx.router_topk(xd, wd, None, k, True)
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(gids, tids) and torch.equal(gw, tw)


def test_routing_table_drives_the_moe():
    # the fused router's table goes straight into the MoE GEMV, as in the decode step
    fx = _fx()
    from flash_next_rtxpro6000_b200 import synthetic as syn
    from flash_next_rtxpro6000_b200.w4a16_nvfp4_gemv import swizzle_blockscale
    from oracle import moe as omoe
    from tests.gpu_util import REL_TOL, rel_err

    E, H, I, M, k = 64, 2048, 512, 4, 10
    L = syn.moe_layer(E, H, I, seed=3)
    d = dev()
    x = syn.activations(M, seed=4)
    rw = (torch.randn(E, H, generator=torch.Generator().manual_seed(6)) * 0.05).bfloat16()
    tw, tids = fx.router_topk(x.to(d), rw.to(d), None, k, True)
    ws = fx.make_workspace(num_routes=k, hidden_size=H, intermediate_size=I, device=d)
    y = fx.draft_moe_gemv(
        hidden_states=x.to(d), topk_ids=tids, topk_weights=tw, w13_weight=L.w13.to(d),
        w13_blockscale_swizzled=swizzle_blockscale(L.s13.to(d)), w13_weight_scale_2=L.g13.to(d),
        w2_weight=L.w2.to(d), w2_blockscale_swizzled=swizzle_blockscale(L.s2.to(d)),
        w2_weight_scale_2=L.g2.to(d), workspace=ws)
    ref = omoe.moe(x.float().numpy(), tids.cpu().numpy(), tw.cpu().numpy(), L.w13.numpy(),
                   L.s13.numpy(), L.g13.numpy(), L.w2.numpy(), L.s2.numpy(), L.g2.numpy(),
                   order="server")
    assert rel_err(to_np(y), ref) <= REL_TOL


def test_reference_value_errors():
    fx = _fx()
    d = dev()
    x, w, _ = _case(2, 64, 256, seed=1)
    x, w = x.to(d), w.to(d)
    bad = [
        (torch.zeros(17, 256, dtype=torch.bfloat16, device=d), w, None),       # M > 16
        (x[:, :200].contiguous(), w[:, :200].contiguous(), None),              # K % 128
        (x, torch.zeros(48, 256, dtype=torch.bfloat16, device=d), None),       # N % 32
        (x.float(), w, None),                                                  # dtype
        (x.cpu(), w, None),                                                    # not CUDA
        (x, w, torch.zeros(64, dtype=torch.float32, device=d)),                # bias dtype
        (torch.zeros(256, 2, dtype=torch.bfloat16, device=d).t(), w, None),   # strided
    ]
    for xx, ww, bb in bad:
        with pytest.raises(ValueError):
            fx.router_gemv(xx, ww, bb)
