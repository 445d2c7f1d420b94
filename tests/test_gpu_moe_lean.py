"""The decode-width MoE layer (moe_lean_kernel, one token) against the CPU oracle and
against the general one-launch layer: config 2 with 512 experts,
other layer shapes (1024 x 256, 2048 x 256), routings that crowd
one expert or repeat ids, expert-parallel slices with fp32 partial sums, a PDL chain in a
CUDA graph, and the tile counters back at zero after every call."""

import numpy as np
import pytest
import torch

from tests.gpu_util import REL_TOL, dev, rel_err, to_np, ulps
from tests.test_gpu_moe import _layer, _oracle, _run, _shared

pytestmark = pytest.mark.gpu


def _fx():
    import flash_next_rtxpro6000_b200 as fx

    return fx


@pytest.mark.parametrize("M", [1])
def test_lean_config2_matches_oracle_and_fused(M):
    fx = _fx()
    from flash_next_rtxpro6000_b200 import synthetic as syn

    E = 512
    assert fx.moe_plan(M, 10, E, 2048, 512)["form"] == "lean"
    assert fx.moe_plan(2, 10, E, 2048, 512)["form"] == "fused"
    L, d = _layer(E)
    x = syn.activations(M, seed=40 + M)
    ids, wts = syn.routing(M, E=E, seed=400 + M)
    ws = fx.make_workspace(num_routes=10, hidden_size=2048, intermediate_size=512, device=dev())
    xd, idd, wd = x.to(dev()), ids.to(dev()), wts.to(dev())
    y = _run(fx, d, xd, idd, wd, ws).clone()
    with fx.moe_path("fused"):
        yf = _run(fx, d, xd, idd, wd, ws).clone()
    torch.cuda.synchronize()
    ref = _oracle(L, x, ids, wts)
    got = to_np(y)
    assert rel_err(got, ref) <= REL_TOL
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 5e-3
    # same arithmetic as the general layer up to the order of the fp32 k sums
    u = ulps(got, to_np(yf))
    big = np.abs(ref) >= 1e-2 * np.abs(ref).max()
    assert u[big].max() <= 2 and (u == 0).mean() > 0.9
    assert int(ws.error_flag.item()) == 0
    assert int(torch.count_nonzero(ws.counters)) == 0


@pytest.mark.parametrize("H,I", [(2048, 256), (1024, 256)])
@pytest.mark.parametrize("M", [1])
def test_lean_other_shapes(M, H, I):
    """Layers with two k chunks in the down projection (I = 256) and a short hidden size.
    The reference model's own 2560 x 640 shape has rows of 320 bytes, which the 128-byte
    TMA boxes do not tile: it takes the general one-launch layer
    (tests/test_gpu_moe.py::test_reference_model_shape)."""
    fx = _fx()
    from flash_next_rtxpro6000_b200 import synthetic as syn

    assert fx.moe_plan(M, 10, 64, H, I)["form"] == "lean"
    assert fx.moe_plan(M, 10, 64, 2560, 640)["form"] == "fused"
    L, d = _layer(64, H=H, I=I, seed=1)
    x = syn.activations(M, K=H, seed=21)
    ids, wts = syn.routing(M, E=64, seed=210 + M)
    ws = fx.make_workspace(num_routes=10, hidden_size=H, intermediate_size=I, device=dev())
    y = _run(fx, d, x.to(dev()), ids.to(dev()), wts.to(dev()), ws)
    torch.cuda.synchronize()
    assert rel_err(to_np(y), _oracle(L, x, ids, wts)) <= REL_TOL
    assert int(ws.error_flag.item()) == 0
    assert int(torch.count_nonzero(ws.counters)) == 0


@pytest.mark.parametrize("M", [1])
def test_lean_crowded_repeated_and_skipped_routes(M):
    """All tokens on one expert, ids repeated within a row, and ids < 0: every route is
    served (a slot holds any set of tokens) and the skipped ones add nothing."""
    fx = _fx()
    from flash_next_rtxpro6000_b200 import synthetic as syn

    L, d = _layer(64)
    x = syn.activations(M, seed=22)
    _, wts = syn.routing(M, E=64, seed=22)
    g = torch.Generator().manual_seed(M)
    mixed = torch.randint(0, 3, (M, 10), generator=g, dtype=torch.int32)  # repeated ids
    mixed[0, 4] = -1
    skipped = mixed.clone()
    skipped[M - 1, :] = -1
    for ids in (torch.full((M, 10), 7, dtype=torch.int32), mixed, skipped):
        ws = fx.make_workspace(num_routes=10, hidden_size=2048, intermediate_size=512,
                               device=dev())
        for shared in (True, False):
            y = _run(fx, d, x.to(dev()), ids.to(dev()), wts.to(dev()), ws, shared=shared)
            torch.cuda.synchronize()
            ref = _oracle(L, x, ids, wts, shared=shared)
            assert rel_err(to_np(y), ref) <= REL_TOL
            if not shared and bool((ids[M - 1] < 0).all()):
                assert int(torch.count_nonzero(y[M - 1])) == 0
        assert int(ws.error_flag.item()) == 0
        assert int(torch.count_nonzero(ws.counters)) == 0


def test_lean_expert_slices_sum_to_layer():
    """Expert-parallel slices (expert_offset, fp32 partial sums) add up to the layer."""
    fx = _fx()
    from flash_next_rtxpro6000_b200 import synthetic as syn

    L, d = _layer(64)
    M = 1
    x = syn.activations(M, seed=23).to(dev())
    ids, wts = syn.routing(M, E=64, seed=23)
    ids, wts = ids.to(dev()), wts.to(dev())
    ws = fx.make_workspace(num_routes=10, hidden_size=2048, intermediate_size=512, device=dev())
    full = _run(fx, d, x, ids, wts, ws, out_f32=True).clone()
    total = torch.zeros_like(full)
    G, per = 4, 16
    for r in range(G):
        sl = slice(r * per, (r + 1) * per)
        part = fx.draft_moe_gemv(
            hidden_states=x, topk_ids=ids, topk_weights=wts, w13_weight=d["w13"][sl].contiguous(),
            w13_blockscale_swizzled=d["s13"][sl].contiguous(),
            w13_weight_scale_2=d["g13"][sl].contiguous(), w2_weight=d["w2"][sl].contiguous(),
            w2_blockscale_swizzled=d["s2"][sl].contiguous(),
            w2_weight_scale_2=d["g2"][sl].contiguous(), workspace=ws,
            shared_expert=_shared(fx, d) if r == 0 else None, expert_offset=r * per, out_f32=True)
        total += part
    assert rel_err(to_np(total), to_np(full)) <= 1e-5
    assert int(torch.count_nonzero(ws.counters)) == 0


def test_lean_back_to_back_pdl_chain():
    """Forty calls in a row on one stream with programmatic dependent launch, captured in
    a graph and replayed: every call's output matches a standalone run bit for bit."""
    fx = _fx()
    from flash_next_rtxpro6000_b200 import synthetic as syn

    L, d = _layer(512)
    M, n = 1, 40
    x = syn.activations(M, seed=24).to(dev())
    routes = [syn.routing(M, E=512, seed=2400 + i) for i in range(n)]
    routes = [(i.to(dev()), w.to(dev())) for i, w in routes]
    ws = fx.make_workspace(num_routes=10, hidden_size=2048, intermediate_size=512, device=dev())
    outs = [torch.empty(M, 2048, dtype=torch.bfloat16, device=dev()) for _ in range(n)]
    cfg = fx.DraftMoeGemvConfig(pdl=True)
    ref = [_run(fx, d, x, i, w, ws).clone() for i, w in routes]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for (i, w), o in zip(routes, outs):
            _run(fx, d, x, i, w, ws, out=o, cfg=cfg)
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for (i, w), o in zip(routes, outs):
            _run(fx, d, x, i, w, ws, out=o, cfg=cfg)
    for o in outs:
        o.zero_()
    g.replay()
    torch.cuda.synchronize()
    for a, b in zip(outs, ref):
        assert torch.equal(a, b)
    assert int(ws.error_flag.item()) == 0
    assert int(torch.count_nonzero(ws.counters)) == 0
    del g
