"""Routed NVFP4 MoE (config 2) on the GPU against the CPU oracle.

Checks, after the reference's own (bench/bench/dg1/dg1_bench.py correctness and
determinism phases, bench/bench/dg1/selftest_cpu.py): output within 2e-2 of the
dequantise-then-matmul layer (with and without the bf16 rounding of the activation
between the two GEMVs), ids < 0 skipped, bitwise reruns,
graph replay on new inputs, the 128x4 swizzled and linear scale layouts agree, and
expert-sliced partial sums add up to the whole layer."""

import numpy as np
import pytest
import torch

from oracle import moe as omoe, nvfp4 as onv
from tests.gpu_util import REL_TOL, dev, rel_err, to_np

pytestmark = pytest.mark.gpu

_LAYERS = {}


def _layer(E, H=2048, I=512, seed=0):
    from flash_next_rtxpro6000_b200 import synthetic as syn

    key = (E, H, I, seed)
    if key not in _LAYERS:
        L = syn.moe_layer(E, H, I, seed=seed)
        sw13 = onv.swizzle_blockscale(L.s13.numpy())
        sw2 = onv.swizzle_blockscale(L.s2.numpy())
        ssw13 = onv.swizzle_blockscale(L.sh_s13.numpy())
        ssw2 = onv.swizzle_blockscale(L.sh_s2.numpy())
        d = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev()) for k, v in dict(
            w13=L.w13.numpy(), s13=sw13, g13=L.g13.numpy(), w2=L.w2.numpy(), s2=sw2,
            g2=L.g2.numpy(), sh_w13=L.sh_w13.numpy(), sh_s13=ssw13, sh_g13=L.sh_g13.numpy(),
            sh_w2=L.sh_w2.numpy(), sh_s2=ssw2, sh_g2=L.sh_g2.numpy(),
            s13_lin=L.s13.numpy(), s2_lin=L.s2.numpy(), sh_s13_lin=L.sh_s13.numpy(),
            sh_s2_lin=L.sh_s2.numpy()).items()}
        _LAYERS[key] = (L, d)
    return _LAYERS[key]


def _shared(fx, d, linear=False):
    sfx = "_lin" if linear else ""
    return fx.SharedExpert(d["sh_w13"], d["sh_s13" + sfx], d["sh_g13"], d["sh_w2"],
                           d["sh_s2" + sfx], d["sh_g2"])


def _run(fx, d, x, ids, wts, ws, shared=True, linear=False, **kw):
    sfx = "_lin" if linear else ""
    return fx.draft_moe_gemv(
        hidden_states=x, topk_ids=ids, topk_weights=wts, w13_weight=d["w13"],
        w13_blockscale_swizzled=d["s13" + sfx], w13_weight_scale_2=d["g13"], w2_weight=d["w2"],
        w2_blockscale_swizzled=d["s2" + sfx], w2_weight_scale_2=d["g2"], workspace=ws,
        shared_expert=_shared(fx, d, linear) if shared else None, scales_swizzled=not linear, **kw)


def _oracle(L, x, ids, wts, shared=True, act_round=True, **kw):
    sh = None
    if shared:
        sh = dict(w13=L.sh_w13.numpy()[0], s13=L.sh_s13.numpy()[0], g13=L.sh_g13.numpy(),
                  w2=L.sh_w2.numpy()[0], s2=L.sh_s2.numpy()[0], g2=L.sh_g2.numpy())
    return omoe.moe(x.float().numpy(), ids.numpy(), wts.numpy(), L.w13.numpy(), L.s13.numpy(),
                    L.g13.numpy(), L.w2.numpy(), L.s2.numpy(), L.g2.numpy(), shared=sh,
                    order="server", act_round=act_round, **kw)


@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("M", [1, 2, 4, 8, 16])
def test_config2_matches_oracle(M, fused):
    """Config 2 at full size (512 experts) at every M, one-launch and three-launch forms."""
    import flash_next_rtxpro6000_b200 as fx
    from flash_next_rtxpro6000_b200 import synthetic as syn

    E = 512
    L, d = _layer(E)
    x = syn.activations(M, seed=5)
    ids, wts = syn.routing(M, E=E, seed=M)
    ws = fx.make_workspace(num_routes=10, hidden_size=2048, intermediate_size=512, device=dev(),
                           fused=fused)
    y = _run(fx, d, x.to(dev()), ids.to(dev()), wts.to(dev()), ws)
    torch.cuda.synchronize()
    got = to_np(y)
    ref = _oracle(L, x, ids, wts)                 # act rounded to bf16 (the kernel's arithmetic)
    ref_dq = _oracle(L, x, ids, wts, act_round=False)
    assert y.shape == (M, 2048) and y.dtype == torch.bfloat16
    assert rel_err(got, ref) <= REL_TOL
    assert rel_err(got, ref_dq) <= REL_TOL
    l2 = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert l2 < 5e-3, l2
    assert int(ws.error_flag.item()) == 0


def test_negative_ids_are_skipped_and_no_shared():
    import flash_next_rtxpro6000_b200 as fx
    from flash_next_rtxpro6000_b200 import synthetic as syn

    L, d = _layer(64)
    M = 3
    x = syn.activations(M, seed=6)
    ids, wts = syn.routing(M, E=64, seed=6)
    ids[1, 3] = -1
    ids[1, 7] = -1
    ids[2, :] = -1
    ws = fx.make_workspace(num_routes=10, hidden_size=2048, intermediate_size=512, device=dev())
    y = _run(fx, d, x.to(dev()), ids.to(dev()), wts.to(dev()), ws, shared=False)
    ref = _oracle(L, x, ids, wts, shared=False)
    got = to_np(y)
    assert np.all(got[2] == 0)
    assert rel_err(got[:2], ref[:2]) <= REL_TOL


@pytest.mark.parametrize("path", ["auto", "fused"])
@pytest.mark.parametrize("M", [1, 16])
def test_deterministic_and_graph_replay(M, path):
    import flash_next_rtxpro6000_b200 as fx
    from flash_next_rtxpro6000_b200 import synthetic as syn

    L, d = _layer(512)
    x = syn.activations(M, seed=7).to(dev())
    ids, wts = syn.routing(M, E=512, seed=70 + M)
    ids, wts = ids.to(dev()), wts.to(dev())
    ws = fx.make_workspace(num_routes=10, hidden_size=2048, intermediate_size=512, device=dev())
    prev = fx.set_moe_path(path)
    try:
        _replay_checks(fx, syn, L, d, x, ids, wts, ws, M)
    finally:
        fx.set_moe_path(prev)


def _replay_checks(fx, syn, L, d, x, ids, wts, ws, M):
    a = _run(fx, d, x, ids, wts, ws).clone()
    b = _run(fx, d, x, ids, wts, ws).clone()
    assert torch.equal(a, b)
    # linear (unswizzled) scale layout gives the same bits as the swizzled one in the
    # general one-launch layer (the decode-width layer reads swizzled scales only)
    with fx.moe_path("fused"):
        a_f = _run(fx, d, x, ids, wts, ws).clone()
        c = _run(fx, d, x, ids, wts, ws, linear=True)
    assert torch.equal(a_f, c)
    xs, is_, ws_ = x.clone(), ids.clone(), wts.clone()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            _run(fx, d, xs, is_, ws_, ws)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        yg = _run(fx, d, xs, is_, ws_, ws)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(yg, a)
    x2 = syn.activations(M, seed=8)
    ids2, wts2 = syn.routing(M, E=512, seed=80 + M)
    xs.copy_(x2.to(dev()))
    is_.copy_(ids2.to(dev()))
    ws_.copy_(wts2.to(dev()))
    g.replay()
    torch.cuda.synchronize()
    ref2 = _oracle(L, x2, ids2, wts2)
    assert rel_err(to_np(yg), ref2) <= REL_TOL
    assert int(torch.count_nonzero(ws.counters)) == 0
    del g


def test_expert_slices_sum_to_layer():
    import flash_next_rtxpro6000_b200 as fx
    from flash_next_rtxpro6000_b200 import synthetic as syn

    L, d = _layer(64)
    M = 16
    x = syn.activations(M, seed=9).to(dev())
    ids, wts = syn.routing(M, E=64, seed=9)
    ids, wts = ids.to(dev()), wts.to(dev())
    ws = fx.make_workspace(num_routes=10, hidden_size=2048, intermediate_size=512, device=dev())
    full = _run(fx, d, x, ids, wts, ws, out_f32=True)
    total = torch.zeros_like(full)
    G = 4
    per = 64 // G
    for r in range(G):
        sl = slice(r * per, (r + 1) * per)
        part = fx.draft_moe_gemv(
            hidden_states=x, topk_ids=ids, topk_weights=wts, w13_weight=d["w13"][sl].contiguous(),
            w13_blockscale_swizzled=d["s13"][sl].contiguous(), w13_weight_scale_2=d["g13"][sl].contiguous(),
            w2_weight=d["w2"][sl].contiguous(), w2_blockscale_swizzled=d["s2"][sl].contiguous(),
            w2_weight_scale_2=d["g2"][sl].contiguous(), workspace=ws,
            shared_expert=_shared(fx, d) if r == 0 else None, expert_offset=r * per, out_f32=True)
        total += part
    assert rel_err(to_np(total), to_np(full)) <= 1e-5


def test_runner_maybe_apply_and_capture_guard():
    import types

    import flash_next_rtxpro6000_b200 as fx
    from flash_next_rtxpro6000_b200 import synthetic as syn

    L, d = _layer(64)
    layer = types.SimpleNamespace(layer_id=0, w13_weight=d["w13"], w13_blockscale_swizzled=d["s13"],
                                  w13_weight_scale_2=d["g13"], w2_weight=d["w2"],
                                  w2_blockscale_swizzled=d["s2"], w2_weight_scale_2=d["g2"])
    x = syn.activations(2, seed=4).to(dev())
    ids, wts = syn.routing(2, E=64, seed=4)
    disp = types.SimpleNamespace(hidden_states=x, hidden_states_scale=None,
                                 topk_output=types.SimpleNamespace(topk_ids=ids.to(dev()),
                                                                   topk_weights=wts.to(dev())))
    runner = fx.DraftMoeGemvRunner()
    out = runner.maybe_apply(layer=layer, dispatch_output=disp)
    ref = _oracle(L, x.cpu(), ids, wts, shared=False)
    assert rel_err(to_np(out.hidden_states), ref) <= REL_TOL
    big = types.SimpleNamespace(hidden_states=torch.zeros(17, 2048, dtype=torch.bfloat16, device=dev()),
                                hidden_states_scale=None, topk_output=disp.topk_output)
    assert runner.maybe_apply(layer=layer, dispatch_output=big) is None


@pytest.mark.parametrize("out_f32", [False, True])
def test_slice_without_routes_writes_zeros(out_f32):
    """An expert-parallel slice that no route reaches (and no shared expert) still
    writes its output: all zeros."""
    import flash_next_rtxpro6000_b200 as fx
    from flash_next_rtxpro6000_b200 import synthetic as syn

    L, d = _layer(64)
    M = 4
    x = syn.activations(M, seed=30).to(dev())
    ids, wts = syn.routing(M, E=32, seed=30)  # every id in [0, 32)
    ids, wts = ids.to(dev()), wts.to(dev())
    ws = fx.make_workspace(num_routes=10, hidden_size=2048, intermediate_size=512, device=dev())
    out = torch.full((M, 2048), 7.0, dtype=torch.float32 if out_f32 else torch.bfloat16,
                     device=dev())
    sl = slice(32, 64)
    fx.draft_moe_gemv(
        hidden_states=x, topk_ids=ids, topk_weights=wts, w13_weight=d["w13"][sl].contiguous(),
        w13_blockscale_swizzled=d["s13"][sl].contiguous(), w13_weight_scale_2=d["g13"][sl].contiguous(),
        w2_weight=d["w2"][sl].contiguous(), w2_blockscale_swizzled=d["s2"][sl].contiguous(),
        w2_weight_scale_2=d["g2"][sl].contiguous(), workspace=ws, expert_offset=32,
        out=out, out_f32=out_f32)
    torch.cuda.synchronize()
    assert int(torch.count_nonzero(out)) == 0


@pytest.mark.parametrize("M", [1, 16])
def test_reference_model_shape(M):
    """The reference model's MoE shape, H = 2560 and I = 640
    (bench/bench/moe_smallm/model_shapes.py:24-30), in both forms."""
    import flash_next_rtxpro6000_b200 as fx
    from flash_next_rtxpro6000_b200 import synthetic as syn

    L, d = _layer(64, H=2560, I=640, seed=1)
    x = syn.activations(M, K=2560, seed=11)
    ids, wts = syn.routing(M, E=64, seed=110 + M)
    ref = _oracle(L, x, ids, wts)
    for fused in (True, False):
        ws = fx.make_workspace(num_routes=10, hidden_size=2560, intermediate_size=640,
                               device=dev(), fused=fused)
        y = _run(fx, d, x.to(dev()), ids.to(dev()), wts.to(dev()), ws)
        torch.cuda.synchronize()
        assert rel_err(to_np(y), ref) <= REL_TOL, fused
        assert int(ws.error_flag.item()) == 0


@pytest.mark.parametrize("M", [1, 5, 16])
def test_crowded_and_repeated_routes(M):
    """Routings the reference's kernels accept but that overfill one MMA block: every
    token on the same few experts (up to 160 routes on one expert) and ids repeated
    within a row.  The one-launch form splits such experts and matches the oracle; the
    three-launch form reports FNX_DEVERR_ROUTES instead of dropping routes silently."""
    import flash_next_rtxpro6000_b200 as fx
    from flash_next_rtxpro6000_b200 import errors
    from flash_next_rtxpro6000_b200 import synthetic as syn

    L, d = _layer(64)
    x = syn.activations(M, seed=12)
    _, wts = syn.routing(M, E=64, seed=12)
    g = torch.Generator().manual_seed(M)
    cases = [torch.randint(0, 3, (M, 10), generator=g, dtype=torch.int32),  # 3 experts
             torch.full((M, 10), 7, dtype=torch.int32)]                     # one expert
    for ids in cases:
        ref = _oracle(L, x, ids, wts)
        ws = fx.make_workspace(num_routes=10, hidden_size=2048, intermediate_size=512,
                               device=dev())
        y = _run(fx, d, x.to(dev()), ids.to(dev()), wts.to(dev()), ws)
        torch.cuda.synchronize()
        assert rel_err(to_np(y), ref) <= REL_TOL
        errors.check_flag(ws.error_flag, "fused MoE")  # no error
        ws3 = fx.make_workspace(num_routes=10, hidden_size=2048, intermediate_size=512,
                                device=dev(), fused=False)
        y3 = _run(fx, d, x.to(dev()), ids.to(dev()), wts.to(dev()), ws3)
        torch.cuda.synchronize()
        crowd = int(torch.bincount(ids.reshape(-1).long()).max())
        if crowd > (16 if M > 8 else 8):  # more routes on one expert than one unit holds
            with pytest.raises(errors.DeviceWaitError) as ei:
                errors.check_flag(ws3.error_flag, "three-launch MoE")
            assert [c for _, c in ei.value.codes] == [9]
        else:
            errors.check_flag(ws3.error_flag, "three-launch MoE")
            assert rel_err(to_np(y3), ref) <= REL_TOL


def test_fused_counters_return_to_zero():
    """The one-launch layer leaves its counters at zero (graph replays need no memset)."""
    import flash_next_rtxpro6000_b200 as fx
    from flash_next_rtxpro6000_b200 import synthetic as syn

    L, d = _layer(512)
    ws = fx.make_workspace(num_routes=10, hidden_size=2048, intermediate_size=512, device=dev())
    for M in (1, 3, 16):
        x = syn.activations(M, seed=13 + M)
        ids, wts = syn.routing(M, E=512, seed=130 + M)
        _run(fx, d, x.to(dev()), ids.to(dev()), wts.to(dev()), ws)
        torch.cuda.synchronize()
        assert int(torch.count_nonzero(ws.counters)) == 0
        assert int(ws.error_flag.item()) == 0
