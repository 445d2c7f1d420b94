"""Decode-step stack (config 3) on the GPU: MoE layers chained through one CUDA graph,
ending in the int8 lm_head with greedy argmax.

Parity is teacher-forced layer by layer: each layer's GPU output is compared with the
CPU oracle fed the same GPU input, within 2e-2 relative error; the greedy tokens of the
head must be bit-exact against the oracle on the stack's final hidden state.  A second
replay of the graph must reproduce every intermediate bit for bit."""

import numpy as np
import pytest
import torch

from oracle import moe as omoe, nvfp4 as onv, w8a16 as ow8
from tests.gpu_util import REL_TOL, dev, rel_err, to_np

pytestmark = pytest.mark.gpu


def _device_layer(L):
    d = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev()) for k, v in dict(
        w13=L.w13.numpy(), s13=onv.swizzle_blockscale(L.s13.numpy()), g13=L.g13.numpy(),
        w2=L.w2.numpy(), s2=onv.swizzle_blockscale(L.s2.numpy()), g2=L.g2.numpy(),
        sw13=L.sh_w13.numpy(), ss13=onv.swizzle_blockscale(L.sh_s13.numpy()),
        sg13=L.sh_g13.numpy(), sw2=L.sh_w2.numpy(), ss2=onv.swizzle_blockscale(L.sh_s2.numpy()),
        sg2=L.sh_g2.numpy()).items()}
    return d


def _oracle_layer(L, x, ids, wts):
    sh = dict(w13=L.sh_w13.numpy()[0], s13=L.sh_s13.numpy()[0], g13=L.sh_g13.numpy(),
              w2=L.sh_w2.numpy()[0], s2=L.sh_s2.numpy()[0], g2=L.sh_g2.numpy())
    return omoe.moe(x, ids.numpy(), wts.numpy(), L.w13.numpy(), L.s13.numpy(), L.g13.numpy(),
                    L.w2.numpy(), L.s2.numpy(), L.g2.numpy(), shared=sh, order="server",
                    act_round=True)


@pytest.mark.parametrize("M", [1, 4, 16])
def test_stack_chained_matches_oracle(M):
    import flash_next_rtxpro6000_b200 as fx
    from flash_next_rtxpro6000_b200 import synthetic as syn

    n_layers, E, V = 3, 64, 16384
    Ls = [syn.moe_layer(E, syn.HIDDEN, syn.INTER, seed=10 + i) for i in range(n_layers)]
    ds = [_device_layer(L) for L in Ls]
    routes = [syn.routing(M, E=E, seed=200 + 10 * M + i) for i in range(n_layers)]
    droutes = [(ids.to(dev()), wts.to(dev())) for ids, wts in routes]
    head = syn.w8_head(V, syn.HIDDEN, seed=3)
    hw, hs = head.w.to(dev()), head.scale.to(dev())
    ws = fx.make_workspace(num_routes=10, hidden_size=syn.HIDDEN, intermediate_size=syn.INTER,
                           device=dev())
    hidden = [syn.activations(M, seed=7).to(dev())] + [
        torch.empty(M, syn.HIDDEN, dtype=torch.bfloat16, device=dev()) for _ in range(n_layers)]
    logits = torch.empty(M, V, dtype=torch.bfloat16, device=dev())
    am = torch.empty(M, dtype=torch.int64, device=dev())
    cfg = fx.DraftMoeGemvConfig(pdl=True)

    def step():
        for i, d in enumerate(ds):
            fx.draft_moe_gemv(
                hidden_states=hidden[i], topk_ids=droutes[i][0], topk_weights=droutes[i][1],
                w13_weight=d["w13"], w13_blockscale_swizzled=d["s13"],
                w13_weight_scale_2=d["g13"], w2_weight=d["w2"], w2_blockscale_swizzled=d["s2"],
                w2_weight_scale_2=d["g2"], workspace=ws,
                shared_expert=fx.SharedExpert(d["sw13"], d["ss13"], d["sg13"], d["sw2"],
                                              d["ss2"], d["sg2"]),
                out=hidden[i + 1], cfg=cfg)
        fx.w8a16_gemv(hidden[n_layers], hw, hs, out=logits, argmax_out=am, pdl=True)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()  # warm-up outside the capture
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for t in hidden[1:] + [logits]:
        t.zero_()
    g.replay()
    torch.cuda.synchronize()
    first = [to_np(t) for t in hidden] + [to_np(logits)]
    first_am = am.cpu().numpy().copy()

    for i, L in enumerate(Ls):
        xin = to_np(hidden[i])
        ref = _oracle_layer(L, xin, *routes[i])
        got = to_np(hidden[i + 1])
        assert np.isfinite(got).all()
        assert rel_err(got, ref) <= REL_TOL, f"layer {i}: rel err {rel_err(got, ref)}"

    ref_logits = ow8.gemv(to_np(hidden[n_layers]), head.w.numpy(), "int8",
                          head.scale.float().numpy())
    assert rel_err(to_np(logits), ref_logits) <= REL_TOL
    np.testing.assert_array_equal(first_am, ow8.argmax_lowest(ref_logits))
    np.testing.assert_array_equal(first_am, ow8.argmax_lowest(to_np(logits)))

    g.replay()
    torch.cuda.synchronize()
    again = [to_np(t) for t in hidden] + [to_np(logits)]
    for a, b in zip(first, again):
        np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(first_am, am.cpu().numpy())
    del g
