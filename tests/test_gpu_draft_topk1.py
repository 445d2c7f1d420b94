"""Greedy draft step (draft_topk1_postprocess, patches/sglang/series/0016-…patch:46-73)
and the draft head with the step fused into its argmax, on the GPU: the reference's own
test cases (test/srt/speculative/test_draft_fuse.py in that patch: hot vocabulary 32768,
batch 1 and 4, with and without the token map, draft_tokens column 1, positions + 1,
topk_p = 1), ties to the lowest column, bf16 logits, full-vocabulary widths, the fused
head against the oracle's argmax of its own bf16 logits, keys and counter left at zero,
and graph replay advancing positions once per replay."""

import numpy as np
import pytest
import torch

from oracle import w8a16 as ow8
from tests.gpu_util import dev

pytestmark = pytest.mark.gpu


def _fx():
    import flash_next_rtxpro6000_b200 as fx

    return fx


def _ws_clear():
    from flash_next_rtxpro6000_b200.w8a16_gemv import _workspace

    ws = _workspace(dev())
    torch.cuda.synchronize()
    return int(ws.argmax_keys.abs().sum()) == 0 and int(ws.argmax_count.item()) == 0


@pytest.mark.parametrize("batch_size", [1, 4])
@pytest.mark.parametrize("use_token_map", [False, True])
def test_reference_case(batch_size, use_token_map):
    fx = _fx()
    d = dev()
    hot = 32768
    g = torch.Generator(device=d).manual_seed(1234 + batch_size)
    logits = torch.randn((batch_size, hot), dtype=torch.float32, device=d, generator=g)
    idx = torch.randint(hot, (batch_size, 1), device=d, generator=g)
    logits.scatter_(1, idx, 1000.0)
    expected_hot = torch.argmax(logits, dim=-1, keepdim=True)
    hot_token_id = None
    expected = expected_hot
    if use_token_map:
        hot_token_id = torch.randperm(hot, device=d, generator=g, dtype=torch.int64) + 100_000
        expected = hot_token_id[expected_hot]
    positions = torch.arange(batch_size, device=d, dtype=torch.int64)
    expected_positions = positions + 1
    draft_tokens = torch.full((batch_size, 3), -1, device=d, dtype=torch.int64)
    topk_p, topk_index = fx.draft_topk1_postprocess(logits, positions, draft_tokens,
                                                    draft_token_column=1,
                                                    hot_token_id=hot_token_id)
    assert torch.equal(topk_index, expected)
    assert torch.equal(draft_tokens[:, 1:2], expected)
    assert torch.equal(draft_tokens[:, 0], torch.full_like(positions, -1))
    assert torch.equal(draft_tokens[:, 2], torch.full_like(positions, -1))
    assert torch.equal(topk_p, torch.ones_like(topk_p))
    assert torch.equal(positions, expected_positions)
    assert _ws_clear()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,V", [(1, 151936), (16, 248320), (5, 49152), (3, 1000)])
def test_matches_oracle_with_ties(dtype, B, V):
    fx = _fx()
    d = dev()
    g = torch.Generator().manual_seed(B * 7 + V)
    logits = (torch.randint(-40, 41, (B, V), generator=g).float() / 8).to(dtype)  # many ties
    hot = torch.randperm(V, generator=g, dtype=torch.int64) * 3 + 7
    pos = torch.randint(0, 1000, (B,), generator=g, dtype=torch.int64)
    dt = torch.full((B, 4), -5, dtype=torch.int64)
    p, ti = fx.draft_topk1_postprocess(logits.to(d), pos.to(d).clone(), None, 0, hot.to(d))
    op, oti, _, _ = ow8.draft_topk1(logits.float().numpy(), pos.numpy(), dt.numpy(), 2,
                                    hot.numpy())
    assert np.array_equal(ti.cpu().numpy(), oti)
    pd = pos.to(d).clone()
    dtd = dt.to(d)
    fx.draft_topk1_postprocess(logits.to(d), pd, dtd, 2, None)
    _, oti2, opos, odt = ow8.draft_topk1(logits.float().numpy(), pos.numpy(), dt.numpy(), 2)
    assert np.array_equal(dtd.cpu().numpy(), odt)
    assert np.array_equal(pd.cpu().numpy(), opos)
    assert _ws_clear()


@pytest.mark.parametrize("M", [1, 4, 16])
def test_fused_draft_head(M):
    fx = _fx()
    from flash_next_rtxpro6000_b200 import synthetic as syn

    d = dev()
    V, K = 49152, 2048
    head = syn.w8_head(V, K, seed=9)
    w, s = head.w.to(d), head.scale.to(d)
    x = syn.activations(M, seed=10).to(d)
    g = torch.Generator().manual_seed(M)
    hot = (torch.randperm(V, generator=g, dtype=torch.int64) + 17).to(d)
    pos = torch.arange(M, dtype=torch.int64, device=d) * 3
    dt = torch.full((M, 5), -1, dtype=torch.int64, device=d)
    logits = torch.empty(M, V, dtype=torch.bfloat16, device=d)
    p, ti = fx.draft_head_topk1(x, w, s, pos, dt, 4, hot, out=logits)
    torch.cuda.synchronize()
    _, oti, _, _ = ow8.draft_topk1(logits.float().cpu().numpy(), np.zeros(M), None, 0,
                                   hot.cpu().numpy())
    assert np.array_equal(ti.cpu().numpy(), oti)
    assert torch.equal(dt[:, 4:5], ti) and torch.equal(p, torch.ones_like(p))
    assert torch.equal(pos, torch.arange(M, dtype=torch.int64, device=d) * 3 + 1)
    # same token as the plain GEMV's fused argmax, mapped
    # (the fused draft step runs the mma.sync form at every M, so the plain call does too)
    am = torch.empty(M, dtype=torch.int64, device=d)
    with fx.dense_path("mma"):
        y = fx.w8a16_gemv(x, w, s, argmax_out=am)
    assert torch.equal(y, logits) and torch.equal(hot[am].view(M, 1), ti)
    assert _ws_clear()


def test_graph_replay_advances_positions():
    fx = _fx()
    from flash_next_rtxpro6000_b200 import synthetic as syn

    d = dev()
    M, V, K = 4, 49152, 2048
    head = syn.w8_head(V, K, seed=11)
    w, s = head.w.to(d), head.scale.to(d)
    x = syn.activations(M, seed=12).to(d)
    pos = torch.zeros(M, dtype=torch.int64, device=d)
    ref_p, ref_t = fx.draft_head_topk1(x, w, s, pos)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fx.draft_head_topk1(x, w, s, pos)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        gp, gt = fx.draft_head_topk1(x, w, s, pos)
    torch.cuda.synchronize()
    start = pos.clone()
    for i in range(3):
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(gt, ref_t)
        assert torch.equal(pos, start + i + 1)
    assert _ws_clear()
