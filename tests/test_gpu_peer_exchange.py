"""The in-kernel greedy-key exchange of the vocab-sharded lm_head on one GPU (a one-rank
exchange with itself: the key stores, the epoch flag and the bounded wait all run): the
greedy tokens and logits equal the plain GEMV's over several calls in a row and inside a
CUDA graph, and no wait expires.  The 2-GPU form is in test_gpu_sharded.py."""

import pytest
import torch

from tests.gpu_util import dev

pytestmark = pytest.mark.gpu


def test_one_rank_exchange_matches_plain_argmax():
    import flash_next_rtxpro6000_b200 as fx
    from flash_next_rtxpro6000_b200 import sharded
    from flash_next_rtxpro6000_b200 import synthetic as syn
    from flash_next_rtxpro6000_b200.w8a16_gemv import _workspace

    d = dev()
    head = syn.w8_head(16384, 2048, seed=21)
    w, s = head.w.to(d), head.scale.to(d)
    ex = sharded.PeerExchange(d)
    try:
        for rep, M in enumerate((1, 4, 16, 3, 16)):
            x = syn.activations(M, seed=30 + rep).to(d)
            y, am = sharded.vocab_sharded_lm_head(x, w, s, 0, ex)
            ref_am = torch.empty(M, dtype=torch.int64, device=d)
            ref_y = fx.w8a16_gemv(x, w, s, argmax_out=ref_am)
            assert torch.equal(am, ref_am) and torch.equal(y, ref_y)
        x = syn.activations(4, seed=40).to(d)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            sharded.vocab_sharded_lm_head(x, w, s, 0, ex)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            _, gam = sharded.vocab_sharded_lm_head(x, w, s, 0, ex)
        ref_am = torch.empty(4, dtype=torch.int64, device=d)
        fx.w8a16_gemv(x, w, s, argmax_out=ref_am)
        for _ in range(3):
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(gam, ref_am)
        assert int(_workspace(d).error_flag.item()) == 0
    finally:
        ex.close()
