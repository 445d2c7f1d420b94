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


def test_peer_that_never_arrives_and_desync_are_reported():
    """A rank whose peer never publishes: the bounded wait runs out (limit set to 50 ms),
    FNX_DEVERR_WAIT_PEER is recorded, the call completes and returns this rank's own token;
    check_flag raises and clears the flag.  Then a peer that appears two calls ahead is
    reported as FNX_DEVERR_PEER_DESYNC at once (no wait), again with the own token.  No
    fault: the missing peer is a second local buffer that nothing writes."""
    import ctypes
    import time

    import flash_next_rtxpro6000_b200 as fx
    from flash_next_rtxpro6000_b200 import _lib, errors
    from flash_next_rtxpro6000_b200 import synthetic as syn
    from flash_next_rtxpro6000_b200.w8a16_gemv import _workspace

    d = dev()
    lib = _lib.lib()
    head = syn.w8_head(8192, 2048, seed=22)
    w, s = head.w.to(d), head.scale.to(d)
    b0 = torch.zeros(_lib.PEER_BUFFER_BYTES, dtype=torch.uint8, device=d)  # this rank
    b1 = torch.zeros(_lib.PEER_BUFFER_BYTES, dtype=torch.uint8, device=d)  # silent "rank 1"
    bufs = (ctypes.c_void_p * 2)(b0.data_ptr(), b1.data_ptr())
    _lib.check(lib.fnx_peer_setup(b0.data_ptr(), bufs, 2, 0), "fnx_peer_setup")
    _lib.check(lib.fnx_peer_set_wait_limit(b0.data_ptr(), 50_000_000), "wait limit")
    ws = _workspace(d)
    ws.error_flag.zero_()
    stream = torch.cuda.current_stream(d).cuda_stream

    def call(M, seed):
        x = syn.activations(M, seed=seed).to(d)
        y = torch.empty(M, w.shape[0], dtype=torch.bfloat16, device=d)
        am = torch.full((M,), -1, dtype=torch.int64, device=d)
        rc = lib.fnx_w8a16_gemv_vocab_sharded(
            x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), _lib.W_INT8, s.data_ptr(),
            _lib.SCALE_BF16_ROW, y.data_ptr(), y.stride(0), 0, am.data_ptr(), 0, M, w.shape[0],
            2048, b0.data_ptr(), None, ctypes.byref(ws.c), 1, stream)
        _lib.check(rc, "vocab_sharded")
        ref = torch.empty(M, dtype=torch.int64, device=d)
        fx.w8a16_gemv(x, w, s, argmax_out=ref)
        return am, ref

    t0 = time.perf_counter()
    am, ref = call(4, 50)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 1.5  # the 50 ms limit, not the 2 s default
    with pytest.raises(errors.DeviceWaitError) as ei:
        errors.check_flag(ws.error_flag, "vocab_sharded")
    assert [c for _, c in ei.value.codes] == [7]
    assert int(ws.error_flag.item()) == 0
    assert torch.equal(am, ref)  # the rank's own shard's token (here the whole head)
    epoch = b0[2560:2564].view(torch.int32)
    assert int(epoch.item()) == 1
    # "rank 1" now shows epoch 4 on every token: two or more calls ahead of call 2
    b0[2048:2560].view(torch.int32).view(8, 16)[1].fill_(4)
    t0 = time.perf_counter()
    am, ref = call(16, 51)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 1.0
    with pytest.raises(errors.DeviceWaitError) as ei:
        errors.check_flag(ws.error_flag, "vocab_sharded")
    assert [c for _, c in ei.value.codes] == [8]
    assert torch.equal(am, ref)
    assert int(epoch.item()) == 2
    ws.error_flag.zero_()
