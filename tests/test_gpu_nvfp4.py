"""NVFP4 W4A16 GEMV on the GPU against the CPU oracle, plus the reference's numerics
checks (kernels/microbench/n1/check_nvfp4_gemv.py): bit-exact one-hot decode of every
code, GEMV within 2e-2 of the dequantise-then-matmul path (config 0: 4096 x 2048),
per-row global scales, split-K agreement, graph replay."""

import numpy as np
import pytest
import torch

from oracle import numerics, nvfp4 as onv
from tests.gpu_util import REL_TOL, dev, rel_err, to_np, ulps

pytestmark = pytest.mark.gpu


def _fx():
    import flash_next_rtxpro6000_b200 as fx

    return fx


@pytest.mark.parametrize("M", [1, 2, 4, 8, 16])
def test_config0_matches_oracle(M):
    fx = _fx()
    from flash_next_rtxpro6000_b200 import synthetic as syn

    x, w = syn.config0(M=M, seed=0)
    y = fx.w4a16_nvfp4_gemv(x.to(dev()), w.wq.to(dev()), w.bs.to(dev()), w.gscale.to(dev()))
    torch.cuda.synchronize()
    ref = onv.gemv(x.float().numpy(), w.wq.numpy(), w.bs.numpy(), w.gscale.numpy())
    got = to_np(y)
    assert y.shape == (M, 4096) and y.dtype == torch.bfloat16
    assert rel_err(got, ref) <= REL_TOL
    u = ulps(got, ref)
    assert u.max() <= 2 and (u == 0).mean() > 0.97


@pytest.mark.parametrize("N,K", [(1000, 2048), (2048, 512), (4096, 4096)])
@pytest.mark.parametrize("per_row", [False, True])
def test_quantized_weight_matches_oracle(N, K, per_row):
    fx = _fx()
    g = torch.Generator().manual_seed(N + K)
    w = (torch.randn(N, K, generator=g) * 0.02).bfloat16()
    wq, bs, gs = onv.quantize(w.float().numpy())
    if per_row:
        gs = (np.abs(np.random.default_rng(0).standard_normal(N)) * gs[0] + 1e-6).astype(np.float32)
    x = torch.randn(4, K, generator=g).bfloat16()
    y = fx.w4a16_nvfp4_gemv(x.to(dev()), torch.from_numpy(wq).to(dev()),
                            torch.from_numpy(bs).to(dev()), torch.from_numpy(gs).to(dev()))
    ref = onv.gemv(x.float().numpy(), wq, bs, gs)
    assert rel_err(to_np(y), ref) <= REL_TOL


def test_one_hot_decode_is_bit_exact():
    # check_nvfp4_gemv.py:92-111: y[0, n] must equal bf16(deq[n, k0]) for one-hot x
    fx = _fx()
    N, K = 256, 2560 - 2560 % 128
    g = torch.Generator().manual_seed(0)
    w = (torch.randn(N, K, generator=g) * 0.05).bfloat16()
    wq, bs, gs = onv.quantize(w.float().numpy())
    deq = onv.dequantize(wq, bs, gs)
    wq_d, bs_d, gs_d = (torch.from_numpy(a).to(dev()) for a in (wq, bs, gs))
    bad = 0
    for k0 in list(range(16)) + [16, 17, 31, 100, 1279, K - 1]:
        x = torch.zeros(1, K, dtype=torch.bfloat16)
        x[0, k0] = 1.0
        y = to_np(fx.w4a16_nvfp4_gemv(x.to(dev()), wq_d, bs_d, gs_d))[0]
        want = numerics.bf16_round(deq[:, k0])
        bad += int((y != want).sum())
    assert bad == 0


def test_every_code_and_scale_decodes_exactly():
    # all 16 codes x a spread of e4m3 scales, one-hot activations
    fx = _fx()
    K = 128
    codes = np.tile(np.arange(16, dtype=np.uint8), K // 16)
    scales = np.array([0x01, 0x07, 0x08, 0x30, 0x38, 0x40, 0x6F, 0x7E, 0x1A, 0x55], np.uint8)
    N = scales.size
    wq = np.stack([onv.pack_codes(codes)] * N)
    bs = np.repeat(scales[:, None], K // 16, axis=1)
    gs = np.array([1.0], np.float32)
    deq = onv.dequantize(wq, bs, gs)
    for k0 in range(16):
        x = torch.zeros(1, K, dtype=torch.bfloat16)
        x[0, k0] = 1.0
        y = to_np(fx.w4a16_nvfp4_gemv(x.to(dev()), torch.from_numpy(wq).to(dev()),
                                      torch.from_numpy(bs).to(dev()), torch.from_numpy(gs).to(dev())))
        assert np.array_equal(y[0], numerics.bf16_round(deq[:, k0])), k0


@pytest.mark.parametrize("M", [1, 16])
def test_split_k_and_graph_replay(M):
    fx = _fx()
    from flash_next_rtxpro6000_b200 import synthetic as syn

    x, w = syn.config0(M=M, seed=2)
    wq, bs, gs = w.wq.to(dev()), w.bs.to(dev()), w.gscale.to(dev())
    xs = x.to(dev()).clone()
    ref = onv.gemv(x.float().numpy(), w.wq.numpy(), w.bs.numpy(), w.gscale.numpy())
    outs = []
    for cfg in (fx.GemvConfig(16, 1, 1, 1), fx.GemvConfig(8, 1, 1, 2), fx.GemvConfig(8, 2, 1, 1)):
        y = fx.w4a16_nvfp4_gemv(xs, wq, bs, gs, cfg=cfg)
        assert rel_err(to_np(y), ref) <= REL_TOL
        outs.append(y)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            fx.w4a16_nvfp4_gemv(xs, wq, bs, gs)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        yg = fx.w4a16_nvfp4_gemv(xs, wq, bs, gs)
    gr.replay()
    torch.cuda.synchronize()
    first = yg.clone()
    gr.replay()
    torch.cuda.synchronize()
    assert torch.equal(first, yg)
    assert rel_err(to_np(yg), ref) <= REL_TOL


@pytest.mark.parametrize("M", [1, 4, 16])
def test_nvfp4_head_argmax(M):
    fx = _fx()
    g = torch.Generator().manual_seed(M)
    N, K = 32768, 2048
    wq = torch.randint(0, 256, (N, K // 2), generator=g, dtype=torch.uint8)
    bs = (torch.randn(N, K // 16, generator=g).abs() * 0.5).to(torch.float8_e4m3fn).view(torch.uint8)
    gs = torch.tensor([1 / 448.0])
    x = torch.randn(M, K, generator=g).bfloat16()
    am = torch.empty(M, dtype=torch.int64, device=dev())
    y = fx.w4a16_nvfp4_gemv(x.to(dev()), wq.to(dev()), bs.to(dev()), gs.to(dev()), argmax_out=am)
    ref = onv.gemv(x.float().numpy(), wq.numpy(), bs.numpy(), gs.numpy())
    assert rel_err(to_np(y), ref) <= REL_TOL
    assert am.cpu().numpy().tolist() == np.argmax(ref, axis=-1).tolist()


def test_quantize_nvfp4_on_device_matches_oracle():
    fx = _fx()
    g = torch.Generator().manual_seed(9)
    w = (torch.randn(300, 512, generator=g) * 0.3).bfloat16()
    wq, bs, gs = fx.quantize_nvfp4(w.to(dev()))
    owq, obs, ogs = onv.quantize(w.float().numpy())
    assert np.array_equal(wq.cpu().numpy(), owq)
    assert np.array_equal(bs.cpu().numpy(), obs)
    assert np.array_equal(gs.cpu().numpy(), ogs)
    deq = fx.dequantize_nvfp4(wq, bs, gs)
    assert np.array_equal(deq.cpu().numpy(), onv.dequantize(owq, obs, ogs))


@pytest.mark.parametrize("case", ["randn", "allcodes", "zero_blocks", "ties", "row_spread"])
def test_quantize_kernel_matches_reference_golden(case):
    """The GPU codec against the reference's own quantize_nvfp4 / dequantize_nvfp4 outputs
    (tests/golden/nvfp4_codec.npz, made by tests/golden/make_golden.py): codes, block
    scales and global scale bit for bit (ties, all-zero blocks, every code, rows spanning
    five decades), dequantisation bit for bit, from bf16 and from fp32 input."""
    import os

    fx = _fx()
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "nvfp4_codec.npz"))
    w = torch.from_numpy(g[f"{case}_w"])
    for src in (w.bfloat16(), w):  # the golden inputs are bf16 values stored as fp32
        wq, bs, gs = fx.quantize_nvfp4(src.to(dev()))
        assert np.array_equal(wq.cpu().numpy(), g[f"{case}_wq"])
        assert np.array_equal(bs.cpu().numpy(), g[f"{case}_bs"])
        assert np.array_equal(gs.cpu().numpy().reshape(-1), g[f"{case}_gscale"].reshape(-1))
        deq = fx.dequantize_nvfp4(wq, bs, gs)
        assert np.array_equal(deq.cpu().numpy().view(np.uint32), g[f"{case}_deq"].view(np.uint32))
        deq16 = fx.dequantize_nvfp4(wq, bs, gs, dtype=torch.bfloat16)
        assert torch.equal(deq16.cpu(), torch.from_numpy(g[f"{case}_deq"]).bfloat16())
