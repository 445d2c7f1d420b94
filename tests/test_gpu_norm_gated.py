"""Fused gated-RMSNorm W8A16 GEMV (w8a16_gemv_norm_gated) on the GPU against the CPU
oracle: the reference's h1 shape (out_proj of the gated-delta block: N = 2560,
K = 48 x 128, group 128), both gates, M in 1..16, int8 / fp8 / bf16 weights, bf16 and
fp32 norm weights, fp32 destination, split-K tilings; the reference's bar is 2e-2
relative error (kernels/microbench/h1/h1_check.py:105-130 compares against the unfused
rms_norm_gated + w8a16_gemv in bf16 ulps)."""

import numpy as np
import pytest
import torch

from oracle import w8a16 as ow8
from tests.gpu_util import REL_TOL, dev, rel_err, to_np, ulps

pytestmark = pytest.mark.gpu


def _fx():
    import flash_next_rtxpro6000_b200 as fx

    return fx


def _case(N, K, M, G, kind, seed, nw_dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(M, K, generator=g) * 0.5).bfloat16()
    z = (torch.randn(M, K, generator=g) * 0.5).bfloat16()
    nw = (torch.randn(G, generator=g) * 0.3 + 1.0).to(nw_dtype)
    if kind == "int8":
        w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
        w_np = w.numpy()
        s = (torch.randn(N, generator=g).abs() / 127).float()
    elif kind == "fp8":
        w = (torch.randn(N, K, generator=g) * 64).to(torch.float8_e4m3fn)
        w_np = w.view(torch.uint8).numpy()
        s = (torch.randn(N, generator=g).abs() / 448).float()
    else:
        w = (torch.randn(N, K, generator=g) * 0.02).bfloat16()
        w_np = w.float().numpy()
        s = torch.ones(1, dtype=torch.float32)
    return x, z, nw, w, s, w_np


def _oracle(x, z, nw, G, w_np, kind, s, sigmoid):
    return ow8.gemv_norm_gated(x.float().numpy(), z.float().numpy(), nw.float().numpy(), G,
                               1e-6, w_np, kind, s.float().numpy(), sigmoid_gate=sigmoid)


def _check(got, ref):
    assert rel_err(got, ref) <= REL_TOL
    # The normalised row is rounded to bf16 before the dot: where the oracle's fp32 value
    # sits on a rounding boundary one element can move by a bf16 step, which moves the
    # logits by far less than their own step.
    u = ulps(got, ref)
    big = np.abs(ref) >= 1e-2 * np.abs(ref).max()
    assert u[big].max() <= 2 and (u == 0).mean() > 0.9


@pytest.mark.parametrize("sigmoid", [True, False])
@pytest.mark.parametrize("M", [1, 2, 4, 9, 16])
@pytest.mark.parametrize("kind", ["fp8", "int8"])
def test_h1_shape_matches_oracle(kind, M, sigmoid):
    fx = _fx()
    N, K, G = 2560, 48 * 128, 128
    x, z, nw, w, s, w_np = _case(N, K, M, G, kind, seed=M * 7 + int(sigmoid))
    d = dev()
    y = fx.w8a16_gemv_norm_gated(x.to(d), w.to(d), s.to(d), z.to(d), nw.to(d), G, 1e-6,
                                 sigmoid_gate=sigmoid)
    torch.cuda.synchronize()
    assert y.shape == (M, N) and y.dtype == torch.bfloat16
    _check(to_np(y), _oracle(x, z, nw, G, w_np, kind, s, sigmoid))


@pytest.mark.parametrize("G", [8, 16, 32, 64, 256])
@pytest.mark.parametrize("M", [1, 5, 16])
def test_group_sizes(G, M):
    fx = _fx()
    N, K = 1000, 1024
    x, z, nw, w, s, w_np = _case(N, K, M, G, "fp8", seed=G + M)
    d = dev()
    y = fx.w8a16_gemv_norm_gated(x.to(d), w.to(d), s.to(d), z.to(d), nw.to(d), G, 1e-6)
    _check(to_np(y), _oracle(x, z, nw, G, w_np, "fp8", s, False))


@pytest.mark.parametrize("M", [1, 4, 16])
def test_fp32_norm_weight_bf16_weight_and_fp32_out(M):
    fx = _fx()
    N, K, G = 768, 2048, 128
    d = dev()
    x, z, nw, w, s, w_np = _case(N, K, M, G, "fp8", seed=3, nw_dtype=torch.float32)
    y16 = fx.w8a16_gemv_norm_gated(x.to(d), w.to(d), s.to(d), z.to(d), nw.to(d), G, 1e-6)
    _check(to_np(y16), _oracle(x, z, nw, G, w_np, "fp8", s, False))
    buf = torch.full((M, N), float("nan"), device=d)
    y32 = fx.w8a16_gemv_norm_gated(x.to(d), w.to(d), s.to(d), z.to(d), nw.to(d), G, 1e-6,
                                   out=buf)
    assert y32 is buf and torch.equal(y32, y16.float())
    x, z, nw, w, s, w_np = _case(N, K, M, G, "bf16", seed=4)
    yb = fx.w8a16_gemv_norm_gated(x.to(d), w.to(d), s.to(d), z.to(d), nw.to(d), G, 1e-6,
                                  sigmoid_gate=True)
    _check(to_np(yb), _oracle(x, z, nw, G, w_np, "bf16", s, True))


@pytest.mark.parametrize("M", [1, 16])
def test_split_k_tilings_agree(M):
    fx = _fx()
    N, K, G = 1280, 2048, 128
    x, z, nw, w, s, w_np = _case(N, K, M, G, "int8", seed=11)
    d = dev()
    args = (x.to(d), w.to(d), s.to(d), z.to(d), nw.to(d), G, 1e-6)
    ref = _oracle(x, z, nw, G, w_np, "int8", s, False)
    base = fx.w8a16_gemv_norm_gated(*args, cfg=fx.GemvConfig(16, 2, 1, 1))
    _check(to_np(base), ref)
    for cfg in ((8, 2, 1, 2), (8, 1, 1, 4)):  # 32 chunks of 64 k each way
        got = fx.w8a16_gemv_norm_gated(*args, cfg=fx.GemvConfig(*cfg))
        assert rel_err(to_np(got), to_np(base)) <= REL_TOL
        _check(to_np(got), ref)


def test_strided_rows_and_zero_rows():
    # rows taken from wider buffers (ldx, ldz > K) and an all-zero row (rstd = 1/sqrt(eps),
    # normalised row 0): the logits of that row are exactly 0
    fx = _fx()
    M, N, K, G = 3, 512, 1024, 128
    x, z, nw, w, s, w_np = _case(N, K, M, G, "fp8", seed=21)
    x[1] = 0
    d = dev()
    xb = torch.zeros(M, K + 64, dtype=torch.bfloat16, device=d)
    zb = torch.zeros(M, K + 128, dtype=torch.bfloat16, device=d)
    xb[:, :K] = x.to(d)
    zb[:, :K] = z.to(d)
    y = fx.w8a16_gemv_norm_gated(xb[:, :K], w.to(d), s.to(d), zb[:, :K], nw.to(d), G, 1e-6)
    got = to_np(y)
    assert np.all(got[1] == 0)
    _check(got, _oracle(x, z, nw, G, w_np, "fp8", s, False))


def test_unsupported_group_and_bad_arguments():
    fx = _fx()
    d = dev()
    x, z, nw, w, s, _ = _case(256, 384, 2, 96, "fp8", seed=5)
    x, z, nw, w, s = x.to(d), z.to(d), nw.to(d), w.to(d), s.to(d)
    assert not fx.w8a16_gemv_norm_gated_supported(x, w, s, z, nw, 96)
    with pytest.raises(NotImplementedError):
        fx.w8a16_gemv_norm_gated(x, w, s, z, nw, 96, 1e-6)
    assert not fx.w8a16_gemv_norm_gated_supported(x, w, s, z, nw, 128)  # 96 norm weights
    assert fx.w8a16_gemv_norm_gated_supported(x, w, s, z, nw.new_ones(128), 128)
    with pytest.raises(ValueError):
        fx.w8a16_gemv_norm_gated(x, w, s, z[:, :128], nw, 96, 1e-6)
    with pytest.raises(ValueError):
        fx.w8a16_gemv_norm_gated(x, w, s, z, nw[:64], 96, 1e-6)


@pytest.mark.parametrize("G", [128, 256])
def test_split_k_slice_staging_and_full_row_fallback(G):
    # 16 k splits of 128 columns: with G = 128 each CTA stages (and normalises) only its
    # split; with G = 256 a group would straddle two splits, so full rows are staged.
    # A grid that is not a multiple of the splits also falls back to full rows.
    fx = _fx()
    M, N, K = 4, 640, 2048
    x, z, nw, w, s, w_np = _case(N, K, M, G, "fp8", seed=G)
    d = dev()
    args = (x.to(d), w.to(d), s.to(d), z.to(d), nw.to(d), G, 1e-6)
    ref = _oracle(x, z, nw, G, w_np, "fp8", s, False)
    for cfg in ((2, 1, 1, 16), (2, 1, 1, 16, 37), (2, 1, 1, 16, 48)):
        _check(to_np(fx.w8a16_gemv_norm_gated(*args, cfg=fx.GemvConfig(*cfg))), ref)
