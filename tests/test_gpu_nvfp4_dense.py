"""NVFP4DenseLinearMethod on the GPU (the reference's nvfp4_dense.py serving class,
patches/sglang/series/0095-…patch:200-260): apply at M <= 16 through the NVFP4 GEMV
against the oracle, apply_into the shared fp32 buffer (bf16 values widened, identical to
apply) and its declines, and the wide-M path (dequantise in row chunks + GEMM) within the
2e-2 bar of the dequantise-then-matmul oracle."""

import types

import numpy as np
import pytest
import torch

from oracle import nvfp4 as onv
from tests.gpu_util import REL_TOL, dev, rel_err, to_np

pytestmark = pytest.mark.gpu


def _layer(N=20000, K=2048, seed=0):
    from flash_next_rtxpro6000_b200 import nvfp4_dense as nd
    from flash_next_rtxpro6000_b200.w4a16_nvfp4_gemv import quantize_nvfp4

    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(N, K, generator=g) * 0.02).bfloat16()
    wq, bs, gs = quantize_nvfp4(w.to(dev()))
    layer = types.SimpleNamespace()
    nd.NVFP4DenseLinearMethod.attach(layer, wq, bs, gs)
    return nd.NVFP4DenseLinearMethod(), layer


@pytest.mark.parametrize("M", [1, 4, 16])
def test_apply_and_apply_into(M):
    m, layer = _layer()
    x = torch.randn(M, 2048, generator=torch.Generator().manual_seed(M)).bfloat16()
    y = m.apply(layer, x.to(dev()))
    ref = onv.gemv(x.float().numpy(), layer.nvfp4_wq.cpu().numpy(), layer.nvfp4_bs.cpu().numpy(),
                   layer.nvfp4_gscale.cpu().numpy())
    assert rel_err(to_np(y), ref) <= REL_TOL
    out = torch.full((M, layer.nvfp4_wq.shape[0]), float("nan"), device=dev())
    got = m.apply_into(layer, x.to(dev()), out)
    assert got is out and torch.equal(out, y.float())
    # declines: a bias, a wrong-shaped destination, no packed weight
    assert m.apply_into(layer, x.to(dev()), out, bias=torch.zeros(1, device=dev())) is None
    assert m.apply_into(layer, x.to(dev()), out[:, :10]) is None
    assert m.apply_into(types.SimpleNamespace(), x.to(dev()), out) is None


def test_wide_m_fallback():
    m, layer = _layer(N=20000)
    x = torch.randn(20, 2048, generator=torch.Generator().manual_seed(7)).bfloat16()
    y = m.apply(layer, x.to(dev()))
    assert y.shape == (20, 20000) and y.dtype == torch.bfloat16
    w = onv.dequantize(layer.nvfp4_wq.cpu().numpy(), layer.nvfp4_bs.cpu().numpy(),
                       layer.nvfp4_gscale.cpu().numpy()).astype(np.float64)
    ref = x.float().numpy().astype(np.float64) @ w.T
    assert rel_err(to_np(y), ref) <= REL_TOL
