"""The torch restatement of the reference's CPU path (oracle/cpu_path.py, the bench's CPU
baseline) agrees with the pinned numpy oracle: the NVFP4 dequantisation bit for bit, the
GEMVs and the MoE layer within the parity tolerance."""

import numpy as np
import torch

from flash_next_rtxpro6000_b200 import synthetic as syn
from oracle import cpu_path, moe as omoe, nvfp4 as onv, w8a16 as ow8
from tests.gpu_util import REL_TOL, rel_err


def test_dequantize_matches_oracle_bit_for_bit():
    w = syn.nvfp4_weight(256, 512, seed=3)
    a = cpu_path.dequantize_nvfp4(w.wq, w.bs, w.gscale).numpy()
    b = onv.dequantize(w.wq.numpy(), w.bs.numpy(), w.gscale.numpy())
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_gemvs_match_oracle():
    x, w = syn.config0(M=2, seed=4)
    y = cpu_path.nvfp4_gemv(x, w.wq, w.bs, w.gscale).float().numpy()
    assert rel_err(y, onv.gemv(x.float().numpy(), w.wq.numpy(), w.bs.numpy(),
                               w.gscale.numpy())) <= REL_TOL
    head = syn.w8_head(4096, 2048, seed=5)
    x = syn.activations(3, seed=6)
    logits, am = cpu_path.lm_head_argmax(x, head.w, head.scale)
    ref = ow8.gemv(x.float().numpy(), head.w.numpy(), "int8", head.scale.float().numpy())
    assert rel_err(logits.float().numpy(), ref) <= REL_TOL


def test_moe_layer_matches_oracle():
    L = syn.moe_layer(16, 512, 256, seed=7)
    ids, wts = syn.routing(2, E=16, top_k=4, seed=8)
    x = syn.activations(2, K=512, seed=9)
    y = cpu_path.moe_layer(x, ids, wts, L).float().numpy()
    sh = dict(w13=L.sh_w13.numpy()[0], s13=L.sh_s13.numpy()[0], g13=L.sh_g13.numpy(),
              w2=L.sh_w2.numpy()[0], s2=L.sh_s2.numpy()[0], g2=L.sh_g2.numpy())
    ref = omoe.moe(x.float().numpy(), ids.numpy(), wts.numpy(), L.w13.numpy(), L.s13.numpy(),
                   L.g13.numpy(), L.w2.numpy(), L.s2.numpy(), L.g2.numpy(), shared=sh)
    assert rel_err(y, ref) <= REL_TOL
