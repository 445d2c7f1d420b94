"""The reference's CPU path for the three benchmark configurations, restated in torch.

Test and measurement infrastructure only: ``bench.py`` times these functions as the CPU
baseline (its ``cpu_baseline`` leg and ``--impl reference``), on all the host's cores
(``torch.set_num_threads``).  Nothing in the library imports this module.

The reference's own CPU path is torch on fp32 tensors: dequantise, then ``torch.matmul``.
Its source cannot travel to the GPU box, so the same steps are restated here:

* NVFP4 GEMV (config 0): ``dequantize_nvfp4`` then ``x.float() @ W.T`` rounded to bf16
  (kernels/sglang/srt/layers/quantization/w4a16_nvfp4_gemv.py:489-510: e2m1 level table
  indexed by the code's low three bits, sign from bit 3, times e4m3 block scale times the
  global scale, repeated over each 16-column block);
* W8A16 lm_head + greedy argmax (config 1): ``w.float() * s[:, None]``, fp32 matmul,
  bf16 logits, argmax (the reference's oracle for that operator, w8a16_gemv.py:92-95 for
  the bf16 rounding);
* routed MoE (config 2): bench/bench/moe_smallm/refs.py:50-78 ``moe_reference``: per
  token and route, dequantise the expert, gate/up projection, silu(gate) * up in fp32,
  down projection, weighted sum; here with the server row order [up; gate] and one global
  scale per expert (patches/sglang/series/0112-...patch:68-76), the activation rounded to
  bf16 between the projections (0112-...patch:224), plus the always-on shared expert.
"""

from __future__ import annotations

import torch

_E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=torch.float32)


def dequantize_nvfp4(wq: torch.Tensor, bs_e4m3_bits: torch.Tensor, gscale) -> torch.Tensor:
    """fp32 [N, K] from packed codes [N, K/2] (low nibble = even k), e4m3 block scales
    [N, K/16] (uint8 bit patterns) and an fp32 global scale (scalar or [N])."""
    N, KH = wq.shape
    codes = torch.stack((wq & 0x0F, wq >> 4), dim=-1).reshape(N, 2 * KH)
    mag = _E2M1[(codes & 0x07).long()]
    val = torch.where((codes & 0x08) != 0, -mag, mag)
    g = torch.as_tensor(gscale, dtype=torch.float32).reshape(-1)
    g = g.reshape(-1, 1) if g.numel() > 1 else g.reshape(1, 1)
    s = bs_e4m3_bits.view(torch.float8_e4m3fn).float() * g
    return val * s.repeat_interleave(16, dim=1)


def nvfp4_gemv(x: torch.Tensor, wq, bs, gscale) -> torch.Tensor:
    return (x.float() @ dequantize_nvfp4(wq, bs, gscale).T).to(torch.bfloat16)


def lm_head_argmax(x: torch.Tensor, w: torch.Tensor, s: torch.Tensor):
    logits = (x.float() @ (w.float() * s.float()[:, None]).T).to(torch.bfloat16)
    return logits, logits.float().argmax(dim=-1)


def _expert(x: torch.Tensor, w13, s13, g13, w2, s2, g2) -> torch.Tensor:
    """One expert on one token row: [H] -> [H] (fp32)."""
    h = dequantize_nvfp4(w13, s13, g13) @ x
    I = h.shape[0] // 2
    up, gate = h[:I], h[I:]
    act = (torch.nn.functional.silu(gate) * up).to(torch.bfloat16).float()
    return dequantize_nvfp4(w2, s2, g2) @ act


def moe_layer(x: torch.Tensor, ids: torch.Tensor, wts: torch.Tensor, layer) -> torch.Tensor:
    """The routed layer with the shared expert: x bf16 [M, H] -> bf16 [M, H].  ``layer``
    carries linear-layout scales (flash_next_rtxpro6000_b200.synthetic.MoeLayer)."""
    xf = x.float()
    out = torch.zeros_like(xf)
    for t in range(x.shape[0]):
        acc = torch.zeros(x.shape[1], dtype=torch.float32)
        for r in range(ids.shape[1]):
            e = int(ids[t, r])
            if e < 0:
                continue
            acc += float(wts[t, r]) * _expert(xf[t], layer.w13[e], layer.s13[e], layer.g13[e, 0],
                                              layer.w2[e], layer.s2[e], layer.g2[e])
        acc += _expert(xf[t], layer.sh_w13[0], layer.sh_s13[0], layer.sh_g13[0],
                       layer.sh_w2[0], layer.sh_s2[0], layer.sh_g2[0])
        out[t] = acc
    return out.to(torch.bfloat16)
