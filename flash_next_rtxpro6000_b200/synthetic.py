"""Seeded synthetic inputs with the shapes and value distributions of the benchmark
configurations (no checkpoints or datasets are available; random weights of the right
format stand in for them).  Everything is drawn on the CPU from
``torch.Generator().manual_seed(seed)`` so the same tensors can feed the GPU kernels and
the CPU oracle.

* config 0 -- NVFP4 GEMV 4096 x 2048: x ~ N(0,1) bf16 [M, 2048]; packed codes uniform
  over the 256 byte values; block scales |N(0,1)| * 0.5 -> e4m3; global scale 1/448.
* config 1 -- W8A16 lm_head: int8 [V, 2048] uniform on [-127, 127]; per-row bf16 scales
  |N(0,1)| / 127; x ~ N(0,1) bf16.  V = 151936 (target) or 49152 (draft head).
* config 2 -- NVFP4 routed MoE: 512 experts, H = 2048, I = 512, config-0-style codes and
  scales per expert (w13 rows [up; gate], scales 128x4 swizzled for the server layout),
  global scales 1/448; routing = top-10 of softmax(N(0,1) logits), lowest id first on
  ties, weights renormalised; an always-on shared expert of the same format.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

HIDDEN = 2048
INTER = 512
EXPERTS = 512
TOPK = 10
VOCAB = 151936
DRAFT_VOCAB = 49152
NVFP4_N = 4096


def _gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def activations(M: int, K: int = HIDDEN, seed: int = 0) -> torch.Tensor:
    return torch.randn(M, K, generator=_gen(seed)).to(torch.bfloat16)


@dataclass
class Nvfp4Weight:
    wq: torch.Tensor      # uint8 [N, K/2]
    bs: torch.Tensor      # uint8 [N, K/16] (e4m3 bits, linear layout)
    gscale: torch.Tensor  # fp32 [1]


def nvfp4_weight(N: int = NVFP4_N, K: int = HIDDEN, seed: int = 0,
                 g: Optional[torch.Generator] = None) -> Nvfp4Weight:
    g = g or _gen(seed)
    wq = torch.randint(0, 256, (N, K // 2), generator=g, dtype=torch.uint8)
    bs = (torch.randn(N, K // 16, generator=g).abs() * 0.5).to(torch.float8_e4m3fn).view(torch.uint8)
    return Nvfp4Weight(wq, bs, torch.tensor([1.0 / 448.0], dtype=torch.float32))


def config0(M: int = 1, seed: int = 0):
    """(x, Nvfp4Weight) of config 0 (x and the weight share one seeded stream)."""
    g = _gen(seed)
    x = torch.randn(M, HIDDEN, generator=g).to(torch.bfloat16)
    w = nvfp4_weight(NVFP4_N, HIDDEN, g=g)
    return x, w


@dataclass
class W8Head:
    w: torch.Tensor      # int8 [V, K]
    scale: torch.Tensor  # bf16 [V]


def w8_head(V: int = VOCAB, K: int = HIDDEN, seed: int = 0) -> W8Head:
    g = _gen(seed)
    w = torch.randint(-127, 128, (V, K), generator=g, dtype=torch.int8)
    s = (torch.randn(V, generator=g).abs() / 127.0).to(torch.bfloat16)
    return W8Head(w, s)


@dataclass
class MoeLayer:
    w13: torch.Tensor        # uint8 [E, 2I, H/2]  rows [up(I); gate(I)]
    s13: torch.Tensor        # uint8 [E, 2I, H/16] linear
    g13: torch.Tensor        # fp32 [E, 2]
    w2: torch.Tensor         # uint8 [E, H, I/2]
    s2: torch.Tensor         # uint8 [E, H, I/16] linear
    g2: torch.Tensor         # fp32 [E]
    sh_w13: torch.Tensor     # shared expert [1, 2I, H/2] etc.
    sh_s13: torch.Tensor
    sh_g13: torch.Tensor     # fp32 [1]
    sh_w2: torch.Tensor
    sh_s2: torch.Tensor
    sh_g2: torch.Tensor

    @property
    def E(self) -> int:
        return self.w13.shape[0]

    @property
    def H(self) -> int:
        return self.w13.shape[2] * 2

    @property
    def I(self) -> int:
        return self.w13.shape[1] // 2


def _codes_and_scales(g: torch.Generator, *shape_rows_k):
    *lead, rows, K = shape_rows_k
    q = torch.randint(0, 256, (*lead, rows, K // 2), generator=g, dtype=torch.uint8)
    s = (torch.randn(*lead, rows, K // 16, generator=g).abs() * 0.5).to(torch.float8_e4m3fn)
    return q, s.view(torch.uint8)


def moe_layer(E: int = EXPERTS, H: int = HIDDEN, I: int = INTER, seed: int = 0) -> MoeLayer:
    g = _gen(seed)
    w13, s13 = _codes_and_scales(g, E, 2 * I, H)
    w2, s2 = _codes_and_scales(g, E, H, I)
    sw13, ss13 = _codes_and_scales(g, 1, 2 * I, H)
    sw2, ss2 = _codes_and_scales(g, 1, H, I)
    gs = 1.0 / 448.0
    return MoeLayer(w13, s13, torch.full((E, 2), gs), w2, s2, torch.full((E,), gs),
                    sw13, ss13, torch.tensor([gs]), sw2, ss2, torch.tensor([gs]))


def routing(M: int, E: int = EXPERTS, top_k: int = TOPK, seed: int = 0):
    """(topk_ids int32 [M, k], topk_weights fp32 [M, k]) from softmax(N(0,1)) logits."""
    g = _gen(seed + 1000)
    logits = torch.randn(M, E, generator=g)
    p = torch.softmax(logits, dim=-1)
    # lowest id first among equal probabilities: stable sort on (-p)
    order = torch.sort(-p, dim=-1, stable=True).indices[:, :top_k]
    w = torch.gather(p, 1, order)
    w = w / w.sum(dim=-1, keepdim=True)
    return order.to(torch.int32), w.float()


def moe_bytes(D: int, H: int = HIDDEN, I: int = INTER, M: int = 1, shared: bool = True) -> int:
    """Algorithmic bytes of one MoE call: each distinct expert's weights + scales once, plus
    x in and the bf16 output."""
    per_expert = (2 * I * H + H * I) * 9 // 16
    return (D + int(shared)) * per_expert + 2 * 2 * H * M


def w8_head_bytes(V: int, K: int, M: int, argmax: bool = True) -> int:
    """Weights + bf16 scales + x + bf16 logits (+ int64 argmax)."""
    return V * K + 2 * V + 2 * K * M + 2 * V * M + (8 * M if argmax else 0)


def nvfp4_bytes(N: int, K: int, M: int) -> int:
    return N * K // 2 + N * K // 16 + 2 * K * M + 2 * N * M
