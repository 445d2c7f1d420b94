"""Generate the golden fixtures that pin the CPU oracle to the reference's own code.

Run in a container that has the reference checkout (it is NOT needed at test time):

    python tests/golden/make_golden.py /path/to/reference

It imports the reference's Python modules by file path, with empty stand-ins for the
``sglang`` packages they live in, and records their outputs on seeded inputs:

* ``nvfp4_codec.npz``   -- quantize_nvfp4 / dequantize_nvfp4
  (kernels/sglang/srt/layers/quantization/w4a16_nvfp4_gemv.py:426-510) on random,
  all-codes (kernels/microbench/n1/check_nvfp4_gemv.py:51-56), zero-block and
  tie-heavy weights;
* ``swizzle.npz``       -- swizzle_blockscale_cpu (bench/bench/moe_smallm/weights.py:156-175);
* ``moe_ref.npz``       -- moe_reference (bench/bench/moe_smallm/refs.py:50-78) on a
  small seeded layer, checkpoint row order;
* ``w8a16_norm_gated.npz`` -- the same kernel's fused gated-RMSNorm form
  (w8a16_gemv.py:186-259, SiLU and sigmoid gates) at M=1 and M=4 under the interpreter
* ``router_topk.npz``   -- the reference's packed-key softmax top-k router (patches
  0110 + 0111, moe_router_softmax_fast.py) under the interpreter: 512/256/128 experts,
  top-10/8/6, renormalised or not, exact ties, a NaN and -0.0 logits;
* ``w8a16_kernel.npz``  -- the reference's Triton W8A16 kernel itself
  (w8a16_gemv.py:642-666) at M=1 under the Triton CPU interpreter, int8 and fp8
  weights, per-row fp32 and bf16 scales, bf16 and fp32 destinations.
"""

from __future__ import annotations

import importlib.util
import os
import subprocess
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _stub(name: str) -> None:
    if name not in sys.modules:
        m = types.ModuleType(name)
        m.__path__ = []
        sys.modules[name] = m


def _load(name: str, path: Path):
    spec = importlib.util.spec_from_file_location(name, str(path))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load_reference(ref: Path):
    for n in ("sglang", "sglang.kernels", "sglang.srt", "sglang.srt.layers",
              "sglang.srt.layers.quantization"):
        _stub(n)
    _load("sglang.kernels.triton_pdl", ref / "kernels/sglang/kernels/triton_pdl.py")
    w8 = _load("sglang.srt.layers.quantization.w8a16_gemv",
               ref / "kernels/sglang/srt/layers/quantization/w8a16_gemv.py")
    w4 = _load("sglang.srt.layers.quantization.w4a16_nvfp4_gemv",
               ref / "kernels/sglang/srt/layers/quantization/w4a16_nvfp4_gemv.py")
    pkg = ref / "bench/bench/moe_smallm"
    spec = importlib.util.spec_from_file_location(
        "moe_smallm", str(pkg / "__init__.py"), submodule_search_locations=[str(pkg)])
    if (pkg / "__init__.py").exists():
        m = importlib.util.module_from_spec(spec)
        sys.modules["moe_smallm"] = m
        spec.loader.exec_module(m)
    else:
        _stub("moe_smallm")
        sys.modules["moe_smallm"].__path__ = [str(pkg)]
    refs = _load("moe_smallm.refs", pkg / "refs.py")
    _load("moe_smallm.model_shapes", pkg / "model_shapes.py")
    weights = _load("moe_smallm.weights", pkg / "weights.py")
    return w8, w4, refs, weights


def nvfp4_cases():
    g = torch.Generator().manual_seed(0)
    cases = {}
    cases["randn"] = (torch.randn(64, 256, generator=g) * 0.02).bfloat16()
    lvl = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
    row = torch.cat([lvl, -lvl])
    cases["allcodes"] = torch.stack([row * s for s in (0.25, 0.5, 1.0, 2.0, 4.0)]).bfloat16()
    z = (torch.randn(16, 128, generator=g) * 3.0).bfloat16()
    z[3, 16:32] = 0
    z[7, :] = 0
    z[9, 0:16] = 1e-30
    cases["zero_blocks"] = z
    # values on the e2m1 midpoints of their block (ties-to-even in both the block scale
    # and the code rounding)
    t = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0] * 2)
    ties = torch.stack([t * s for s in (1.0, 0.125, 3.0, 0.0078125)])
    cases["ties"] = ties.repeat(1, 4).bfloat16()
    rows = torch.randn(32, 512, generator=g) * torch.logspace(-3, 2, 32).unsqueeze(1)
    cases["row_spread"] = rows.bfloat16()
    return cases


def make_nvfp4(w4):
    out = {}
    for name, w in nvfp4_cases().items():
        wq, bs, gs = w4.quantize_nvfp4(w)
        deq = w4.dequantize_nvfp4(wq, bs, gs)
        out[f"{name}_w"] = w.float().numpy()
        out[f"{name}_wq"] = wq.numpy()
        out[f"{name}_bs"] = bs.numpy()
        out[f"{name}_gscale"] = gs.float().numpy()
        out[f"{name}_deq"] = deq.numpy()
    np.savez_compressed(HERE / "nvfp4_codec.npz", **out)


def make_swizzle(weights):
    g = torch.Generator().manual_seed(1)
    out = {}
    shapes = {"a": (1, 128, 8), "b": (2, 130, 5), "c": (3, 256, 32)}
    for k, shp in shapes.items():
        if k == "a":
            sf = torch.arange(int(np.prod(shp)), dtype=torch.float32).reshape(shp) % 448
        else:
            sf = torch.rand(shp, generator=g) * 400
        sf8 = sf.to(torch.float8_e4m3fn)
        out[f"{k}_in"] = sf8.view(torch.uint8).numpy()
        out[f"{k}_out"] = weights.swizzle_blockscale_cpu(sf8).view(torch.uint8).numpy()
    np.savez_compressed(HERE / "swizzle.npz", **out)


def make_moe(refs, w4):
    g = torch.Generator().manual_seed(2)
    E, H, I, T, K = 8, 256, 128, 3, 4
    w13q = torch.empty(E, 2 * I, H // 2, dtype=torch.uint8)
    w13s = torch.empty(E, 2 * I, H // 16, dtype=torch.uint8)
    w2q = torch.empty(E, H, I // 2, dtype=torch.uint8)
    w2s = torch.empty(E, H, I // 16, dtype=torch.uint8)
    g13 = torch.empty(E, 2)
    g2 = torch.empty(E)
    for e in range(E):
        gu = (torch.randn(2 * I, H, generator=g) * 0.05).bfloat16()  # [gate; up]
        q, bs, gs = w4.quantize_nvfp4(gu)
        w13q[e], w13s[e], g13[e] = q, bs, gs.reshape(1).expand(2)
        dn = (torch.randn(H, I, generator=g) * 0.05).bfloat16()
        q2, bs2, gs2 = w4.quantize_nvfp4(dn)
        w2q[e], w2s[e], g2[e] = q2, bs2, gs2.reshape(())
    ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).to(torch.int32)
    wts = torch.rand(T, K, generator=g).softmax(-1)
    x = torch.randn(T, H, generator=g).bfloat16()
    lw = types.SimpleNamespace(
        shape=types.SimpleNamespace(intermediate=I), w13_weight=w13q,
        w13_weight_scale=w13s.view(torch.float8_e4m3fn), w2_weight=w2q,
        w2_weight_scale=w2s.view(torch.float8_e4m3fn), w13_weight_scale_2=g13,
        w2_weight_scale_2=g2)
    y = refs.moe_reference(lw, x, ids, wts)
    np.savez_compressed(
        HERE / "moe_ref.npz", w13=w13q.numpy(), s13=w13s.numpy(), g13=g13.numpy(),
        w2=w2q.numpy(), s2=w2s.numpy(), g2=g2.numpy(), ids=ids.numpy(), wts=wts.numpy(),
        x=x.float().numpy(), y=y.float().numpy())


_INTERP = r'''
import os, sys, numpy as np, torch
sys.path.insert(0, os.path.dirname(sys.argv[1]))
import make_golden as mg
w8, w4, refs, weights = mg.load_reference(mg.Path(sys.argv[2]))
g = torch.Generator().manual_seed(3)
out = {}
N, K = 96, 256
x = torch.randn(1, K, generator=g).bfloat16()
wi = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
sf = (torch.randn(N, generator=g).abs() / 127).float()
sb = sf.bfloat16()
wf = (torch.randn(N, K, generator=g) * 64).to(torch.float8_e4m3fn)
out["x"] = x.float().numpy()
out["w_int8"] = wi.numpy()
out["scale_f32"] = sf.numpy()
out["scale_bf16"] = sb.float().numpy()
out["w_fp8"] = wf.view(torch.uint8).numpy()
# the reference's M == 1 wide-N tile (w8a16_gemv.py:497) and a split-K tile (:452);
# passed explicitly because the planner queries the GPU's SM count
tile = (32, 256, 1, False, None, 4, 3)
split = (16, 64, 4, False, None, 4, 3)
out["y_int8_f32s"] = w8.w8a16_gemv(x, wi, sf, cfg=tile).float().numpy()
out["y_int8_bf16s"] = w8.w8a16_gemv(x, wi, sb, cfg=tile).float().numpy()
out["y_fp8_f32s"] = w8.w8a16_gemv(x, wf, sf, cfg=tile).float().numpy()
out["y_fp8_split"] = w8.w8a16_gemv(x, wf, sf, cfg=split).float().numpy()
buf = torch.zeros(1, N, dtype=torch.float32)
out["y_fp8_f32out"] = w8.w8a16_gemv(x, wf, sf, cfg=tile, out=buf).numpy()
np.savez_compressed(sys.argv[3], **out)
'''


_INTERP_NORM = r'''
import os, sys, numpy as np, torch
sys.path.insert(0, os.path.dirname(sys.argv[1]))
import make_golden as mg
w8, w4, refs, weights = mg.load_reference(mg.Path(sys.argv[2]))
g = torch.Generator().manual_seed(11)
out = {}
N, K, G = 64, 256, 128
wi = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
sf = (torch.randn(N, generator=g).abs() / 127).float()
nwb = (1.0 + 0.25 * torch.randn(G, generator=g)).bfloat16()
out["w_int8"] = wi.numpy()
out["scale_f32"] = sf.numpy()
out["norm_w"] = nwb.float().numpy()
# the fused gated-RMSNorm form of the reference kernel (w8a16_gemv.py:186-259), launched
# with an explicit tile whose BLOCK_K is the norm group (the planner queries the GPU).
# The interpreter's tl.dot on bf16 operands returns values near 1e9 even without the norm,
# so every row runs through the M = 1 broadcast path; the tl.dot path (:214-233) applies
# the same per-row statistics
tile = (32, G, 1, False, None, 4, 2)
for M in (1, 4):
    x = (torch.randn(M, K, generator=g) * 3).bfloat16()
    z = torch.randn(M, K, generator=g).bfloat16()
    out[f"x{M}"] = x.float().numpy()
    out[f"z{M}"] = z.float().numpy()
    for sig in (False, True):
        y = torch.zeros(M, N, dtype=torch.bfloat16)
        for m in range(M):
            ym = torch.zeros(1, N, dtype=torch.bfloat16)
            w8._launch(x[m:m + 1].contiguous(), wi, sf, ym, 1, N, K, True, tile,
                       norm=(z[m:m + 1].contiguous(), nwb, G, 1e-6, sig))
            y[m] = ym[0]
        out[f"y{M}_{'sigmoid' if sig else 'silu'}"] = y.float().numpy()
np.savez_compressed(sys.argv[3], **out)
'''


def make_w8a16_norm_interp(ref: Path):
    env = dict(os.environ, TRITON_INTERPRET="1", CUDA_VISIBLE_DEVICES="")
    subprocess.run([sys.executable, "-c", _INTERP_NORM, str(Path(__file__).resolve()), str(ref),
                    str(HERE / "w8a16_norm_gated.npz")], check=True, env=env, cwd=str(HERE))


def make_w8a16_interp(ref: Path):
    env = dict(os.environ, TRITON_INTERPRET="1", CUDA_VISIBLE_DEVICES="")
    code = _INTERP
    subprocess.run([sys.executable, "-c", code, str(Path(__file__).resolve()), str(ref),
                    str(HERE / "w8a16_kernel.npz")], check=True, env=env, cwd=str(HERE))


_INTERP_ROUTER = r'''
import sys, types, importlib.util, numpy as np, torch
for n in ("sglang", "sglang.kernels", "sglang.kernels.jit", "sglang.kernels.ops",
          "sglang.kernels.ops.moe"):
    m = types.ModuleType(n); m.__path__ = []; sys.modules[n] = m
u = types.ModuleType("sglang.kernels.jit.utils"); u.is_arch_support_pdl = lambda: False
sys.modules["sglang.kernels.jit.utils"] = u
spec = importlib.util.spec_from_file_location("rfast", sys.argv[1])
rf = importlib.util.module_from_spec(spec); spec.loader.exec_module(rf)
g = torch.Generator().manual_seed(5)
out = {}
cases = {
    # 512 experts, the served top-10 (renormalised) and a plain top-8
    "a": ((torch.randn(4, 512, generator=g) * 2).bfloat16(), 10, True),
    "b": ((torch.randn(3, 512, generator=g) * 2).bfloat16(), 8, False),
    # coarse values: many exact ties (lowest id must win), fewer experts
    "c": ((torch.randint(-3, 4, (5, 256), generator=g).float() * 0.5).bfloat16(), 10, True),
    # a NaN logit and -0.0 entries
    "d": ((torch.randn(2, 128, generator=g)).bfloat16(), 6, True),
}
cases["d"][0][0, 7] = float("nan")
cases["d"][0][1, 3:9] = -0.0
for key, (scores, k, renorm) in cases.items():
    zero = torch.zeros(scores.shape[1], dtype=torch.float32)
    w, i = rf.route_softmax_fast(scores, zero, k, renorm)
    out[f"scores_{key}"] = scores.float().numpy()
    out[f"topk_{key}"] = np.array([k, int(renorm)])
    out[f"w_{key}"] = w.numpy()
    out[f"ids_{key}"] = i.numpy()
np.savez_compressed(sys.argv[2], **out)
'''


def make_router_topk_interp(ref: Path):
    """The reference's softmax top-k router (patches 0110 + 0111 applied to an empty tree,
    python/sglang/kernels/ops/moe/moe_router_softmax_fast.py) under the Triton CPU
    interpreter -> router_topk.npz."""
    import shutil
    import tempfile

    tmp = Path(tempfile.mkdtemp())
    try:
        subprocess.run(["git", "init", "-q"], cwd=tmp, check=True)
        rel = "python/sglang/kernels/ops/moe/moe_router_softmax_fast.py"
        for p in ("0110", "0111"):
            patch = next((ref / "patches/sglang/series").glob(f"{p}-*.patch"))
            subprocess.run(["git", "apply", f"--include={rel}", str(patch)], cwd=tmp, check=True)
        env = dict(os.environ, TRITON_INTERPRET="1", CUDA_VISIBLE_DEVICES="")
        subprocess.run([sys.executable, "-c", _INTERP_ROUTER, str(tmp / rel),
                        str(HERE / "router_topk.npz")], check=True, env=env, cwd=str(HERE))
    finally:
        shutil.rmtree(tmp)


def main():
    ref = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FNX_REFERENCE", ""))
    if not (ref / "kernels").is_dir():
        sys.exit("usage: make_golden.py <reference checkout>")
    w8, w4, refs, weights = load_reference(ref)
    make_nvfp4(w4)
    make_swizzle(weights)
    make_moe(refs, w4)
    make_w8a16_interp(ref)
    make_w8a16_norm_interp(ref)
    make_router_topk_interp(ref)
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
