"""W8A16 GEMV on the GPU against the CPU oracle (parity), plus the reference's own
operator-level checks (kernels/microbench/w8a16v2/verify_v3.py, the P0032 and P0040
pytest files): 2e-2 relative error, bit-exact greedy argmax, bitwise graph replay,
counters back at zero, fp32 destination bit-identical to the widened bf16 result,
split-K agreement, two-destination store, ValueError on a bad destination."""

import numpy as np
import pytest
import torch

from oracle import numerics, w8a16 as ow8
from tests.gpu_util import REL_TOL, dev, rel_err, to_np, ulps

pytestmark = pytest.mark.gpu


def _fx():
    import flash_next_rtxpro6000_b200 as fx

    return fx


def _workspace(d):
    from flash_next_rtxpro6000_b200.w8a16_gemv import _workspace as ws

    return ws(d)


def _case(N, K, M, kind, sdtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).bfloat16()
    if kind == "int8":
        w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
        w_np = w.numpy()
    else:
        w = (torch.randn(N, K, generator=g) * 64).to(torch.float8_e4m3fn)
        w_np = w.view(torch.uint8).numpy()
    s = (torch.randn(N, generator=g).abs() / 127).to(sdtype)
    return x, w, s, w_np


@pytest.mark.parametrize("kind", ["int8", "fp8"])
@pytest.mark.parametrize("sdtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("M", [1, 2, 4, 8, 9, 16])
@pytest.mark.parametrize("N,K", [(1000, 2048), (4096, 512), (3072, 1024)])
def test_gemv_matches_oracle(kind, sdtype, M, N, K):
    fx = _fx()
    x, w, s, w_np = _case(N, K, M, kind, sdtype, seed=N + K + M)
    y = fx.w8a16_gemv(x.to(dev()), w.to(dev()), s.to(dev()))
    torch.cuda.synchronize()
    ref = ow8.gemv(x.float().numpy(), w_np, kind, s.float().numpy())
    got = to_np(y)
    assert y.shape == (M, N) and y.dtype == torch.bfloat16
    assert rel_err(got, ref) <= REL_TOL
    # Outside heavy cancellation (|ref| >= 1% of the row scale) the fp32 accumulation
    # order can only move the bf16 rounding by a step or two.
    u = ulps(got, ref)
    big = np.abs(ref) >= 1e-2 * np.abs(ref).max()
    assert u[big].max() <= 2 and (u == 0).mean() > 0.97


@pytest.mark.parametrize("M", [1, 4, 16])
def test_fp32_out_is_widened_bf16(M):
    # P0032 test_draft_logits_out: out= fp32 is bit-identical to the bf16 result widened.
    fx = _fx()
    x, w, s, _ = _case(2048, 2048, M, "fp8", torch.float32, seed=7)
    x, w, s = x.to(dev()), w.to(dev()), s.to(dev())
    y16 = fx.w8a16_gemv(x, w, s)
    buf = torch.full((M, 2048), float("nan"), device=dev())
    y32 = fx.w8a16_gemv(x, w, s, out=buf)
    assert y32 is buf
    assert torch.equal(y32, y16.float())


def test_bad_out_raises():
    fx = _fx()
    x, w, s, _ = _case(256, 512, 2, "int8", torch.float32, seed=1)
    x, w, s = x.to(dev()), w.to(dev()), s.to(dev())
    for bad in (torch.empty(2, 255, device=dev(), dtype=torch.bfloat16),
                torch.empty(2, 256, device=dev(), dtype=torch.float16),
                torch.empty(256, 2, device=dev(), dtype=torch.bfloat16).t()):
        with pytest.raises(ValueError):
            fx.w8a16_gemv(x, w, s, out=bad)
    with pytest.raises(ValueError):
        fx.w8a16_gemv(x, w, s, out2=torch.empty(2, 10, device=dev()), split_n=0)


@pytest.mark.parametrize("M", [1, 16])
@pytest.mark.parametrize("split_n", [100, 128, 255])
def test_two_destination_store(M, split_n):
    fx = _fx()
    x, w, s, _ = _case(256, 1024, M, "int8", torch.bfloat16, seed=3)
    x, w, s = x.to(dev()), w.to(dev()), s.to(dev())
    full = fx.w8a16_gemv(x, w, s)
    a = torch.empty(M, split_n, device=dev(), dtype=torch.bfloat16)
    b = torch.empty(M, 256 - split_n, device=dev(), dtype=torch.bfloat16)
    y, y2 = fx.w8a16_gemv(x, w, s, out=a, out2=b, split_n=split_n)
    assert torch.equal(torch.cat([y, y2], dim=1), full)


@pytest.mark.parametrize("M", [1, 4, 16])
def test_split_k_configs_agree(M):
    fx = _fx()
    N, K = 1280, 2048
    x, w, s, w_np = _case(N, K, M, "fp8", torch.float32, seed=909)
    x, w, s = x.to(dev()), w.to(dev()), s.to(dev())
    wmin = max(1, (M + 1) // 2)
    base = fx.w8a16_gemv(x, w, s, cfg=fx.GemvConfig(16, 2, 1, 1))
    ref = ow8.gemv(x.float().cpu().numpy(), w_np, "fp8", s.cpu().numpy())
    for ks in (2, 4, 8):
        cpu = 32 // ks
        warps = cpu if cpu <= 16 else cpu // 2
        cpw = cpu // warps
        if warps < wmin:
            continue
        got = fx.w8a16_gemv(x, w, s, cfg=fx.GemvConfig(warps, cpw, 1, ks))
        assert rel_err(to_np(got), to_np(base)) <= REL_TOL
        assert rel_err(to_np(got), ref) <= REL_TOL
    ws = _workspace(dev())
    torch.cuda.synchronize()
    assert int(ws.counters.abs().sum()) == 0


@pytest.mark.parametrize("M", [1, 9])
def test_split_k_grids_agree_bitwise(M):
    # With a grid that is a multiple of ksplit each CTA stages only its k split of x and
    # publishes its split sums already unscaled; any other grid stages whole rows.  The
    # power-of-two unscale is exact, so every grid gives the same bits.
    fx = _fx()
    N, K = 1280, 2048
    x, w, s, w_np = _case(N, K, M, "int8", torch.float32, seed=77)
    x, w, s = x.to(dev()), w.to(dev()), s.to(dev())
    outs = [fx.w8a16_gemv(x, w, s, cfg=fx.GemvConfig(8, 1, 1, 4, grid)) for grid in (0, 40, 37, 3)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    ref = ow8.gemv(x.float().cpu().numpy(), w_np, "int8", s.cpu().numpy())
    assert rel_err(to_np(outs[0]), ref) <= REL_TOL


@pytest.mark.parametrize("M", [1, 4, 16])
def test_graph_replay_bitwise_and_counters_reset(M):
    # verify_v3.py:46-83
    fx = _fx()
    N, K = 6144, 2048
    x, w, s, w_np = _case(N, K, M, "int8", torch.bfloat16, seed=11)
    w, s = w.to(dev()), s.to(dev())
    xs = x.to(dev()).clone()
    am = torch.empty(M, dtype=torch.int64, device=dev())
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            fx.w8a16_gemv(xs, w, s, argmax_out=am)
            fx.w8a16_gemv(xs, w, s, cfg=fx.GemvConfig(8, 1, 1, 4))
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        y1g = fx.w8a16_gemv(xs, w, s, argmax_out=am)
        y2g = fx.w8a16_gemv(xs, w, s, cfg=fx.GemvConfig(8, 1, 1, 4))
    g.replay()
    torch.cuda.synchronize()
    a1, a2, am1 = y1g.clone(), y2g.clone(), am.clone()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(a1, y1g) and torch.equal(a2, y2g) and torch.equal(am1, am)
    ref = ow8.gemv(x.float().numpy(), w_np, "int8", s.float().cpu().numpy())
    assert rel_err(to_np(a1), ref) <= REL_TOL and rel_err(to_np(a2), ref) <= REL_TOL
    x2 = torch.randn(M, K).bfloat16()
    xs.copy_(x2.to(dev()))
    g.replay()
    torch.cuda.synchronize()
    ref2 = ow8.gemv(x2.float().numpy(), w_np, "int8", s.float().cpu().numpy())
    assert rel_err(to_np(y1g), ref2) <= REL_TOL
    assert torch.equal(am.cpu(), torch.from_numpy(ow8.argmax_lowest(to_np(y1g))))
    ws = _workspace(dev())
    assert int(ws.counters.abs().sum()) == 0
    assert int(ws.argmax_keys.abs().sum()) == 0 and int(ws.argmax_count.sum()) == 0
    del g


@pytest.mark.parametrize("V", [49152, 151936])
@pytest.mark.parametrize("M", [1, 4, 16])
def test_lm_head_argmax_bit_exact(V, M):
    """Config 1: int8 [V, 2048] lm_head with bf16 per-row scales; the greedy argmax must
    equal the oracle's (fp64 logits rounded to bf16, lowest row on ties)."""
    fx = _fx()
    from flash_next_rtxpro6000_b200 import synthetic as syn

    head = syn.w8_head(V, syn.HIDDEN, seed=0)
    x = syn.activations(M, seed=1)
    w, s = head.w.to(dev()), head.scale.to(dev())
    am = torch.empty(M, dtype=torch.int64, device=dev())
    y = fx.w8a16_gemv(x.to(dev()), w, s, argmax_out=am)
    torch.cuda.synchronize()
    exact = ow8.gemv_f64(x.float().numpy(), head.w.numpy(), "int8", head.scale.float().numpy())
    ref = numerics.bf16_round_from_f64(exact)
    got = to_np(y)
    assert rel_err(got, ref) <= REL_TOL
    want = ow8.argmax_lowest(ref)
    assert am.cpu().numpy().tolist() == want.tolist()
    # the fused argmax agrees with torch.argmax of the kernel's own logits
    assert am.cpu().tolist() == torch.argmax(y.float(), dim=-1).cpu().tolist()


@pytest.mark.parametrize("M", [1, 4, 16])
def test_silu_mul_matches_oracle_and_two_step(M):
    # P0040 test_w8a16_gemv_silu.py: fused within 1 ulp mean / 4 max of the two-kernel path
    fx = _fx()
    N, K = 1024, 2048
    # the reference test's weights: randn * 0.02, per-row amax / 448, fp8 e4m3
    g = torch.Generator().manual_seed(20260903 + M + N)
    wf = torch.randn(N, K, generator=g) * 0.02
    s = (wf.abs().amax(dim=1) / 448.0).clamp(min=1e-12)
    w = (wf / s[:, None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    w_np = w.view(torch.uint8).numpy()
    x = torch.randn(M, K, generator=g).bfloat16()
    xd, wd, sd = x.to(dev()), w.to(dev()), s.to(dev())
    fused = fx.w8a16_gemv_silu_mul(xd, wd, sd)
    assert fused.shape == (M, N // 2) and fused.dtype == torch.bfloat16
    gu = fx.w8a16_gemv(xd, wd, sd)
    h = N // 2
    two = (torch.nn.functional.silu(gu[:, :h].float()) * gu[:, h:].float()).bfloat16()
    golden = ow8.silu_mul(x.float().numpy(), w_np, "fp8", s.numpy())
    f, t = to_np(fused), to_np(two)
    assert rel_err(f, golden) <= REL_TOL
    u = ulps(f, t)
    assert u.mean() <= 1.0 and u.max() <= 4
    assert np.abs(f - golden).max() <= np.abs(t - golden).max() * 1.5 + 1e-6


def test_zero_tokens_is_a_no_op():
    fx = _fx()
    x = torch.empty(0, 512, dtype=torch.bfloat16, device=dev())
    w = torch.zeros(64, 512, dtype=torch.int8, device=dev())
    y = fx.w8a16_gemv(x, w, torch.ones(64, device=dev()))
    assert y.shape == (0, 64)


def test_bf16_gemv_matches_matmul():
    fx = _fx()
    g = torch.Generator().manual_seed(5)
    x = torch.randn(3, 1024, generator=g).bfloat16()
    w = (torch.randn(700, 1024, generator=g) * 0.05).bfloat16()
    y = fx.bf16_gemv(x.to(dev()), w.to(dev()))
    ref = (x.double() @ w.double().t()).numpy()
    assert rel_err(to_np(y), numerics.bf16_round_from_f64(ref)) <= REL_TOL
