"""The CPU oracle against the reference's own outputs and known answers.

Fixtures come from tests/golden/make_golden.py, which runs the reference's Python code
(quantize_nvfp4 / dequantize_nvfp4, swizzle_blockscale_cpu, moe_reference and the Triton
W8A16 kernel under the CPU interpreter) on seeded inputs.
"""

import os

import numpy as np
import pytest

from oracle import moe, numerics, nvfp4, router, w8a16

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _npz(name):
    return np.load(os.path.join(GOLD, name))


# ---------------------------------------------------------------- known answers
def test_unpack_low_nibble_first():
    # bench/bench/moe_smallm/tests_cpu.py:140-144
    codes = nvfp4.unpack_codes(np.array([[0x21, 0xF8]], dtype=np.uint8))
    v = numerics.e2m1_to_f32(codes)[0]
    assert v.tolist() == [0.5, 1.0, -0.0, -6.0]
    assert np.signbit(v[2])


def test_bytes_per_weight_is_nine_sixteenths():
    # bench/bench/moe_smallm/tests_cpu.py:40-46 (4 bits + one e4m3 per 16 weights)
    H, I = 2560, 640
    n = 2 * I * H + H * I
    codes = n // 2
    scales = n // 16
    assert codes + scales == n * 9 // 16 == 2_764_800


def test_code_eight_is_negative_zero():
    # kernels/microbench/n1/check_nvfp4_gemv.py:35-38
    assert numerics.e2m1_to_f32(np.array([8], np.uint8))[0] == 0.0
    assert np.signbit(numerics.e2m1_to_f32(np.array([8], np.uint8))[0])


def test_swizzle_permutation_known_answer():
    # bench/bench/moe_smallm/tests_cpu.py:125-138
    sf = (np.arange(128 * 8) % 448).astype(np.float32).reshape(1, 128, 8)
    sf8 = numerics.f32_to_e4m3(sf)
    sw = nvfp4.swizzle_blockscale(sf8)
    assert sw.shape == (1, 128, 8)
    assert sorted(sw.ravel().tolist()) == sorted(sf8.ravel().tolist())
    assert not np.array_equal(sw.ravel(), sf8.ravel())
    assert nvfp4.swizzle_blockscale(np.zeros((2, 130, 5), np.uint8)).shape == (2, 256, 8)


def test_swizzled_offset_matches_permutation():
    rng = np.random.default_rng(0)
    sf = rng.integers(0, 255, (256, 32), dtype=np.uint8)
    flat = nvfp4.swizzle_blockscale(sf).ravel()
    for m, kb in [(0, 0), (1, 3), (31, 4), (32, 5), (127, 31), (128, 0), (200, 17), (255, 31)]:
        assert flat[nvfp4.swizzled_offset(m, kb, 32)] == sf[m, kb]
    assert np.array_equal(nvfp4.unswizzle_blockscale(nvfp4.swizzle_blockscale(sf), 256, 32), sf)


# ---------------------------------------------------------------- reference goldens
@pytest.mark.parametrize("case", ["randn", "allcodes", "zero_blocks", "ties", "row_spread"])
def test_quantize_matches_reference_bitwise(case):
    g = _npz("nvfp4_codec.npz")
    wq, bs, gs = nvfp4.quantize(g[f"{case}_w"])
    assert np.array_equal(wq, g[f"{case}_wq"])
    assert np.array_equal(bs, g[f"{case}_bs"])
    assert np.array_equal(gs, g[f"{case}_gscale"].reshape(-1))


@pytest.mark.parametrize("case", ["randn", "allcodes", "zero_blocks", "ties", "row_spread"])
def test_dequantize_matches_reference_bitwise(case):
    g = _npz("nvfp4_codec.npz")
    deq = nvfp4.dequantize(g[f"{case}_wq"], g[f"{case}_bs"], g[f"{case}_gscale"])
    assert np.array_equal(deq.view(np.uint32), g[f"{case}_deq"].astype(np.float32).view(np.uint32))


def test_all_reachable_codes_round_trip():
    # kernels/microbench/n1/check_nvfp4_gemv.py:41-60: every code but 8 appears and
    # the round trip is exact
    g = _npz("nvfp4_codec.npz")
    w = g["allcodes_w"]
    wq, bs, gs = nvfp4.quantize(w)
    assert np.array_equal(nvfp4.dequantize(wq, bs, gs), w)
    seen = set(nvfp4.unpack_codes(wq).ravel().tolist())
    assert seen == set(range(16)) - {8}


@pytest.mark.parametrize("k", ["a", "b", "c"])
def test_swizzle_matches_reference(k):
    g = _npz("swizzle.npz")
    assert np.array_equal(nvfp4.swizzle_blockscale(g[f"{k}_in"]), g[f"{k}_out"])


def test_moe_matches_reference_moe_reference():
    g = _npz("moe_ref.npz")
    y = moe.moe(g["x"], g["ids"], g["wts"], g["w13"], g["s13"], g["g13"], g["w2"], g["s2"],
                g["g2"], order="checkpoint", act_round=False)
    ref = g["y"]
    # the reference accumulates in fp32, the oracle in fp64: at most one bf16 step apart
    assert numerics.ulp_diff_bf16(y, ref).max() <= 1
    assert (numerics.ulp_diff_bf16(y, ref) == 0).mean() > 0.95


def test_moe_server_order_is_row_swap_of_checkpoint_order():
    g = _npz("moe_ref.npz")
    I = g["w13"].shape[1] // 2
    w13s = np.concatenate([g["w13"][:, I:], g["w13"][:, :I]], axis=1)
    s13s = np.concatenate([g["s13"][:, I:], g["s13"][:, :I]], axis=1)
    a = moe.moe_f64(g["x"], g["ids"], g["wts"], g["w13"], g["s13"], g["g13"], g["w2"], g["s2"],
                    g["g2"], order="checkpoint")
    b = moe.moe_f64(g["x"], g["ids"], g["wts"], w13s, s13s, g["g13"], g["w2"], g["s2"], g["g2"],
                    order="server")
    assert np.array_equal(a, b)


@pytest.mark.parametrize("key,kind,scale", [
    ("y_int8_f32s", "int8", "scale_f32"),
    ("y_int8_bf16s", "int8", "scale_bf16"),
    ("y_fp8_f32s", "fp8", "scale_f32"),
    ("y_fp8_split", "fp8", "scale_f32"),
    ("y_fp8_f32out", "fp8", "scale_f32"),
])
def test_w8a16_matches_reference_kernel(key, kind, scale):
    g = _npz("w8a16_kernel.npz")
    w = g["w_int8"] if kind == "int8" else g["w_fp8"]
    y = w8a16.gemv(g["x"], w, kind, g[scale])
    exact = w8a16.gemv_f64(g["x"], w, kind, g[scale])
    ref = g[key]
    # Under the Triton CPU interpreter the reference's bf16 casts truncate instead of
    # rounding (bench/bench/dg1/selftest_cpu.py:1-11), so outputs may sit one bf16 step
    # toward zero from the oracle's round-to-nearest; never further, never away from 0.
    den = np.abs(ref).max()
    assert np.abs(y - ref).max() / den < 2e-2
    assert numerics.ulp_diff_bf16(y, ref).max() <= 1
    off = y != ref
    assert np.all(np.abs(ref[off]) <= np.abs(exact[off]) + 1e-6 * np.abs(exact[off]))
    # its outputs are bf16 values, also in the fp32 destination (w8a16_gemv.py:92-95)
    assert np.array_equal(numerics.bf16_round(ref), ref)


def test_argmax_lowest_index_on_ties():
    logits = np.array([[1.0, 3.0, 3.0, 2.0], [5.0, 5.0, 5.0, 5.0]], dtype=np.float32)
    assert w8a16.argmax_lowest(logits).tolist() == [1, 0]


def test_bf16_round_ties_to_even():
    v = np.array([1.0, 1.00390625, 1.005859375, 1.0078125, -2.0], dtype=np.float32)
    assert numerics.bf16_bits(v).tolist() == [0x3F80, 0x3F80, 0x3F81, 0x3F81, 0xC000]


def test_e4m3_encode_saturation_and_ties():
    v = np.array([448, 449, 464, 465, 480, -500, 2**-10, 2**-9 * 1.5, 0.0], dtype=np.float32)
    assert numerics.f32_to_e4m3(v).tolist() == [126, 126, 126, 127, 127, 255, 0, 2, 0]


def _bf16_truncate(a):
    return (np.asarray(a, np.float32).view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)


@pytest.mark.parametrize("M", [1, 4])
@pytest.mark.parametrize("gate", ["silu", "sigmoid"])
def test_norm_gated_oracle_matches_reference_kernel(M, gate):
    # The reference's fused gated-RMSNorm GEMV run under the Triton CPU interpreter, whose
    # bf16 casts truncate.  With the same truncating cast the oracle reproduces it bit for
    # bit; with round-to-nearest (the GPU's cast) it stays inside the 2e-2 bar.
    g = _npz("w8a16_norm_gated.npz")
    args = (g[f"x{M}"], g[f"z{M}"], g["norm_w"], 128, 1e-6)
    sig = gate == "sigmoid"
    ref = g[f"y{M}_{gate}"]
    xt = w8a16.gated_rmsnorm(*args, sigmoid_gate=sig, bf16_cast=_bf16_truncate)
    yt = _bf16_truncate(w8a16.gemv_f64(xt, g["w_int8"], "int8", g["scale_f32"]).astype(np.float32))
    assert np.array_equal(yt, ref)
    y = w8a16.gemv_norm_gated(*args, g["w_int8"], "int8", g["scale_f32"], sigmoid_gate=sig)
    assert np.abs(y - ref).max() / np.abs(ref).max() < 2e-2


@pytest.mark.parametrize("case", ["a", "b", "c", "d"])
def test_router_topk_oracle_matches_reference_kernel(case):
    # The reference's packed-key softmax top-k (patches 0110 + 0111) under the Triton CPU
    # interpreter: ids bit-exact (ties to the lowest id, NaN floored, -0.0 as +0.0),
    # weights to fp32 rounding (the kernel's exp is ex2.approx-based), NaN rows NaN.
    g = _npz("router_topk.npz")
    k, renorm = (int(v) for v in g[f"topk_{case}"])
    w, ids = router.softmax_topk(g[f"scores_{case}"], k, bool(renorm))
    assert np.array_equal(ids, g[f"ids_{case}"])
    ref = g[f"w_{case}"]
    nan = np.isnan(ref)
    assert np.array_equal(nan, np.isnan(w))
    assert np.allclose(w[~nan], ref[~nan], rtol=2e-6, atol=1e-9)
