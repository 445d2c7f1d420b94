// Shared device building blocks of the weight-only quantized GEMV kernels (sm_100a).
//
// Every kernel in this library computes y[m, n] = sum_k W[n, k] * x[m, k] for M <= 16
// tokens by streaming the weight rows once from HBM.  The arithmetic is done on the
// tensor cores with `mma.sync.m16n8k16` in "swap-AB" form: the weights are the 16-row A
// operand and the (at most 16) tokens are the 8-wide B operand, so one instruction covers
// 256 weights and the CUDA cores only have to dequantise.
//
// Numerics (these follow the reference's own exactness argument,
// kernels/sglang/srt/layers/quantization/w4a16_nvfp4_gemv.py:25-29):
//  * an int8 weight, an fp8 e4m3 weight and an e2m1 * e4m3 NVFP4 product are all exact
//    in fp16, so the A operand is the exact dequantised weight;
//  * the activations are bf16.  They are multiplied by a per-token power of two chosen
//    from the row's max |x| (so the largest element lands in [2^14, 2^15)) and then
//    converted to fp16, which is exact for every element within 2^-31 of the row max
//    (smaller ones are rounded to the fp16 subnormal grid, an absolute error below
//    2^-40 of the row max).  The epilogue multiplies by the inverse power of two, which
//    is exact, so the result equals an fp32-accumulated dot of the bf16 inputs;
//  * accumulation is fp32 in the tensor core; the per-row scale is applied once per
//    output after the k reduction (w8a16_gemv.py:266-270) and the result is rounded to
//    bf16 before any fp32 widening (w8a16_gemv.py:92-95).
//
// k permutation.  The reduction over k is order-free, so each lane reads 16 contiguous
// bytes of a weight row (one 128-bit load) and the fragment slots of MMA j map to
// k0 = c*T + 4j + {0,1,2,3} (c = lane % 4, T = k per lane per chunk).  The B fragment of
// the same MMA then needs x[token][k0 .. k0+3], which the staging below stores in exactly
// that order, so the x fragments are conflict-free 128-bit shared-memory loads.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace fnx {

// Weight element formats (values are part of the C ABI, include/fnx_gemv.h).
enum WType : int { W_INT8 = 0, W_FP8 = 1, W_BF16 = 2, W_NVFP4 = 3 };

// Per-row (or scalar) output scale formats (C ABI values).
enum ScaleKind : int {
  SCALE_NONE = 0,      // 1.0
  SCALE_F32_SCALAR = 1,
  SCALE_F32_ROW = 2,
  SCALE_BF16_SCALAR = 3,
  SCALE_BF16_ROW = 4,
};

// One "chunk" is 64 bytes of one weight row per group of four lanes (16 B per lane).
template <int WT> struct WTraits;
template <> struct WTraits<W_INT8> { static constexpr int T = 16; };   // k per lane per chunk
template <> struct WTraits<W_FP8> { static constexpr int T = 16; };
template <> struct WTraits<W_BF16> { static constexpr int T = 8; };
template <> struct WTraits<W_NVFP4> { static constexpr int T = 32; };

template <int WT> struct Geo {
  static constexpr int T = WTraits<WT>::T;
  static constexpr int CH = 4 * T;        // k per chunk (all four lanes of a row)
  static constexpr int MMAS = T / 4;      // m16n8k16 instructions per chunk
  static constexpr int Q = T / 8;         // 16-byte x units per lane per chunk
};

// ------------------------------------------------------------------------------------
// Global loads
// ------------------------------------------------------------------------------------

// Streaming weight load: read-only path, no L1 allocation, L2 evict-first so the
// weights (read exactly once per call) do not push activations and scratch out of L2.
__device__ __forceinline__ uint4 ldg_stream(const void* p, uint64_t pol) {
  uint4 v;
  asm volatile(
      "ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p), "l"(pol));
  return v;
}

__device__ __forceinline__ uint32_t ldg_u16_stream(const void* p, uint64_t pol) {
  unsigned short v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.u16 %0, [%1], %2;"
               : "=h"(v)
               : "l"(p), "l"(pol));
  return (uint32_t)v;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Loads that must observe other CTAs' writes of this same launch (split-K partials,
// MoE partials): bypass L1.
__device__ __forceinline__ float ld_cg_f32(const float* p) {
  float v;
  asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ void st_cg_f32(float* p, float v) {
  asm volatile("st.global.cg.f32 [%0], %1;" ::"l"(p), "f"(v));
}

// ------------------------------------------------------------------------------------
// Programmatic dependent launch (the B200 form of the reference's PDL helpers,
// kernels/sglang/kernels/triton_pdl.py:60-83).  Both are no-ops when the launch did
// not set the programmatic-serialization attribute.
// ------------------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Named barrier over `nthreads` threads (a group of warps inside the CTA).
__device__ __forceinline__ void group_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------------------------------------------
// Dequantisation of one 32-bit word of a weight row into two fp16x2 A-fragment halves:
// `lo` holds k0, k0+1 and `hi` holds k0+2, k0+3 (low half = lower k).
// ------------------------------------------------------------------------------------

// int8: XOR 0x80 maps the signed byte b to u = b + 128; 0x6400 | u is the fp16 value
// 1024 + u, and subtracting 1152 leaves b exactly.
__device__ __forceinline__ void deq_int8_word(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  uint32_t a = __byte_perm(u, 0x64646464u, 0x4140);
  uint32_t b = __byte_perm(u, 0x64646464u, 0x4342);
  const uint32_t bias = 0x64806480u;  // fp16 1152.0 in both halves
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(lo) : "r"(a), "r"(bias));
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(hi) : "r"(b), "r"(bias));
}

// fp8 e4m3: native packed conversion (lower byte -> lower half).
__device__ __forceinline__ void deq_fp8_word(uint32_t w, uint32_t& lo, uint32_t& hi) {
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(lo) : "h"((unsigned short)(w & 0xFFFFu)));
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(hi) : "h"((unsigned short)(w >> 16)));
}

// NVFP4: four bytes = eight e2m1 codes, low nibble = even k
// (w4a16_nvfp4_gemv.py:7-8).  Each byte becomes one fp16x2 (low nibble -> low half).
__device__ __forceinline__ void deq_e2m1_word(uint32_t w, uint32_t (&h)[4]) {
  asm("{\n\t.reg .b8 q0, q1, q2, q3;\n\t"
      "mov.b32 {q0, q1, q2, q3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, q0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, q1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, q2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, q3;\n\t}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(w));
}

// Two e4m3 block scales (lower byte = lower k block) -> fp16x2.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two_bytes) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"((unsigned short)two_bytes));
  return r;
}

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Broadcast the low / high fp16 of a pair to both halves.
__device__ __forceinline__ uint32_t bcast_lo(uint32_t v) { return __byte_perm(v, 0, 0x1010); }
__device__ __forceinline__ uint32_t bcast_hi(uint32_t v) { return __byte_perm(v, 0, 0x3232); }

// ------------------------------------------------------------------------------------
// Tensor-core MMA (fp32 accumulate).
// ------------------------------------------------------------------------------------
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ------------------------------------------------------------------------------------
// One chunk of one lane: 16 B of row g (va) and row g+8 (vb), their NVFP4 block scales
// (sa, sb: two e4m3 bytes each) and the B fragments; accumulates into acc[nt][4].
// xs points at this lane's 16-byte x units for token (nt*8 + g); the unit q of the
// chunk holds k0 .. k0+7 of MMAs 2q and 2q+1.
// ------------------------------------------------------------------------------------
template <int WT, int NT>
__device__ __forceinline__ void chunk_mma(float (&acc0)[NT][4], float (&acc1)[NT][4],
                                          const uint4& va, const uint4& vb, uint32_t sa,
                                          uint32_t sb, const uint4 (&xf)[NT][Geo<WT>::Q],
                                          int nt_act = NT) {
  // MMAs alternate between two accumulator sets (even / odd j) so that consecutive
  // tensor-core instructions do not wait on each other's results.
  const uint32_t wa[4] = {va.x, va.y, va.z, va.w};
  const uint32_t wb[4] = {vb.x, vb.y, vb.z, vb.w};
  if constexpr (WT == W_INT8 || WT == W_FP8) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t a0, a2, a1, a3;
      if constexpr (WT == W_INT8) {
        deq_int8_word(wa[j], a0, a2);
        deq_int8_word(wb[j], a1, a3);
      } else {
        deq_fp8_word(wa[j], a0, a2);
        deq_fp8_word(wb[j], a1, a3);
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        if (nt >= nt_act) break;
        const uint4& u = xf[nt][j >> 1];
        const uint32_t b0 = (j & 1) ? u.z : u.x;
        const uint32_t b1 = (j & 1) ? u.w : u.y;
        mma_f16((j & 1) ? acc1[nt] : acc0[nt], a0, a1, a2, a3, b0, b1);
      }
    }
  } else if constexpr (WT == W_BF16) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint32_t a0 = wa[2 * j], a2 = wa[2 * j + 1];
      const uint32_t a1 = wb[2 * j], a3 = wb[2 * j + 1];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        if (nt >= nt_act) break;
        const uint4& u = xf[nt][0];
        const uint32_t b0 = j ? u.z : u.x;
        const uint32_t b1 = j ? u.w : u.y;
        mma_bf16(j ? acc1[nt] : acc0[nt], a0, a1, a2, a3, b0, b1);
      }
    }
  } else {  // W_NVFP4
    const uint32_t sfa = e4m3x2_to_f16x2(sa);
    const uint32_t sfb = e4m3x2_to_f16x2(sb);
    const uint32_t sa0 = bcast_lo(sfa), sa1 = bcast_hi(sfa);
    const uint32_t sb0 = bcast_lo(sfb), sb1 = bcast_hi(sfb);
#pragma unroll
    for (int q = 0; q < 4; ++q) {  // word q serves MMAs 2q (byte 0,1) and 2q+1 (byte 2,3)
      uint32_t ha[4], hb[4];
      deq_e2m1_word(wa[q], ha);
      deq_e2m1_word(wb[q], hb);
      const uint32_t s_a = (q < 2) ? sa0 : sa1;
      const uint32_t s_b = (q < 2) ? sb0 : sb1;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int j = 2 * q + h;
        const uint32_t a0 = hmul2(ha[2 * h], s_a);
        const uint32_t a2 = hmul2(ha[2 * h + 1], s_a);
        const uint32_t a1 = hmul2(hb[2 * h], s_b);
        const uint32_t a3 = hmul2(hb[2 * h + 1], s_b);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          if (nt >= nt_act) break;
          const uint4& u = xf[nt][j >> 1];
          const uint32_t b0 = (j & 1) ? u.z : u.x;
          const uint32_t b1 = (j & 1) ? u.w : u.y;
          mma_f16(h ? acc1[nt] : acc0[nt], a0, a1, a2, a3, b0, b1);
        }
      }
    }
  }
}

// ------------------------------------------------------------------------------------
// Activation staging.  A staged row (token or MoE route pair) is K fp16 (or bf16 for a
// bf16 weight) stored in 16-byte units; unit (chunk, q, c) holds
// k = chunk*CH + c*T + q*8 .. +7 at byte offset ((chunk*Q + q)*4 + c)*16.  The row
// stride is 2K + 64 bytes, so the eight lanes of one 128-bit load phase (two rows, four
// lanes each) hit eight distinct 16-byte bank groups.
// ------------------------------------------------------------------------------------
__host__ __device__ constexpr int stage_row_bytes(int K) { return 2 * K + 64; }

template <int WT>
__device__ __forceinline__ int stage_unit_offset(int k) {  // k multiple of 8
  constexpr int CH = Geo<WT>::CH, T = Geo<WT>::T, Q = Geo<WT>::Q;
  const int chunk = k / CH;
  const int rem = k - chunk * CH;
  const int c = rem / T;
  const int q = (rem - c * T) >> 3;
  return ((chunk * Q + q) * 4 + c) * 16;
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b16) {
  return __uint_as_float(b16 << 16);
}

// Exponent e such that max_abs * 2^e lies in [2^14, 2^15); 0 for an all-zero row.
__device__ __forceinline__ int stage_exponent(float max_abs) {
  if (!(max_abs > 0.f)) return 0;
  const uint32_t bits = __float_as_uint(max_abs);
  int ex = (int)((bits >> 23) & 0xFF) - 127;  // floor(log2) for normals; -127 for denormals
  int e = 14 - ex;
  if (e > 100) e = 100;
  if (e < -40) e = -40;
  return e;
}

__device__ __forceinline__ float pow2f(int e) {  // exact for e in [-126, 127]
  return __uint_as_float((uint32_t)(e + 127) << 23);
}

// Convert 8 bf16 (a 16-byte vector) to 8 fp16 scaled by 2^e (e in [-40, 100], so the
// factor is a normal float and the multiply is exact before the fp16 rounding).
__device__ __forceinline__ uint4 bf16x8_to_f16x8_scaled(const uint4 v, int e) {
  const float f = pow2f(e);
  const uint32_t in[4] = {v.x, v.y, v.z, v.w};
  uint32_t out[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float lo = bf16_bits_to_f32(in[i] & 0xFFFFu) * f;
    const float hi = bf16_bits_to_f32(in[i] >> 16) * f;
    const __half2 h = __floats2half2_rn(lo, hi);
    out[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

__device__ __forceinline__ float bf16x8_absmax(const uint4 v) {
  const uint32_t in[4] = {v.x, v.y, v.z, v.w};
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m = fmaxf(m, fabsf(bf16_bits_to_f32(in[i] & 0xFFFFu)));
    m = fmaxf(m, fabsf(bf16_bits_to_f32(in[i] >> 16)));
  }
  return m;
}

// Order-preserving 16-bit key of a bf16 value for the greedy argmax: larger value ->
// larger key; -0 is folded onto +0 so that equal logits tie (torch.argmax semantics).
__device__ __forceinline__ uint32_t bf16_order_key(uint32_t b) {
  b &= 0xFFFFu;
  if (b == 0x8000u) b = 0;
  return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
}

// argmax key: value key in the high 32 bits, (0xFFFFFFFF - index) in the low 32 bits, so
// the maximum key is the largest value and, among equal values, the lowest index.
__device__ __forceinline__ unsigned long long argmax_key(uint32_t bf16_bits, uint32_t index) {
  return ((unsigned long long)bf16_order_key(bf16_bits) << 32) |
         (unsigned long long)(0xFFFFFFFFu - index);
}

__device__ __forceinline__ float load_row_scale(const void* scale, int kind, int64_t n) {
  switch (kind) {
    case SCALE_F32_SCALAR: return __ldg(reinterpret_cast<const float*>(scale));
    case SCALE_F32_ROW: return __ldg(reinterpret_cast<const float*>(scale) + n);
    case SCALE_BF16_SCALAR:
      return bf16_bits_to_f32(__ldg(reinterpret_cast<const unsigned short*>(scale)));
    case SCALE_BF16_ROW:
      return bf16_bits_to_f32(__ldg(reinterpret_cast<const unsigned short*>(scale) + n));
    default: return 1.f;
  }
}

__device__ __forceinline__ float silu_f32(float g) { return g / (1.0f + expf(-g)); }

__device__ __forceinline__ uint4 ldg_cg_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// The two-pass fp16 staging of the columns [kb, ke) of activation rows (multiples of 8;
// shared memory holds exactly that range, row stride stage_row_bytes(ke - kb)) from
// produced 16-byte units.  Work item idx is row r = idx / ((ke - kb) / 8) and unit
// u = kb / 8 + idx % ((ke - kb) / 8); unit(in, r, u) returns its 8 bf16 values (zeros
// when in is false, past the last item).  Every lane of a warp calls it together, on 32
// consecutive items starting at a multiple of 32, so it may use warp shuffles.  Pass 1
// finds each row's max |value| over the range, pass 2 converts with the row's power of
// two (fp16); unscale[r] receives the inverse power of two
// that the epilogue applies, or 0 where has_row(r) is false.  Threads t0 .. t0 + nth - 1
// (whole warps) take part and synchronise on named barrier bar_id; unscale[] has room for
// 2 x 16 words: [16, 32) collects the row maxima as float bits (non-negative floats
// order like their bits).
template <int WT, typename RowFn, typename UnitFn>
__device__ __forceinline__ void stage_units_f16(uint8_t* xs, float* unscale, int nrows, int kb,
                                                int ke, RowFn has_row, UnitFn unit, int t0,
                                                int nth, int bar_id) {
  const int tid = threadIdx.x - t0, lane = threadIdx.x & 31;
  const int srow = stage_row_bytes(ke - kb);
  const int upr = (ke - kb) >> 3, u0 = kb >> 3;
  const int total = nrows * upr;
  unsigned* smax = reinterpret_cast<unsigned*>(unscale + 16);
  for (int r = tid; r < nrows; r += nth) smax[r] = 0u;
  group_sync(bar_id, nth);
  auto at = [&](int idx) -> uint4 {
    const bool in = idx < total;
    const int r = in ? idx / upr : 0;
    return unit(in, r, u0 + (in ? idx - r * upr : 0));
  };
  constexpr int kHold = 4;  // units kept in registers between the two passes
  const int wbase = tid - lane;  // first work item of this warp (warp-uniform loops)
  uint4 held[kHold];
  // Row maximum of one unit per lane: one atomic per warp when the warp's units all
  // lie in one row, else one per lane.
  auto row_max = [&](int idx, const uint4 v) {
    const int r = idx < total ? idx / upr : -1;
    unsigned bits = __float_as_uint(bf16x8_absmax(v));
    const int r0 = __shfl_sync(0xffffffffu, r, 0);
    if (__all_sync(0xffffffffu, r == r0)) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) bits = max(bits, __shfl_xor_sync(0xffffffffu, bits, o));
      if (lane == 0 && r0 >= 0) atomicMax(&smax[r0], bits);
    } else if (r >= 0) {
      atomicMax(&smax[r], bits);
    }
  };
#pragma unroll
  for (int j = 0; j < kHold; ++j) held[j] = at(tid + j * nth);
#pragma unroll
  for (int j = 0; j < kHold; ++j)
    if (wbase + j * nth < total) row_max(tid + j * nth, held[j]);
  for (int b = wbase + kHold * nth; b < total; b += kHold * nth) {  // batches of kHold
    uint4 v[kHold];
#pragma unroll
    for (int j = 0; j < kHold; ++j) v[j] = at(b + lane + j * nth);
#pragma unroll
    for (int j = 0; j < kHold; ++j)
      if (b + j * nth < total) row_max(b + lane + j * nth, v[j]);
  }
  group_sync(bar_id, nth);
  auto put = [&](int idx, const uint4 v) {
    if (idx >= total) return;
    const int r = idx / upr, u = idx - r * upr;
    const int e = stage_exponent(__uint_as_float(smax[r]));
    *reinterpret_cast<uint4*>(xs + (size_t)r * srow + stage_unit_offset<WT>(8 * u)) =
        bf16x8_to_f16x8_scaled(v, e);
  };
#pragma unroll
  for (int j = 0; j < kHold; ++j) put(tid + j * nth, held[j]);
  for (int b = wbase + kHold * nth; b < total; b += kHold * nth) {
    uint4 v[kHold];
#pragma unroll
    for (int j = 0; j < kHold; ++j) v[j] = at(b + lane + j * nth);
#pragma unroll
    for (int j = 0; j < kHold; ++j) put(b + lane + j * nth, v[j]);
  }
  for (int r = tid; r < nrows; r += nth)
    unscale[r] = has_row(r) ? pow2f(-stage_exponent(__uint_as_float(smax[r]))) : 0.f;
}

// The bf16 form (bf16 weights): the units are copied unchanged, unscale[r] = 1 (or 0).
template <int WT, typename RowFn, typename UnitFn>
__device__ __forceinline__ void stage_units_bf16(uint8_t* xs, float* unscale, int nrows, int kb,
                                                 int ke, RowFn has_row, UnitFn unit, int t0,
                                                 int nth) {
  const int tid = threadIdx.x - t0, lane = threadIdx.x & 31;
  const int srow = stage_row_bytes(ke - kb);
  const int upr = (ke - kb) >> 3, u0 = kb >> 3;
  const int total = nrows * upr;
  for (int b = tid - lane; b < total; b += nth) {  // warp-uniform: unit() may shuffle
    const int idx = b + lane;
    const bool in = idx < total;
    const int r = in ? idx / upr : 0;
    const int u = in ? idx - r * upr : 0;
    const uint4 v = unit(in, r, u0 + u);
    if (in) *reinterpret_cast<uint4*>(xs + (size_t)r * srow + stage_unit_offset<WT>(8 * u)) = v;
  }
  for (int r = tid; r < nrows; r += nth) unscale[r] = has_row(r) ? 1.f : 0.f;
}

// Stage the columns [kb, ke) of `nrows` activation rows of bf16 into shared memory in
// the fragment order above (column kb first).  Row r is read from src(r) (a bf16 pointer, or nullptr for a
// row that is never used): converted to fp16 with the row's power of two
// (stage_units_f16), or copied unchanged (bf16 weights).  Reads use ld.global.cg: the
// rows may have been written by the previous kernel of a programmatic-dependent pair.
// Callers synchronise the participating threads (named barrier bar_id) after the call.
template <int WT, typename SrcFn>
__device__ __forceinline__ void stage_rows(uint8_t* xs, float* unscale, int nrows, int kb,
                                           int ke, SrcFn src, int t0, int nth, int bar_id) {
  auto has_row = [&](int r) { return src(r) != nullptr; };
  auto unit = [&](bool in, int r, int u) -> uint4 {
    const __nv_bfloat16* p = in ? src(r) : nullptr;
    return p ? ldg_cg_u4(p + 8 * u) : make_uint4(0u, 0u, 0u, 0u);
  };
  if constexpr (WT == W_BF16)
    stage_units_bf16<WT>(xs, unscale, nrows, kb, ke, has_row, unit, t0, nth);
  else
    stage_units_f16<WT>(xs, unscale, nrows, kb, ke, has_row, unit, t0, nth, bar_id);
}

// Gated RMSNorm folded into the activation load (the prologue of w8a16_gemv_norm_gated,
// w8a16_gemv.py:186-190, :220-233, :246-255): every contiguous G-value slice of a row is
// one RMS group and y = x * rsqrt(sum(x^2) / G + eps) * w[k % G] * gate(z), with
// gate(z) = z * sigmoid(z) (silu) or sigmoid(z), cast to bf16 (round to nearest even)
// before the dot.  G is a power of two in [8, 256].
struct NormGate {
  const __nv_bfloat16* z;  // [M, K] bf16 gates, row stride ldz elements
  int64_t ldz;
  const void* w;           // [G] norm weight, bf16 or fp32 (w_f32)
  int w_f32;
  int G;
  float eps;
  int sigmoid;
};

// One 16-byte unit (8 values at row offset k0) of the normalised row.  All 32 lanes call
// it together on 32 consecutive units starting at a multiple of 32: a group's G/8 units
// are then G/8 consecutive lanes, which add their sums of squares with shuffles.
__device__ __forceinline__ uint4 norm_gated_unit(const uint4 xv, const uint4 zv, int k0,
                                                 const NormGate& ng) {
  const uint32_t xin[4] = {xv.x, xv.y, xv.z, xv.w};
  const uint32_t zin[4] = {zv.x, zv.y, zv.z, zv.w};
  float xf[8], zf[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    xf[2 * i] = bf16_bits_to_f32(xin[i] & 0xFFFFu);
    xf[2 * i + 1] = bf16_bits_to_f32(xin[i] >> 16);
    zf[2 * i] = bf16_bits_to_f32(zin[i] & 0xFFFFu);
    zf[2 * i + 1] = bf16_bits_to_f32(zin[i] >> 16);
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss = fmaf(xf[i], xf[i], ss);
  for (int o = 1; o < (ng.G >> 3); o <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rstd = rsqrtf(ss * (1.f / (float)ng.G) + ng.eps);  // 1/G is exact
  const int kw = k0 & (ng.G - 1);
  float nw[8];
  if (ng.w_f32) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(ng.w) + (kw >> 2));
    const float4 b = __ldg(reinterpret_cast<const float4*>(ng.w) + (kw >> 2) + 1);
    nw[0] = a.x; nw[1] = a.y; nw[2] = a.z; nw[3] = a.w;
    nw[4] = b.x; nw[5] = b.y; nw[6] = b.z; nw[7] = b.w;
  } else {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(ng.w) + (kw >> 3));
    const uint32_t in[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      nw[2 * i] = bf16_bits_to_f32(in[i] & 0xFFFFu);
      nw[2 * i + 1] = bf16_bits_to_f32(in[i] >> 16);
    }
  }
  uint32_t out[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float y[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float z = zf[2 * i + h];
      const float sg = __fdividef(1.f, 1.f + __expf(-z));  // 0 where exp overflows
      y[h] = xf[2 * i + h] * rstd * nw[2 * i + h] * (ng.sigmoid ? sg : z * sg);
    }
    const __nv_bfloat162 b = __floats2bfloat162_rn(y[0], y[1]);
    out[i] = *reinterpret_cast<const uint32_t*>(&b);
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

// ------------------------------------------------------------------------------------
// Asynchronous pipeline primitives: mbarriers and bulk (TMA) copies into shared memory.
// Every wait is bounded: after kWaitLimitNs of polling it reports failure, and the
// caller records an error code and leaves its loop instead of spinning forever.
// ------------------------------------------------------------------------------------
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

// Device error codes (C ABI values, FNX_DEVERR_* in include/fnx_gemv.h).
enum ErrCode : int { ERR_NONE = 0, ERR_WAIT_FULL = 1, ERR_WAIT_EMPTY = 2, ERR_WAIT_RED = 3,
                     ERR_WAIT_RFREE = 4, ERR_DRAIN = 5, ERR_WAIT_X = 6, ERR_WAIT_PEER = 7,
                     ERR_PEER_DESYNC = 8, ERR_ROUTES = 9, ERR_WAIT_EXPERT = 10,
                     ERR_RING = 11 };

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Arrive once and announce `bytes` of bulk-copy transactions for the current phase.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// As mbar_test, but a thread whose phase has not completed is suspended (it issues no
// instructions) until the phase completes or about `suspend_ns` nanoseconds pass, so
// waiting warps leave the issue slots to the warps that have work.
__device__ __forceinline__ bool mbar_test_suspend(uint64_t* bar, uint32_t parity,
                                                  uint32_t suspend_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(suspend_ns)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait until the phase with the given parity has completed; false after the time limit.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_test(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (;;) {
    if (mbar_test_suspend(bar, parity, 1000000u)) return true;
    if (global_ns() - t0 > kWaitLimitNs) return false;
  }
}

// Generic-proxy writes to shared memory become ordered before later async-proxy (bulk
// copy) accesses of the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Load with acquire semantics at GPU scope: writes released before the value this load
// returns (by a release or acq_rel atomic, or a fence ahead of a relaxed one) are visible to
// this thread's later reads.
__device__ __forceinline__ unsigned ld_acquire_gpu_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Atomic add with acquire-release semantics at GPU scope: this thread's earlier writes
// (and those ordered before them, e.g. by __syncwarp) are visible to whoever observes the
// new value, and the returned old value carries the writes of earlier releasers.
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Bulk copy global -> this CTA's shared memory, completing `bytes` on the mbarrier.
// dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

// Asynchronous 4/8/16-byte global -> shared copies (cp.async) whose completion this
// thread later hands to an mbarrier with cp_async_arrive (one arrival, counted in the
// barrier's expected count).  Source and destination must be aligned to the size.
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ uint4 lds128(const uint8_t* p) {
  return *reinterpret_cast<const uint4*>(p);
}

// ------------------------------------------------------------------------------------
// Shared-memory tile layout.  A 16-row weight tile is stored as two halves of 8 rows
// (physical rows 0..7 and 8..15), each at a row pitch of UB bytes, the second half
// starting `tile_half_offset(UB)` bytes in; a half is one contiguous bulk copy when the
// rows are contiguous in global memory.  The eight lanes of one 128-bit load phase hold
// MMA rows g0 and g0 + 1 (g0 even); lanes with an odd g read the other half (MMA row g is
// physical row g + 8 and vice versa), and the half offset puts the two rows of a phase
// 64 bytes apart modulo 128, so the phase touches eight distinct bank groups.
// ------------------------------------------------------------------------------------
__host__ __device__ constexpr int tile_half_offset(int ub) {
  return 8 * ub + ((64 - (ub % 128)) % 128 + 128) % 128;
}
__host__ __device__ constexpr int tile_bytes(int ub) {
  return ((tile_half_offset(ub) + 8 * ub) + 127) / 128 * 128;
}
// A persistent CTA's units are u0, u0 + step, ...  UnitCursor walks them, with
// u / div and u % div and the ring stage (ordinal % ns) and its phase parity
// ((ordinal / ns) & 1), without a division per unit.
struct UnitCursor {
  int u, q, r, s, ph;
  int dq, dr, div, ns, step;
  __device__ __forceinline__ void init(int u0, int step_, int div_, int ns_) {
    step = step_;
    div = div_;
    ns = ns_;
    u = u0;
    q = u0 / div_;
    r = u0 - q * div_;
    dq = step_ / div_;
    dr = step_ - dq * div_;
    s = 0;
    ph = 0;
  }
  __device__ __forceinline__ void next() {
    u += step;
    q += dq;
    r += dr;
    if (r >= div) {
      r -= div;
      ++q;
    }
    if (++s == ns) {
      s = 0;
      ph ^= 1;
    }
  }
};

// Physical row of MMA row g (0..7) and of MMA row g + 8, for the lane's g.
__device__ __forceinline__ int phys_lo(int g) { return (g & 1) ? g + 8 : g; }
__device__ __forceinline__ int phys_hi(int g) { return (g & 1) ? g : g + 8; }
__device__ __forceinline__ int tile_row_offset(int r, int ub) {
  return r < 8 ? r * ub : tile_half_offset(ub) + (r - 8) * ub;
}

// Stage the columns [kb, ke) of the first nrows activation rows like stage_rows, with
// the rows brought in by the bulk-copy engine: issue_x_rows (called once, by one thread
// of the CTA, before or during this call) copies each raw bf16 row into its own
// shared-memory slot, completing on xbar (phase 0), so the whole block arrives after one
// memory latency.  With `direct` (one or two rows, where the copy engine's latency is
// not repaid) no copy is issued and pass 1 loads the units from global memory itself.  The participating warps then split the
// rows into segments of whole 32-unit batches (several warps per row when there are few
// rows) and, with no division in the loops:
//   pass 1: each lane keeps a running max |value| over its units (with the fused norm,
//           NORM, it first replaces each unit by its normalised, gated bf16 value,
//           z read from global memory); one warp reduction and one shared atomic per
//           segment give the row maxima;
//   pass 2: each unit is converted to fp16 with its row's power of two and moved to its
//           fragment slot (a permutation inside its weight chunk: a warp reads its 32
//           units, which cover whole chunks, before writing them back).
// x rows, ldx and kb keep 16-byte alignment; with the norm, kb and ke are multiples of
// the group.  An expired wait records ERR_WAIT_X and stages nothing further.
// The bulk copies of stage_rows_bulk, issued by one thread: the raw bf16 columns
// [kb, ke) of rows 0 .. nrows - 1 into their shared-memory row slots, completing on xbar.
__device__ __forceinline__ void issue_x_rows(uint8_t* xs, int nrows, int kb, int ke,
                                             const __nv_bfloat16* x, int64_t ldx, uint64_t* xbar) {
  const int kx = ke - kb;
  const int srow = stage_row_bytes(kx);
  mbar_arrive_expect_tx(xbar, (uint32_t)(nrows * kx * 2));
  const uint64_t pol = policy_evict_last();  // every CTA reads the same rows
  for (int r = 0; r < nrows; ++r)
    bulk_g2s(xs + (size_t)r * srow, x + (size_t)r * ldx + kb, (uint32_t)(kx * 2), xbar, pol);
}

template <int WT, bool NORM>
__device__ __forceinline__ void stage_rows_bulk(uint8_t* xs, float* unscale, int nrows, int kb,
                                                int ke, const __nv_bfloat16* x, int64_t ldx,
                                                const NormGate ng, uint64_t* xbar, int* err,
                                                bool direct, int t0, int nth, int bar_id) {
  const int tid = threadIdx.x - t0, lane = threadIdx.x & 31;
  const int kx = ke - kb;
  const int srow = stage_row_bytes(kx);
  const int upr = kx >> 3;                      // 16-byte units per row
  const int nwarps = nth >> 5, w = tid >> 5;
  const int segs = max(1, min(nwarps / nrows, (upr + 31) >> 5));  // warps per row
  const int seg_len = ((upr + segs - 1) / segs + 31) & ~31;         // units, whole batches
  const int tasks = nrows * segs;
  unsigned* smax = reinterpret_cast<unsigned*>(unscale + 16);
  for (int r = tid; r < nrows; r += nth) smax[r] = 0u;
  group_sync(bar_id, nth);
  if (!direct && !mbar_wait(xbar, 0)) {
    record_error(err, ERR_WAIT_X);
    return;
  }
  if constexpr (WT == W_BF16 && !NORM) {  // the raw rows are the fragment layout already
    if (direct)
      for (int i = tid; i < nrows * upr; i += nth) {
        const int r = i / upr, u = i - r * upr;
        *reinterpret_cast<uint4*>(xs + (size_t)r * srow + u * 16) =
            ldg_cg_u4(x + (size_t)r * ldx + kb + 8 * u);
      }
    for (int r = tid; r < nrows; r += nth) unscale[r] = 1.f;
  } else {
    for (int task = w; task < tasks; task += nwarps) {  // pass 1
      const int r = task / segs, sg = task - r * segs;
      const int u0 = sg * seg_len, u1 = min(upr, u0 + seg_len);
      uint8_t* row = xs + (size_t)r * srow;
      float m = 0.f;
      for (int b = u0; b < u1; b += 64) {  // two batches per step, warp-uniform
        uint4 v[2], zv[2];
        bool in[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // all loads of the step first
          const int u = b + 32 * h + lane;
          in[h] = u < u1;
          v[h] = zv[h] = make_uint4(0u, 0u, 0u, 0u);
          if (in[h]) v[h] = direct ? ldg_cg_u4(x + (size_t)r * ldx + kb + 8 * u) : lds128(row + u * 16);
          if constexpr (NORM)
            if (in[h]) zv[h] = ldg_cg_u4(ng.z + (size_t)r * ng.ldz + kb + 8 * u);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int u = b + 32 * h + lane;
          if constexpr (NORM) v[h] = norm_gated_unit(v[h], zv[h], kb + 8 * u, ng);
          if (in[h] && (NORM || direct)) *reinterpret_cast<uint4*>(row + u * 16) = v[h];
          if (in[h]) m = fmaxf(m, bf16x8_absmax(v[h]));
        }
      }
      unsigned bits = __float_as_uint(m);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) bits = max(bits, __shfl_xor_sync(0xffffffffu, bits, o));
      if (lane == 0 && u0 < u1) atomicMax(&smax[r], bits);
    }
    group_sync(bar_id, nth);
    if constexpr (WT == W_BF16) {  // normalised rows, already in the fragment layout
      for (int r = tid; r < nrows; r += nth) unscale[r] = 1.f;
    } else {
      for (int task = w; task < tasks; task += nwarps) {  // pass 2
        const int r = task / segs, sg = task - r * segs;
        const int u0 = sg * seg_len, u1 = min(upr, u0 + seg_len);
        uint8_t* row = xs + (size_t)r * srow;
        const int e = stage_exponent(__uint_as_float(smax[r]));
        for (int b = u0; b < u1; b += 32) {  // warp-uniform
          const int u = b + lane;
          const bool in = u < u1;
          uint4 v = make_uint4(0u, 0u, 0u, 0u);
          if (in) v = bf16x8_to_f16x8_scaled(lds128(row + u * 16), e);
          __syncwarp();  // every lane has read its raw unit before any lane overwrites a chunk
          if (in) *reinterpret_cast<uint4*>(row + stage_unit_offset<WT>(8 * u)) = v;
        }
      }
      for (int r = tid; r < nrows; r += nth)
        unscale[r] = pow2f(-stage_exponent(__uint_as_float(smax[r])));
    }
  }
}

}  // namespace fnx
