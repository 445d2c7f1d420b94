// NVFP4 load-time codec on the GPU: quantise a [N, K] bf16 / fp32 weight to packed e2m1
// codes + e4m3 block-16 scales + one fp32 global scale, and dequantise back.
//
// The codes must be bit-identical to the reference's quantiser (the ModelOpt convention of
// kernels/sglang/srt/layers/quantization/w4a16_nvfp4_gemv.py:426-472), so the fp32 steps
// follow its order exactly, each an IEEE-rounded operation:
//   gscale = max(amax(|W|) / (448 * 6), 1e-30);   enc = 1 / gscale
//   per 16-value block b:  sb = min(max((amax_b / 6) * enc, 0), 448)  -> e4m3, nearest-even
//                          eff = float(e4m3) / enc
//                          code = nearest-even e2m1 of (w / eff)  (saturating at 6), sign
//                                 from w / eff < 0 (so -0 encodes as +0), 0 when eff == 0
// The two roundings are the hardware conversions cvt.rn.satfinite.{e4m3x2,e2m1x2}.f32:
// round to nearest with ties to the even code is exactly the reference's
// bucketize-with-tie-correction rule (w4a16_nvfp4_gemv.py:410-423).
// Dequantisation: value = e2m1(code) * (e4m3(bs) * gscale) in fp32 (w4a16_nvfp4_gemv.py:
// 489-510: the scale product first, then the code times it).
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>

#include "fnx_common.cuh"

namespace fnx {

namespace {

__device__ __forceinline__ float load_w(const void* w, int64_t ldw, int w_f32, int64_t n, int64_t k) {
  if (w_f32) return reinterpret_cast<const float*>(w)[n * ldw + k];
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(w)[n * ldw + k]);
}

__device__ __forceinline__ uint32_t f32_to_e4m3_rn(float v) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.f), "f"(v));
  return r & 0xFFu;  // v in the low byte
}

__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
  const uint32_t h2 = e4m3x2_to_f16x2(b & 0xFFu);  // low half = the byte's value
  return __half2float(__ushort_as_half((unsigned short)(h2 & 0xFFFFu)));
}

// Two values -> one byte of e2m1 codes (lo in the low nibble).
__device__ __forceinline__ uint32_t f32x2_to_e2m1(float lo, float hi) {
  uint16_t r;
  asm("{\n\t.reg .b8 t;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\t"
      "cvt.u16.u8 %0, t;\n\t}"
      : "=h"(r)
      : "f"(hi), "f"(lo));
  return r & 0xFFu;
}

__device__ __forceinline__ float e2m1_to_f32(uint32_t code) {
  const float mag[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  const float m = mag[code & 7u];
  return (code & 8u) ? -m : m;
}

// max |w| over the matrix as float bits into *amax (non-negative floats order like
// their bits); *amax is zero on entry.
__global__ void __launch_bounds__(256) absmax_kernel(const void* w, int64_t ldw, int w_f32, int N,
                                                    int K, unsigned* amax) {
  __shared__ unsigned wmax[8];
  float m = 0.f;
  const int64_t total = (int64_t)N * K;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / K, k = i - n * K;
    m = fmaxf(m, fabsf(load_w(w, ldw, w_f32, n, k)));
  }
  unsigned bits = __float_as_uint(m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) bits = max(bits, __shfl_xor_sync(0xffffffffu, bits, o));
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = bits;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned b = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) b = max(b, wmax[i]);
    atomicMax(amax, b);
  }
}

// One thread per 16-value block (row n, block b).
__global__ void __launch_bounds__(256) quantize_kernel(const void* w, int64_t ldw, int w_f32, int N,
                                                      int K, uint8_t* wq, int64_t ldwq,
                                                      uint8_t* bs, int64_t ldbs, float* gscale,
                                                      const unsigned* amax) {
  const int nb = K / 16;
  const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const float gmax = __uint_as_float(*amax);
  const float gs = fmaxf(gmax / 2688.f, 1e-30f);
  const float enc = 1.f / gs;
  if (q == 0) *gscale = gs;
  if (q >= (int64_t)N * nb) return;
  const int64_t n = q / nb;
  const int b = (int)(q - n * nb);
  float v[16];
  float am = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    v[i] = load_w(w, ldw, w_f32, n, (int64_t)b * 16 + i);
    am = fmaxf(am, fabsf(v[i]));
  }
  const float sb = fminf(fmaxf((am / 6.f) * enc, 0.f), 448.f);
  const uint32_t s8 = f32_to_e4m3_rn(sb);
  const float eff = e4m3_to_f32(s8) / enc;
  uint32_t words[2] = {0u, 0u};
  if (eff > 0.f) {
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      float a0 = v[i] / eff, a1 = v[i + 1] / eff;
      a0 = a0 == 0.f ? 0.f : a0;  // -0 encodes as +0 (the sign comes from a < 0)
      a1 = a1 == 0.f ? 0.f : a1;
      words[i >> 3] |= f32x2_to_e2m1(a0, a1) << (8 * ((i >> 1) & 3));
    }
  }
  uint2* dst = reinterpret_cast<uint2*>(wq + n * ldwq + (int64_t)b * 8);
  *dst = make_uint2(words[0], words[1]);
  bs[n * ldbs + b] = (uint8_t)s8;
}

__global__ void __launch_bounds__(256) dequantize_kernel(const uint8_t* wq, int64_t ldwq,
                                                        const uint8_t* bs, int64_t ldbs,
                                                        const float* gscale, int per_row,
                                                        void* out, int64_t ldo, int out_f32,
                                                        int N, int K) {
  const int nb = K / 16;
  const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= (int64_t)N * nb) return;
  const int64_t n = q / nb;
  const int b = (int)(q - n * nb);
  const float g = per_row ? gscale[n] : gscale[0];
  const float s = e4m3_to_f32(bs[n * ldbs + b]) * g;
  const uint2 cw = *reinterpret_cast<const uint2*>(wq + n * ldwq + (int64_t)b * 8);
  const uint32_t words[2] = {cw.x, cw.y};
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint32_t code = (words[i >> 3] >> (4 * (i & 7))) & 0xFu;
    const float val = e2m1_to_f32(code) * s;
    const int64_t k = (int64_t)b * 16 + i;
    if (out_f32) reinterpret_cast<float*>(out)[n * ldo + k] = val;
    else reinterpret_cast<__nv_bfloat16*>(out)[n * ldo + k] = __float2bfloat16_rn(val);
  }
}

}  // namespace

int launch_nvfp4_quantize(const void* w, int64_t ldw, int w_f32, int N, int K, uint8_t* wq,
                          int64_t ldwq, uint8_t* bs, int64_t ldbs, float* gscale,
                          unsigned* scratch, cudaStream_t stream) {
  if (cudaMemsetAsync(scratch, 0, sizeof(unsigned), stream) != cudaSuccess) return 2;
  const int64_t total = (int64_t)N * K;
  const int g1 = (int)std::min<int64_t>((total + 255) / 256, 4 * 148);
  absmax_kernel<<<g1 > 0 ? g1 : 1, 256, 0, stream>>>(w, ldw, w_f32, N, K, scratch);
  const int64_t blocks = (int64_t)N * (K / 16);
  const int64_t g2 = (blocks + 255) / 256;
  quantize_kernel<<<(unsigned)(g2 > 0 ? g2 : 1), 256, 0, stream>>>(w, ldw, w_f32, N, K, wq, ldwq,
                                                                   bs, ldbs, gscale, scratch);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

int launch_nvfp4_dequantize(const uint8_t* wq, int64_t ldwq, const uint8_t* bs, int64_t ldbs,
                            const float* gscale, int per_row, void* out, int64_t ldo, int out_f32,
                            int N, int K, cudaStream_t stream) {
  const int64_t blocks = (int64_t)N * (K / 16);
  if (blocks == 0) return 0;
  dequantize_kernel<<<(unsigned)((blocks + 255) / 256), 256, 0, stream>>>(
      wq, ldwq, bs, ldbs, gscale, per_row, out, ldo, out_f32, N, K);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

}  // namespace fnx
