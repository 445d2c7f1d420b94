// MoE router for M <= 16 tokens: bf16 logits projection x . W^T (+ bias) in fp32 and the
// softmax top-k that turns the logits into the routing table the MoE kernels read.
//
// Replaces the reference's
//   router_gemv            kernels/sglang/srt/layers/moe/router_gemv.py:10-93
//   route_softmax_fast     patches/sglang/series/0110-…patch:27-184 and 0111-…patch
//                          (python/sglang/kernels/ops/moe/moe_router_softmax_fast.py)
// and fuses the two into one launch (the last CTA of the projection runs the top-k),
// which removes the router's separate launch from the MoE prologue.
//
// Projection.  One CTA per 16 experts (weight rows), 16 warps: warp w takes the 32-column
// blocks w, w + 16, ... of K.  Per block a lane loads 16 bytes of weight rows g and g + 8
// and 16 bytes of token rows g (and g + 8 at M > 8), and two mma.sync.m16n8k16 (bf16 in,
// fp32 accumulate) consume them: the k order inside a block is permuted identically for
// both operands, which leaves the dot product unchanged.  The 16 warps' partial tiles
// are summed in warp order in shared memory (fixed order, deterministic).
//
// Top-k.  One warp per token row of N <= 512 logits (16 per lane): the row max and the
// sum of exp(l - max), then topk picks of the largest 64-bit key
// (order-preserving bits of the logit) << 32 | (2^32 - 1 - expert), so one max gives the
// winner with the lowest expert id on ties; NaN ranks as -1e30 (its weight is 0, but it
// makes the row sum and so every weight of the row NaN, as in the reference); -0.0 ranks
// as +0.0.  weight = exp(l - max) / sum, renormalised by the sum of the picked weights
// when that is positive (exp and division in the reference's fast forms).
#include "fnx_common.cuh"
#include "fnx_kernels.h"

namespace fnx {

namespace {

__device__ __forceinline__ uint32_t order32(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float unorder32(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

__device__ __forceinline__ void mma_bf16_16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ld16(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}

// Softmax top-k of one row (one warp).  val(n) returns the biased logit of expert n < N.
template <typename ValFn>
__device__ __forceinline__ void softmax_topk_row(ValFn val, int N, int topk, bool renorm,
                                                 float* ow, int32_t* oi) {
  const int lane = threadIdx.x & 31;
  constexpr int kPer = 16;  // N <= 512
  float v[kPer];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int n = lane + 32 * j;
    v[j] = n < N ? val(n) : -INFINITY;
    mx = fmaxf(mx, v[j]);  // fmaxf skips NaN; a NaN still poisons the sum below
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  // exp and the division as the reference's router evaluates them (tl.exp: ex2.approx of
  // x * log2(e); the fp32 division of Triton: div.full), i.e. __expf and __fdividef
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < kPer; ++j)
    if (lane + 32 * j < N) sum += __expf(v[j] - mx);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  unsigned long long key[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int n = lane + 32 * j;
    float r = v[j] != v[j] ? -1e30f : v[j];  // NaN ranks as the -1e30 floor
    if (r == 0.f) r = 0.f;                   // -0.0 ranks as +0.0
    key[j] = n < N ? ((unsigned long long)order32(r) << 32) | (0xFFFFFFFFu - (uint32_t)n) : 0ull;
  }
  float my_w = 0.f;
  int my_id = 0;
  for (int k = 0; k < topk; ++k) {
    unsigned long long mine = 0ull;
#pragma unroll
    for (int j = 0; j < kPer; ++j) mine = key[j] > mine ? key[j] : mine;
    // warp max of the 64-bit keys as two 32-bit reductions: the value half, then the id
    // half among the lanes that hold that value
    const uint32_t hi = __reduce_max_sync(0xffffffffu, (uint32_t)(mine >> 32));
    const uint32_t lo =
        __reduce_max_sync(0xffffffffu, (uint32_t)(mine >> 32) == hi ? (uint32_t)mine : 0u);
    const unsigned long long best = ((unsigned long long)hi << 32) | lo;
#pragma unroll
    for (int j = 0; j < kPer; ++j)
      if (key[j] == best) key[j] = 0ull;  // keys are unique (the expert id is in them)
    const int n = (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
    const float w = __fdividef(__expf(unorder32((uint32_t)(best >> 32)) - mx), sum);
    if (lane == k) {
      my_w = w;
      my_id = n;
    }
  }
  if (renorm) {
    float rs = lane < topk ? my_w : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, o);
    my_w = my_w / (rs > 0.f ? rs : 1.f);
  }
  if (lane < topk) {
    ow[lane] = my_w;
    oi[lane] = my_id;
  }
}

constexpr int kRouterWarps = 16;

template <int NT>
__global__ void __launch_bounds__(kRouterWarps * 32, 1) router_kernel(const RouterArgs a) {
  __shared__ float red[kRouterWarps][NT * 4][32];
  __shared__ unsigned last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int row0 = blockIdx.x * 16;
  const __nv_bfloat16* wa = a.w + (size_t)(row0 + g) * a.ldw + 8 * c;
  const __nv_bfloat16* wb = wa + (size_t)8 * a.ldw;
  pdl_wait();  // the activations may come from the previous kernel
  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int r = 0; r < 4; ++r) acc[nt][r] = 0.f;
  const int nblk = a.K >> 5;
#pragma unroll 4
  for (int b = warp; b < nblk; b += kRouterWarps) {
    const int k0 = b * 32;
    const uint4 al = ld16(wa + k0), ah = ld16(wb + k0);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int t = nt * 8 + g;
      const uint4 xv = t < a.M ? ld16(a.x + (size_t)t * a.ldx + k0 + 8 * c) : make_uint4(0u, 0u, 0u, 0u);
      mma_bf16_16816(acc[nt], al.x, ah.x, al.y, ah.y, xv.x, xv.y);
      mma_bf16_16816(acc[nt], al.z, ah.z, al.w, ah.w, xv.z, xv.w);
    }
  }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int r = 0; r < 4; ++r) red[warp][nt * 4 + r][lane] = acc[nt][r];
  __syncthreads();
  if (threadIdx.x < NT * 4 * 32) {
    const int j = threadIdx.x >> 5, l = threadIdx.x & 31;  // fragment register j of lane l
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kRouterWarps; ++w) s += red[w][j][l];
    const int nt = j >> 2, r = j & 3;
    const int row = row0 + (l >> 2) + (r >= 2 ? 8 : 0);
    const int tok = nt * 8 + 2 * (l & 3) + (r & 1);
    if (a.bias) s += __bfloat162float(a.bias[row]);
    if (tok < a.M) st_cg_f32(a.logits + (size_t)tok * a.ldl + row, s);
  }
  if (a.topk <= 0) {
    pdl_trigger();
    return;
  }
  // The last CTA to finish its logits runs the top-k over all of them: the barrier
  // orders the CTA's logit stores before thread 0's release-acquire increment, and the
  // last CTA's acquire (through the second barrier) makes every CTA's stores visible.
  __syncthreads();
  if (threadIdx.x == 0)
    last = atom_add_acq_rel_gpu(a.counter, 1u) == gridDim.x - 1 ? 1u : 0u;
  __syncthreads();
  if (!last) return;
  for (int t = warp; t < a.M; t += kRouterWarps) {
    const float* lrow = a.logits + (size_t)t * a.ldl;
    softmax_topk_row([&](int n) { return ld_cg_f32(lrow + n); }, a.N, a.topk, a.renorm != 0,
                     a.out_w + (size_t)t * a.ldk, a.out_ids + (size_t)t * a.ldk);
  }
  if (threadIdx.x == 0) *a.counter = 0u;  // ready for the next call
  pdl_trigger();
}

__global__ void __launch_bounds__(128) softmax_topk_kernel(const TopkArgs a) {
  const int t = blockIdx.x * 4 + (threadIdx.x >> 5);
  pdl_wait();
  if (t < a.M) {
    if (a.scores_f32) {
      const float* row = reinterpret_cast<const float*>(a.scores) + (size_t)t * a.lds;
      softmax_topk_row([&](int n) { return ld_cg_f32(row + n) + (a.bias ? a.bias[n] : 0.f); },
                       a.N, a.topk, a.renorm != 0, a.out_w + (size_t)t * a.ldk,
                       a.out_ids + (size_t)t * a.ldk);
    } else {
      const unsigned short* row = reinterpret_cast<const unsigned short*>(a.scores) + (size_t)t * a.lds;
      softmax_topk_row(
          [&](int n) { return bf16_bits_to_f32(row[n]) + (a.bias ? a.bias[n] : 0.f); }, a.N,
          a.topk, a.renorm != 0, a.out_w + (size_t)t * a.ldk, a.out_ids + (size_t)t * a.ldk);
    }
  }
  pdl_trigger();
}

}  // namespace

int launch_router(const RouterArgs& a, cudaStream_t stream) {
  const void* k = a.M > 8 ? (const void*)router_kernel<2> : (const void*)router_kernel<1>;
  return launch_with_pdl(k, a, a.N / 16, kRouterWarps * 32, 0, a.pdl, stream);
}

int launch_softmax_topk(const TopkArgs& a, cudaStream_t stream) {
  return launch_with_pdl((const void*)softmax_topk_kernel, a, (a.M + 3) / 4, 128, 0, a.pdl,
                         stream);
}

}  // namespace fnx
