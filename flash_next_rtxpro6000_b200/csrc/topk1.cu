// Greedy top-1 of draft logits with the draft chain step: the B200 form of
// draft_topk1_postprocess (patches/sglang/series/0016-spec-remove-per-draft-step-glue-in-
// the-topk-1-chain-.patch:46-73 and the split reduction it finalises).
//
// Each CTA scans one slice of one row: keys (order-preserving bits of the logit) << 32 |
// (2^32 - 1 - column), so the maximum key is the largest logit with the lowest column on
// ties (torch.argmax; a positive-signed NaN ranks above +inf).  The CTA's maximum goes to
// keys[row] with a 64-bit atomicMax; the CTA that arrives last (release-acquire counter)
// decodes every row, applies the chain step (hot-vocabulary token map, draft_tokens
// column, topk_p = 1, position + 1) and leaves keys and counter at zero for the next call.
#include "fnx_common.cuh"
#include "fnx_kernels.h"

namespace fnx {

namespace {

__device__ __forceinline__ uint32_t order32(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kTop1Threads = 256;

__global__ void __launch_bounds__(kTop1Threads) top1_kernel(const Top1Args a) {
  __shared__ unsigned long long wbest[kTop1Threads / 32];
  __shared__ unsigned last;
  const int m = blockIdx.y;
  const int per = (a.V + a.splits - 1) / a.splits;
  const int v0 = blockIdx.x * per;
  const int v1 = min(a.V, v0 + per);
  pdl_wait();  // the logits come from the previous kernel
  unsigned long long best = 0ull;
  if (a.logits_f32) {
    const float* row = reinterpret_cast<const float*>(a.logits) + (size_t)m * a.ldl;
#pragma unroll 8
    for (int v = v0 + threadIdx.x; v < v1; v += kTop1Threads) {
      const unsigned long long k =
          ((unsigned long long)order32(ld_cg_f32(row + v)) << 32) | (0xFFFFFFFFu - (uint32_t)v);
      best = k > best ? k : best;
    }
  } else {
    const unsigned short* row = reinterpret_cast<const unsigned short*>(a.logits) + (size_t)m * a.ldl;
#pragma unroll 8
    for (int v = v0 + threadIdx.x; v < v1; v += kTop1Threads) {
      const unsigned long long k = ((unsigned long long)order32(bf16_bits_to_f32(row[v])) << 32) |
                                   (0xFFFFFFFFu - (uint32_t)v);
      best = k > best ? k : best;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if ((threadIdx.x & 31) == 0) wbest[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kTop1Threads / 32; ++w) best = wbest[w] > best ? wbest[w] : best;
    if (best) atomicMax(a.keys + m, best);
    // release: this CTA's atomicMax before its arrival; acquire for the last CTA
    last = atom_add_acq_rel_gpu(a.count, 1u) == gridDim.x * gridDim.y - 1 ? 1u : 0u;
  }
  __syncthreads();
  if (last) {
    if (threadIdx.x < a.M) {
      const unsigned long long key = atomicExch(a.keys + threadIdx.x, 0ull);
      draft_chain_store(a.chain, threadIdx.x, (int64_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull)));
    }
    if (threadIdx.x == 0) *a.count = 0u;
  }
  pdl_trigger();
}

}  // namespace

int launch_top1(const Top1Args& a, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.splits, a.M);
  cfg.blockDim = dim3(kTop1Threads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.pdl ? 1 : 0;
  void* params[1] = {const_cast<Top1Args*>(&a)};
  return cudaLaunchKernelExC(&cfg, (const void*)top1_kernel, params) == cudaSuccess ? 0 : 2;
}

}  // namespace fnx
