// Internal launch interface between the C ABI (fnx_api.cu) and the kernels.
// Argument blocks are plain structs of device pointers and sizes.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace fnx {

struct DenseArgs {
  const void* x;          // bf16 [M, K], row stride ldx elements, rows 16-byte aligned
  int64_t ldx;
  const uint8_t* w;       // weight rows, row stride ldw BYTES (16-byte multiple)
  int64_t ldw;
  const uint8_t* bs;      // NVFP4 e4m3 block scales [N, K/16], row stride ldbs bytes
  int64_t ldbs;
  const void* scale;      // per-row / scalar output scale (ScaleKind)
  int scale_kind;
  void* y;                // [M, ldy] bf16 or fp32 (out_f32)
  int64_t ldy;
  void* y2;               // second destination for columns >= split_n (or null)
  int64_t ldy2;
  int64_t split_n;        // 0: single destination
  int out_f32;
  unsigned long long* am_keys;  // [M] argmax keys (zero between calls), or null
  unsigned int* am_count;       // CTA arrival counter (zero between calls)
  int64_t* am_out;              // [M] argmax row (global row id), or null
  unsigned long long* am_key_out;  // [M] raw argmax key copy (sharded heads), or null
  int64_t row_offset;           // global id of local row 0 (vocab shards)
  float* ws;              // split-K partials [row_tiles * ksplit * 256]
  unsigned int* ws_cnt;   // split-K counters [row_tiles] (zero between calls)
  int M, N, K;            // N = output columns (fused SiLU: H, weight rows 2H)
  int ksplit;
  int silu;
  int W, G;               // warps per group, groups per CTA
  int row_tiles, n_units;
  int pdl;
};

struct MoeArgs {
  const void* x;          // bf16 [M, H] hidden states (row stride ldx elements)
  int64_t ldx;
  const int32_t* ids;     // [M, R] routed expert ids (< 0: skipped)
  const float* wts;       // [M, R] router weights
  int M, R, E, H, I;
  // routed experts: w13 [E, 2I, H/2] rows [up(I); gate(I)], w2 [E, H, I/2]
  const uint8_t* w13;
  const uint8_t* s13;     // e4m3 block scales of w13 per expert (2I x H/16)
  const float* g13;       // global scale of expert e at g13[e * g13_stride]
  int64_t g13_stride;
  const uint8_t* w2;
  const uint8_t* s2;      // (H x I/16) per expert
  const float* g2;
  int64_t g2_stride;
  // optional always-on shared expert in the same format (one expert)
  const uint8_t* sh_w13;
  const uint8_t* sh_s13;
  const float* sh_g13;
  const uint8_t* sh_w2;
  const uint8_t* sh_s2;
  const float* sh_g2;
  int has_shared;
  int swizzled;           // block scales in the 128x4 swizzled layout (server format)
  // expert slice owned by this launch (expert-parallel shards): ids outside
  // [e_lo, e_lo + E_local) are skipped; weight tensors hold the local experts only.
  int e_lo;
  // scratch
  void* act;              // bf16 [M * (R + 1), I]
  float* part;            // fp32 [M * (R + 1), H]
  unsigned int* cnt;      // [H / 16] (zero between calls)
  // output: bf16 [M, H] (or fp32 partial sums when out_f32, for cross-rank reduction)
  void* out;
  int64_t ldo;
  int out_f32;
  int W, G;
  int pdl;
};

int launch_dense(const DenseArgs& a, int wtype, int nt, int cpw, int grid, size_t smem,
                 cudaStream_t stream);
int launch_moe_up(const MoeArgs& a, int nt, int grid, size_t smem, cudaStream_t stream);
int launch_moe_down(const MoeArgs& a, int nt, int grid, size_t smem, cudaStream_t stream);
int launch_argmax_decode(const unsigned long long* keys, int64_t* out, int M,
                         cudaStream_t stream);

int dense_occupancy(int wtype, int nt, int cpw, int threads, size_t smem);
int moe_up_occupancy(int nt, int cpw, int threads, size_t smem);
int moe_down_occupancy(int nt, int cpw, int threads, size_t smem);
size_t moe_up_smem(int M, int R, int E, int H, int W, int G, int NT);
size_t moe_down_smem(int M, int R, int E, int I, int W, int G, int NT);

// Streaming multiprocessors of the current device (cached per device).
int num_sms();
// Raise a kernel's dynamic shared-memory limit once per device; false on failure.
bool prepare_kernel(const void* func);

// Launch `func(args)` with the programmatic-stream-serialization attribute when `pdl`.
template <typename Args>
int launch_with_pdl(const void* func, const Args& args, int grid, int threads, size_t smem,
                    int pdl, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  void* params[1] = {const_cast<Args*>(&args)};
  return cudaLaunchKernelExC(&cfg, func, params) == cudaSuccess ? 0 : 2;
}

}  // namespace fnx
