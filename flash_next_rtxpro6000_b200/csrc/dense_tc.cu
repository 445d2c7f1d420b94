// Dense weight-only GEMV on the 5th-generation tensor cores (tcgen05), for the verify
// widths: y[m, n] = bf16((sum_k W[n, k] x[m, k]) * s[n]) for m < M <= 16 tokens.
//
// Same operator contract as dense_gemv.cuh (the reference's _w8a16_gemv_kernel,
// kernels/sglang/srt/layers/quantization/w8a16_gemv.py:132-322: per-row or scalar scale,
// bf16 rounding of (acc * s), two destinations, fp32 widened output, fused greedy argmax),
// with the contraction moved from mma.sync to tcgen05.mma:
//
//   * A = 128 weight rows x 16 k, dequantised EXACTLY to fp16 (int8: 1024 + u - 1152;
//     fp8 e4m3: cvt) by converter warps and written straight into tensor memory
//     (tcgen05.st), so the dequantised weights never pass through shared memory;
//   * B = the 16 token rows (bf16 scaled per token by a power of two into fp16, exact),
//     staged once per CTA in shared memory in the K-major no-swizzle canonical layout;
//   * D = 128 x 16 fp32 in tensor memory, read by the epilogue with tcgen05.ld.
//
// Work split (stream-K).  The weight matrix is cut into 128-row blocks of K / 128 chunks
// (one chunk = 128 rows x 128 bytes = one TMA box); the NB * KC chunks are divided into
// gridDim.x contiguous ranges of equal size (+-1), so every CTA streams the same number of
// bytes whatever NB is.  A block that straddles two or more ranges is finished by the
// contributor that arrives last: each contributor stores its fp32 partial sums in its own
// slot and adds its chunk count to a per-block counter; the one that completes the count
// sums the slots in k order (deterministic), applies the scales and resets the counter.
//
// Roles (448 threads, one CTA per SM):
//   warp 0      TMA producer (one 2-D box per chunk into an NS-stage ring, 128-byte
//               swizzle so that the converters' row reads are bank-conflict free) and
//               owner of the tensor-memory allocation;
//   warp 1      MMA issuer (one thread): 8 x tcgen05.mma M=128 N=16 K=16 per chunk,
//               tcgen05.commit to release the A buffer and, at a block's end, the D buffer;
//   warps 2-9   converters: warp w owns TMEM lanes 32 (w % 4) .. + 31 (its rows) and one
//               k half of each chunk;
//   warps 10-13 epilogue: one TMEM lane quadrant each.
// Every wait is bounded (kWaitLimitNs) and records an error code; all roles fall through
// to the final barrier, after which warp 0 frees the tensor memory.
#include <cuda.h>

#include <cstring>

#include "fnx_common.cuh"
#include "fnx_kernels.h"

namespace fnx {

namespace {

constexpr int kTcRows = 128;                         // weight rows per block (TMEM lanes)
constexpr int kTcBoxK = 128;                         // k per TMA box (128 bytes per row)
constexpr int kTcBoxBytes = kTcRows * kTcBoxK;       // 16 KB
constexpr int kTcChunkK = 2 * kTcBoxK;               // k per chunk: two boxes, one stage
constexpr int kTcChunkBytes = 2 * kTcBoxBytes;       // 32 KB
#ifndef FNX_TC_ABUFS
#define FNX_TC_ABUFS 3
#endif
constexpr int kTcABufs = FNX_TC_ABUFS;               // A buffers in tensor memory
constexpr int kTcACols = kTcChunkK / 2;              // 32-bit columns of one A buffer
constexpr int kTcN = 16;                             // MMA N: tokens (padded with zeros)
// Independent accumulators per block: the k steps of a chunk alternate between them, so
// consecutive MMAs do not wait for each other's D (at N = 16 one MMA's latency, not the
// tensor core's throughput, would bound the rate); the epilogue sums them in a fixed order.
#ifndef FNX_TC_ND
#define FNX_TC_ND 2
#endif
constexpr int kTcND = FNX_TC_ND;
constexpr int kTcDCol = kTcABufs * kTcACols;         // first D column (two D buffer sets)
constexpr int kTcDSet = kTcND * kTcN;                // columns of one D buffer set
constexpr int kTcTmemCols = kTcDCol + 2 * kTcDSet <= 256 ? 256 : 512;
constexpr int kTcConv = 8;
constexpr int kTcEpi = 4;
constexpr int kTcThreads = (2 + kTcConv + kTcEpi) * 32;
static_assert(kTcDCol + 2 * kTcDSet <= kTcTmemCols, "tensor memory columns");
static_assert(kTcND >= 1 && kTcND <= kTcChunkK / 16, "accumulators per chunk of k steps");

// Instruction descriptor of tcgen05.mma.kind::f16: D fp32 (bits 4-5 = 1), A and B fp16
// (bits 7-9, 10-12 = 0), both K-major (bits 15, 16 = 0), N >> 3 at bits 17-22, M >> 4 at
// bits 24-28.
constexpr uint32_t kTcIdesc = (1u << 4) | ((uint32_t)(kTcN >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  const uint32_t s = smem_u32(p);
  return p + ((1024u - (s & 1023u)) & 1023u);
}

// Shared-memory descriptor of a K-major operand without swizzle: 8-row x 16-byte core
// matrices, SBO = byte distance between 8-row groups, LBO = between the two 16-byte k
// halves of one K = 16 step; version 1 (bits 46-47), layout type 0 (bits 61-63).
__device__ __forceinline__ uint64_t smem_desc_k_noswz(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[128 x 16] (+)= A[128 x 16 from TMEM] * B[16 x 16 from smem]^T, and the commit that
// arrives on an mbarrier once every MMA the issuing thread started has completed; issued
// by one elected lane of a converged warp (all 32 lanes call them; the lowest active
// lane, lane 0, is elected every time, so commits track the same thread's MMAs).
__device__ __forceinline__ void tc_mma_elect(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(kTcIdesc), "r"(accumulate), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void tc_commit_elect(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}"
      ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_st_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
      "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
      "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tc_ld_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// A wait whose outcome is the same on every lane (the warp then runs .sync.aligned
// tensor-memory instructions, which need all 32 lanes).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

// 2-D TMA box load (no multicast): box origin (x = byte column, y = row), completing on bar.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

}  // namespace

// Shared-memory layout (offsets from the 1024-byte aligned base).
struct TcLayout {
  int stages, xs, bars, misc, total;
};

__host__ __device__ inline TcLayout tc_layout(int K, int NS) {
  TcLayout L;
  int off = 0;
  L.stages = off;
  off += NS * kTcChunkBytes;
  L.xs = off;                      // [K / 8][16 tokens][8 fp16]
  off += K * 2 * kTcN;
  L.bars = off;                    // full, empty [NS]; afull, afree [3]; dfull, dfree [2]; xready; mmadone
  off += (2 * NS + 2 * kTcABufs + 4 + 2) * 8;
  L.misc = dense_align(off, 16);   // unscale[16] floats, then the TMEM base address
  off = L.misc + kTcN * 4 + 16;
  L.total = off + 1024;            // slack for aligning the dynamic base to 1024 bytes
  return L;
}

struct TcArgs {
  CUtensorMap wmap;   // weights [N rows, row bytes], box 128 x 128 bytes, 128-byte swizzle
  DenseArgs d;
  int KC;             // chunks per 128-row block (K / 128)
  int NB;             // 128-row blocks
  long long total;    // NB * KC
  float* part;        // partial slots [gridDim.x][2][128][16] fp32
  unsigned* pcnt;     // per-block arrival counters, indexed by the block's first CTA (x4 quadrants)
};

namespace {

// CTA whose chunk range holds chunk w when `total` chunks are split into G ranges
// [c * total / G, (c + 1) * total / G): the largest c with floor(c * total / G) <= w.
__device__ __forceinline__ int tc_cta_of(long long w, long long total, int G) {
  return (int)(((w + 1) * (long long)G - 1) / total);
}

// Stage the M token rows as fp16 scaled by a power of two (exact), in the K-major
// canonical layout of the B operand: 16-byte unit (k / 8, token) at ((k / 8) * 16 + token)
// * 16.  Tokens M..15 are zero.  Warp gw of the `nwarps` staging warps takes tokens gw,
// gw + nwarps, ...  A row of up to kTcHoldU units per lane (K <= 2048) is read once and
// held in registers between its max and its conversion, so it costs one load round trip
// (two for longer rows).  Ends with a proxy fence (the tensor core reads the rows through
// the async proxy).
constexpr int kTcHoldU = 8;

__device__ __forceinline__ void tc_stage_x(uint8_t* xs, float* unscale, const DenseArgs& a,
                                           int gw, int nwarps, int lane) {
  const int K = a.K, nu = K / 8;
  const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(a.x);
  for (int m = gw; m < kTcN; m += nwarps) {
    if (m < a.M) {
      const uint8_t* row = reinterpret_cast<const uint8_t*>(x + (size_t)m * a.ldx);
      float mx = 0.f;
      if (nu <= 32 * kTcHoldU) {
        uint4 v[kTcHoldU];
#pragma unroll
        for (int j = 0; j < kTcHoldU; ++j) {  // every load of the row in flight at once
          const int u = lane + 32 * j;
          v[j] = u < nu ? ldg_cg_u4(row + (size_t)u * 16) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int j = 0; j < kTcHoldU; ++j) mx = fmaxf(mx, bf16x8_absmax(v[j]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const int e = stage_exponent(mx);
#pragma unroll
        for (int j = 0; j < kTcHoldU; ++j) {
          const int u = lane + 32 * j;
          if (u < nu)
            *reinterpret_cast<uint4*>(xs + ((size_t)u * kTcN + m) * 16) = bf16x8_to_f16x8_scaled(v[j], e);
        }
        if (lane == 0) unscale[m] = pow2f(-e);
      } else {
        for (int u = lane; u < nu; u += 32) mx = fmaxf(mx, bf16x8_absmax(ldg_cg_u4(row + (size_t)u * 16)));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const int e = stage_exponent(mx);
        for (int u = lane; u < nu; u += 32)
          *reinterpret_cast<uint4*>(xs + ((size_t)u * kTcN + m) * 16) =
              bf16x8_to_f16x8_scaled(ldg_cg_u4(row + (size_t)u * 16), e);
        if (lane == 0) unscale[m] = pow2f(-e);
      }
    } else {
      for (int u = lane; u < nu; u += 32)
        *reinterpret_cast<uint4*>(xs + ((size_t)u * kTcN + m) * 16) = make_uint4(0u, 0u, 0u, 0u);
      if (lane == 0) unscale[m] = 0.f;
    }
  }
  fence_proxy_async_smem();
}

}  // namespace

template <int WT>
__global__ void __launch_bounds__(kTcThreads, 1) dense_tc_kernel(const __grid_constant__ TcArgs A) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const DenseArgs& a = A.d;
  uint8_t* smem = align1024(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int M = a.M, N = a.N, K = a.K, NS = a.NS, KC = A.KC;
  const TcLayout L = tc_layout(K, NS);
  uint8_t* stages = smem + L.stages;
  uint8_t* xs = smem + L.xs;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + NS;
  uint64_t* afull = empty + NS;
  uint64_t* afree = afull + kTcABufs;
  uint64_t* dfull = afree + kTcABufs;
  uint64_t* dfree = dfull + 2;
  uint64_t* xready = dfree + 2;
  uint64_t* mmadone = xready + 1;
  float* unscale = reinterpret_cast<float*>(smem + L.misc);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + L.misc + kTcN * 4);
  const int G = gridDim.x, cta = blockIdx.x;
  const long long total = A.total;
  const long long lo = (long long)cta * total / G, hi = (long long)(cta + 1) * total / G;
  const int nchunk = (int)(hi - lo);

  // One chunk of weights: one or two boxes of 128 rows x 128 bytes into ring stage s.
  // The last chunk of a row holds one box when K is an odd multiple of 128.
  auto issue_chunk = [&](int i, uint64_t pol) {
    const int s = i % NS;
    const long long w = lo + i;
    const int b = (int)(w / KC), kc = (int)(w - (long long)b * KC);
    const bool two = K - kc * kTcChunkK > kTcBoxK;
    mbar_arrive_expect_tx(&full[s], (uint32_t)(two ? kTcChunkBytes : kTcBoxBytes));
    uint8_t* st = stages + (size_t)s * kTcChunkBytes;
    tma_load_2d(st, &A.wmap, kc * kTcChunkK, b * kTcRows, &full[s], pol);
    if (two) tma_load_2d(st + kTcBoxBytes, &A.wmap, kc * kTcChunkK + kTcBoxK, b * kTcRows, &full[s], pol);
  };
  // The producer lane fills the whole ring before the tensor-memory allocation and the
  // block barrier: the weights do not depend on the previous kernel, and the first boxes
  // are then in flight ~0.6 us earlier.
  int pre = 0;
  if (tid == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&A.wmap)) : "memory");
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kTcConv);
    }
    for (int b = 0; b < kTcABufs; ++b) {
      mbar_init(&afull[b], kTcConv);
      mbar_init(&afree[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&dfull[b], 1);
      mbar_init(&dfree[b], kTcEpi);
    }
    mbar_init(xready, kTcConv + kTcEpi);
    mbar_init(mmadone, 1);
    mbar_fence_init();
    fence_proxy_async_smem();  // the initialised barriers are seen by the copy engine
    const uint64_t pol = policy_evict_first();
    pre = nchunk < NS ? nchunk : NS;
    for (int i = 0; i < pre; ++i) issue_chunk(i, pol);
  } else if (warp >= 2) {
    // Converters and epilogue warps stage the token rows meanwhile, so that their loads
    // go out ahead of most of the ring's boxes rather than queue behind them.
    pdl_wait();
    tc_stage_x(xs, unscale, a, warp - 2, kTcConv + kTcEpi, lane);
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(tslot)), "r"(kTcTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    // The weights do not depend on the previous kernel: no dependency wait here.
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int issued = pre;
      for (int i = pre; i < nchunk; ++i) {
        const int s = i % NS;
        if (!mbar_wait(&empty[s], ((i / NS) & 1) ^ 1)) {
          record_error(a.err, ERR_WAIT_EMPTY);
          break;
        }
        issue_chunk(i, pol);
        issued = i + 1;
      }
      // no box may still be landing when the CTA exits
      for (int j = issued > NS ? issued - NS : 0; j < issued; ++j)
        if (!mbar_wait(&full[j % NS], (j / NS) & 1)) record_error(a.err, ERR_DRAIN);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop (converged) and one elected lane issues: a single lane
    // looping alone issued an N = 16 MMA every ~47 cycles on B200, a converged warp with
    // elect.sync every ~27.  Lane 0 is always the one elected, so it also commits.
    bool ok = warp_wait(xready, 0);
    if (!ok && lane == 0) record_error(a.err, ERR_WAIT_X);
    // B descriptor of k step 0; k step t of the matrix starts 2 * 16 tokens * 16 bytes
    // later, i.e. + 32 in the descriptor's address field (16-byte units)
    const uint64_t bdesc0 = smem_desc_k_noswz(smem_u32(xs), kTcN * 16, 8 * 16);
    long long w = lo;
    int i = 0, sg = 0;
    while (ok && w < hi) {
      const int b = (int)(w / KC);
      const long long seg0 = w;
      const long long seg1 = hi < (long long)(b + 1) * KC ? hi : (long long)(b + 1) * KC;
      const int db = sg & 1;
      if (sg >= 2 && !warp_wait(&dfree[db], ((sg >> 1) & 1) ^ 1)) {
        if (lane == 0) record_error(a.err, ERR_WAIT_RFREE);
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tbase + (uint32_t)(kTcDCol + db * kTcDSet);
      for (; w < seg1; ++w, ++i) {
        const int ab = i % kTcABufs;
        if (!warp_wait(&afull[ab], (i / kTcABufs) & 1)) {
          if (lane == 0) record_error(a.err, ERR_WAIT_FULL);
          ok = false;
          break;
        }
        tc_fence_after();
        const int kc = (int)(w - (long long)b * KC);
        const int nj = (K - kc * kTcChunkK >= kTcChunkK ? kTcChunkK : K - kc * kTcChunkK) / 16;
        const uint64_t bd = bdesc0 + (uint64_t)kc * (kTcChunkK / 16) * 32;
        const uint32_t at = tbase + (uint32_t)(ab * kTcACols);
        const uint32_t acc0 = w == seg0 ? 0u : 1u;  // the block's first chunk starts each accumulator
        // Straight-line issue: a branch between two elect.sync MMAs makes the warp
        // reconverge before each one (measured ~120 instead of ~30 cycles per MMA).
#pragma unroll
        for (int j = 0; j < kTcBoxK / 16; ++j)
          tc_mma_elect(d_tmem + (uint32_t)((j % kTcND) * kTcN), at + 8 * j, bd + 32 * j,
                       j < kTcND ? acc0 : 1u);
        if (nj > kTcBoxK / 16) {
#pragma unroll
          for (int j = kTcBoxK / 16; j < kTcChunkK / 16; ++j)
            tc_mma_elect(d_tmem + (uint32_t)((j % kTcND) * kTcN), at + 8 * j, bd + 32 * j, 1u);
        }
        tc_commit_elect(&afree[ab]);
      }
      if (!ok) break;
      tc_commit_elect(&dfull[db]);
      ++sg;
    }
    // every MMA has completed before the tensor memory is freed
    tc_commit_elect(mmadone);
    if (!warp_wait(mmadone, 0) && lane == 0) record_error(a.err, ERR_DRAIN);
  } else {
    // the token rows were staged before the block barrier (which made the barriers usable)
    __syncwarp();
    if (lane == 0) mbar_arrive(xready);

    if (warp < 2 + kTcConv) {
      // ---------------------------------------------------------------- converters
      // Row r = 32 (warp % 4) + lane of the block (TMEM lane r), box h of each chunk (k
      // half): eight 16-byte units of the swizzled box row (unit u at (u ^ (r % 8)) * 16),
      // 128 weights -> 64 fp16 pairs -> A columns h * 64 .. + 63 of the chunk's buffer, in
      // two halves so that the second half's loads overlap the first half's store.
      const int q = warp & 3, h = (warp - 2) >> 2;
      const int r = 32 * q + lane;
      const uint32_t t_row = tbase + ((uint32_t)(32 * q) << 16);
      for (int i = 0; i < nchunk; ++i) {
        const int s = i % NS, ab = i % kTcABufs;
        if (!warp_wait(&full[s], (i / NS) & 1)) {
          if (lane == 0) record_error(a.err, ERR_WAIT_FULL);
          break;
        }
        if (i >= kTcABufs && !warp_wait(&afree[ab], ((i / kTcABufs) & 1) ^ 1)) {
          if (lane == 0) record_error(a.err, ERR_WAIT_RFREE);
          break;
        }
        tc_fence_after();
        const long long w = lo + i;
        const int kc = (int)(w % KC);
        if (h == 0 || K - kc * kTcChunkK > kTcBoxK) {  // a one-box chunk leaves box 1 empty
          const uint8_t* rowp = stages + (size_t)s * kTcChunkBytes + h * kTcBoxBytes + r * kTcBoxK;
#pragma unroll
          for (int p = 0; p < 2; ++p) {
            uint32_t reg[32];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const uint4 v = lds128(rowp + (((4 * p + u) ^ (r & 7)) << 4));
              const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                if constexpr (WT == W_INT8) deq_int8_word(wv[t], reg[8 * u + 2 * t], reg[8 * u + 2 * t + 1]);
                else deq_fp8_word(wv[t], reg[8 * u + 2 * t], reg[8 * u + 2 * t + 1]);
              }
            }
            tc_st_x32(t_row + (uint32_t)(ab * kTcACols + h * (kTcBoxK / 2) + p * 32), reg);
          }
        }
        __syncwarp();  // every lane's reads of the stage are complete
        if (lane == 0) mbar_arrive(&empty[s]);
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[ab]);
      }
    } else {
      // ---------------------------------------------------------------- epilogue
      const int q = warp & 3;
      const int rq = 32 * q + lane;  // row within the block = TMEM lane
      const bool per_row = a.scale_kind == SCALE_F32_ROW || a.scale_kind == SCALE_BF16_ROW;
      const float scalar_scale = per_row ? 0.f : load_row_scale(a.scale, a.scale_kind, 0);
      unsigned long long best[kTcN];
#pragma unroll
      for (int m = 0; m < kTcN; ++m) best[m] = 0ull;
      bool ok = warp_wait(xready, 0);  // unscale[] is written
      if (!ok) record_error(a.err, ERR_WAIT_X);
      long long w = lo;
      int sg = 0;
      while (ok && w < hi) {
        const int b = (int)(w / KC);
        const long long blk0 = (long long)b * KC, blk1 = blk0 + KC;
        const long long seg0 = w, seg1 = hi < blk1 ? hi : blk1;
        const int db = sg & 1;
        const int n = b * kTcRows + rq;
        // the row's scale is read while the block's MMAs run, not after them
        const float s = per_row && n < N ? load_row_scale(a.scale, a.scale_kind, n) : scalar_scale;
        if (!warp_wait(&dfull[db], (sg >> 1) & 1)) {
          record_error(a.err, ERR_WAIT_RED);
          break;
        }
        tc_fence_after();
        float v[kTcN];
#pragma unroll
        for (int m = 0; m < kTcN; ++m) v[m] = 0.f;
#pragma unroll
        for (int ac = 0; ac < kTcND; ++ac) {  // accumulators summed in a fixed order
          uint32_t d[kTcN];
          tc_ld_x16(tbase + ((uint32_t)(32 * q) << 16) + (uint32_t)(kTcDCol + db * kTcDSet + ac * kTcN), d);
          tc_wait_ld();
#pragma unroll
          for (int m = 0; m < kTcN; ++m) v[m] += __uint_as_float(d[m]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dfree[db]);
        bool fin = seg0 == blk0 && seg1 == blk1;
        if (!fin) {
          // A block shared with other CTAs.  Its ranges are counted in chunks on the
          // counter of the CTA that holds its first chunk; each range's sums go to a slot
          // (0 = the range starts inside the block, 1 = it starts at the block's first
          // chunk), and the last range to arrive adds the slots in k order.  A range that
          // finds every other range already counted is the last one without publishing
          // its own sums (the usual case for a CTA's final block, whose other part the
          // next CTA ran at its start).
          const int c0 = tc_cta_of(blk0, total, G);
          const unsigned nseg = (unsigned)(seg1 - seg0);
          unsigned seen = 0;
          if (lane == 0) seen = ld_acquire_gpu_u32(&A.pcnt[c0 * 4 + q]);
          seen = __shfl_sync(0xffffffffu, seen, 0);
          fin = seen + nseg == (unsigned)KC;
          if (!fin) {
            const int ht = seg0 > blk0 ? 0 : 1;
            float* slot = A.part + (((size_t)cta * 2 + ht) * kTcRows + rq) * kTcN;
#pragma unroll
            for (int m = 0; m < kTcN; ++m) st_cg_f32(slot + m, v[m]);
            __threadfence();
            __syncwarp();
            unsigned prev = 0;
            if (lane == 0) prev = atomicAdd(&A.pcnt[c0 * 4 + q], nseg);
            prev = __shfl_sync(0xffffffffu, prev, 0);
            fin = prev + nseg == (unsigned)KC;
            if (fin) __threadfence();
          }
          __syncwarp();
          if (fin) {  // sum the ranges in k order (this CTA's own from registers)
            const int c1 = tc_cta_of(blk1 - 1, total, G);
            float t[kTcN];
#pragma unroll
            for (int m = 0; m < kTcN; ++m) t[m] = 0.f;
            for (int cc = c0; cc <= c1; ++cc) {
              if (cc == cta) {
#pragma unroll
                for (int m = 0; m < kTcN; ++m) t[m] += v[m];
              } else {
                const float* sp = A.part + (((size_t)cc * 2 + (cc == c0 ? 1 : 0)) * kTcRows + rq) * kTcN;
#pragma unroll
                for (int m = 0; m < kTcN; ++m) t[m] += ld_cg_f32(sp + m);
              }
            }
#pragma unroll
            for (int m = 0; m < kTcN; ++m) v[m] = t[m];
            __syncwarp();
            if (lane == 0) A.pcnt[c0 * 4 + q] = 0u;
          }
        }
        if (fin && n < N) {
          void* dst = a.y;
          int64_t ld = a.ldy, col = n;
          if (a.split_n > 0 && n >= a.split_n) {
            dst = a.y2;
            ld = a.ldy2;
            col = n - a.split_n;
          }
#pragma unroll
          for (int m = 0; m < kTcN; ++m) {
            if (m >= M) break;
            const __nv_bfloat16 o = __float2bfloat16_rn(v[m] * unscale[m] * s);
            if (a.out_f32)
              reinterpret_cast<float*>(dst)[(size_t)m * ld + col] = __bfloat162float(o);
            else
              reinterpret_cast<__nv_bfloat16*>(dst)[(size_t)m * ld + col] = o;
            const unsigned long long k =
                argmax_key((uint32_t)__bfloat16_as_ushort(o), (uint32_t)(a.row_offset + n));
            best[m] = k > best[m] ? k : best[m];
          }
        }
        w = seg1;
        ++sg;
      }
      if (a.am_keys) {
#pragma unroll
        for (int m = 0; m < kTcN; ++m) {
          if (m >= M) break;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best[m], o);
            best[m] = other > best[m] ? other : best[m];
          }
        }
        if (lane == 0) {
#pragma unroll
          for (int m = 0; m < kTcN; ++m) {
            if (m >= M) break;
            if (best[m] != 0ull) atomicMax(&a.am_keys[m], best[m]);
          }
        }
        __threadfence();
        __syncwarp();
        unsigned prev = 0;
        if (lane == 0) prev = atomicAdd(a.am_count, 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev == (unsigned)G * kTcEpi - 1) {  // the last epilogue warp of the grid
          __threadfence();
          unsigned long long key = lane < M ? atomicExch(&a.am_keys[lane], 0ull) : 0ull;
          if (a.peerbuf) key = peer_key_max(a.peerbuf, key, M, a.err);  // whole warp
          if (lane < M) {
            const int64_t row = (int64_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
            if (a.am_out) a.am_out[lane] = row;
            if (a.am_key_out) a.am_key_out[lane] = key;
          }
          if (lane == 0) *a.am_count = 0u;
        }
      }
    }
  }
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(kTcTmemCols)
                 : "memory");
  }
}

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver's tensor-map encoder, found through the runtime (no link against libcuda).
EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

using TcKernel = void (*)(const TcArgs);

TcKernel tc_kernel(int wt) {
  if (wt == W_INT8) return dense_tc_kernel<W_INT8>;
  if (wt == W_FP8) return dense_tc_kernel<W_FP8>;
  return nullptr;
}

constexpr size_t kTcMaxSmem = 227 * 1024;

}  // namespace

bool dense_tc_plan(int wt, int K, int& NS, size_t& smem) {
  if (!tc_kernel(wt) || K < kTcBoxK || K % kTcBoxK) return false;
  const TcLayout L0 = tc_layout(K, 0);
  const long long room = (long long)kTcMaxSmem - L0.total - 16LL * 8;  // + barriers of the stages
  const long long ns = room / kTcChunkBytes;
  if (ns < 3) return false;
  NS = (int)(ns < 10 ? ns : 10);
  smem = (size_t)tc_layout(K, NS).total;
  return smem <= kTcMaxSmem;
}

int dense_tc_grid(int N, int K) {
  const long long total = (long long)((N + kTcRows - 1) / kTcRows) * ((K + kTcChunkK - 1) / kTcChunkK);
  const long long sms = num_sms();
  return (int)(total < sms ? total : sms);
}

int64_t dense_tc_partial_floats(int grid) { return (int64_t)grid * 2 * kTcRows * kTcN; }
int64_t dense_tc_counters(int grid) { return (int64_t)grid * 4; }

int launch_dense_tc(const DenseArgs& d, int wt, int grid, size_t smem, float* part, unsigned* pcnt,
                    cudaStream_t stream) {
  TcKernel k = tc_kernel(wt);
  EncodeTiledFn enc = encode_tiled();
  if (!k || !enc) return 1;
  if (!prepare_kernel((const void*)k)) return 2;
  TcArgs A;
  memset(&A, 0, sizeof(A));
  const cuuint64_t dims[2] = {(cuuint64_t)d.K, (cuuint64_t)d.N};  // bytes per row (8-bit), rows
  const cuuint64_t strides[1] = {(cuuint64_t)d.ldw};
  const cuuint32_t box[2] = {(cuuint32_t)kTcBoxK, (cuuint32_t)kTcRows};
  const cuuint32_t estr[2] = {1, 1};
  if (enc(&A.wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(d.w), dims, strides, box,
          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return 3;
  A.d = d;
  A.KC = (d.K + kTcChunkK - 1) / kTcChunkK;
  A.NB = (d.N + kTcRows - 1) / kTcRows;
  A.total = (long long)A.NB * A.KC;
  A.part = part;
  A.pcnt = pcnt;
  if (grid < 1 || grid > A.total) return 1;  // every CTA needs a chunk (partial-slot order)
  return launch_with_pdl((const void*)k, A, grid, kTcThreads, smem, d.pdl, stream);
}

}  // namespace fnx
