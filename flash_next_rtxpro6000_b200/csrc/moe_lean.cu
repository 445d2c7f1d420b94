// NVFP4 routed-MoE layer for one-token decode (M = 1; the code serves M <= 2) in ONE
// launch, laid out for latency: the whole layer's weight bytes are cut into equal shares
// per SM and every CTA puts its share in flight as soon as the routing is known.
//
// Same operator and numerics as the reference's one-token pair (patches/sglang/series/
// 0112-...patch:182-227 gate/up + SiLU, :229-287 down + route sum) and as moe_fused.cu:
//   act[d, t, :] = bf16( silu(g13 * <gate, x_t>) * g13 * <up, x_t> )         (0112:220-224)
//   out[t, :]    = bf16( sum_r w[t, r] * g2 * <W2, act[d(t, r), t]>  + shared expert )
// with the route sum in route order, then the shared expert (deterministic, no float
// atomics).
//
// Slots.  The routed experts of the call, in ascending id order, after the always-on
// shared expert (slot 0 when present); each slot keeps the set of tokens routed to it, so
// a repeated id or many tokens on one expert cost nothing extra and drop nothing.
//
// Work.  Gate/up TILES: 8 act columns of one slot (the up and gate rows of columns
// {128 b + 32 q + 2 p + h : q < 4, h < 2}, whose swizzled block scales form 32-byte
// pieces) over all of H.  Down BLOCKS: 16 output rows {128 b + 32 q + 4 p + i : q, i < 4}
// (64-byte scale pieces); CTA c owns blocks c, c + grid, ... and computes every slot's
// contribution to them, so it finishes its rows itself: the route sum needs no partials
// in global memory and no second launch.  The gate/up tiles are split into contiguous
// per-CTA ranges such that tiles + own down blocks give every CTA the same byte count.
// Ring items: the CTA's tiles, then its down blocks in groups of four slots.
//
// Roles (576 threads, one CTA per SM, all CTAs resident: a down block waits for the
// tiles of other CTAs):
//   warp 0     producer: one TMA box per weight half (8 rows x H/2 bytes of a tile, 16 rows
//              x I/2 of a down slot, 128-byte swizzle) and one per scale set;
//   warps 1-16 four groups of four consumer warps; group g takes items g, g + 4, ... (the
//              decode -> scale -> mma chains are latency bound: four warps per sub-partition)
//              tile: warp w of the group reduces k quarter w (mma.sync, swap-AB, the act
//              columns as MMA rows); the tile's leader warp
//              (rotating) sums the four quarters in k order, applies the scales and SiLU,
//              stores the bf16 act values and counts the tile as stored (CTA scope);
//              down: once every tile of the layer is stored (one acquire on the layer's
//              tile counter), the consumer warps stage all act rows into shared memory as
//              fp16 scaled by each row's power of two; warp w then takes slot 4 k + w of
//              each item, runs the 16-row block over I and writes the per-route results
//              into shared memory;
//   warp 17    signaller: publishes stored tiles to the other CTAs (one GPU-scope fence and
//              one counter add per batch of tiles), so that the fence's latency stalls no
//              consumer.
//   At the end the consumer warps sum each owned row in route order and store it; the
//   last CTA out resets the tile counters (graph replay needs no memset).
// Every wait is bounded (kWaitLimitNs) and records an error code.
#include <cuda.h>

#include <array>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "fnx_common.cuh"
#include "fnx_kernels.h"

namespace fnx {

namespace {

constexpr int kLnGroups = 4;
constexpr int kLnGroupWarps = 4;
constexpr int kLnConsumers = kLnGroups * kLnGroupWarps;
constexpr int kLnSignalWarp = 1 + kLnConsumers;
constexpr int kLnThreads = (2 + kLnConsumers) * 32;
constexpr int kLnMaxM = 1;  // measured on B200: M = 1 18.96 vs 19.56 us (general one-launch
                            // layer), M = 2 29.7 vs 27.1 us; the code serves M <= 2
constexpr int kLnSlotsPerItem = kLnGroupWarps;  // down: one slot per warp of the group
constexpr int kLnMaxIch = 4;                    // I / 128 held in registers (I <= 512)
constexpr int kLnMaxQ = 4;                      // k steps of a tile's quarter (H <= 2048)

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t lds_u16(const uint8_t* p) {
  return *reinterpret_cast<const unsigned short*>(p);
}

// TMA box loads (no multicast) into this CTA's shared memory, completing on bar.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            int c3, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)),
      "l"(pol)
      : "memory");
}

// A bounded mbarrier wait whose outcome is the same on every lane of the warp.
__device__ __forceinline__ bool warp_all_wait(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

}  // namespace

// Shared-memory layout (identical on host and device, offsets from a 1024-aligned base).
// Stage = one gate/up tile (up box, gate box: 8 rows x H/2 B each, then the two scale sets
// of H/64 x 32 B) or four down slots (box of 16 rows x I/2 B, then I/64 x 64 B of scales,
// each slot 1024-aligned for the swizzled box).
struct LeanLayout {
  int pitch1, tile1, pitch2, slot2, stage;
  int ring, xs, acts, aun, red, res, rw, rslot, bitmap, wbase, sexp, stok, sg13, sg2, unscale,
      bars, misc, total;
  int nblk, dcap;
};

__host__ __device__ inline int ln_align(int v, int a) { return (v + a - 1) / a * a; }

__host__ __device__ inline LeanLayout lean_layout(int M, int R, int E, int H, int I, int NS, int G) {
  LeanLayout L;
  L.pitch1 = 8 * (H / 2);                 // bytes of one 8-row box
  L.tile1 = 2 * L.pitch1 + H;
  L.pitch2 = 16 * (I / 2);                // bytes of one 16-row box
  L.slot2 = ln_align(L.pitch2 + I, 1024);
  const int t2 = kLnSlotsPerItem * L.slot2;
  L.stage = ln_align(L.tile1 > t2 ? L.tile1 : t2, 1024);
  const int n = M * R;
  L.nblk = (H / 16 + G - 1) / G;
  L.dcap = (E < n ? E : n) + 1;
  int off = 0;
  L.ring = off;
  off += NS * L.stage;
  L.xs = off;
  off += M * stage_row_bytes(H);
  L.acts = off;                           // act rows (slot, token) as scaled fp16, B order
  off += L.dcap * M * stage_row_bytes(I);
  L.aun = off;                            // their unscale factors
  off += ln_align(L.dcap * M * 4, 16);
  L.red = off;                            // [group][buffer][4 warps][32 lanes] float4
  off += kLnGroups * 2 * kLnGroupWarps * 32 * 16;
  L.res = off;                            // [nblk][M][R + 1][16] per-route row results
  off += L.nblk * M * (R + 1) * 16 * 4;
  L.rw = off;
  off += ln_align(n * 4, 16);
  L.rslot = off;
  off += ln_align(n * 2, 16);
  const int nw = (E + 31) / 32;
  L.bitmap = off;
  off += ln_align(nw * 4, 16);
  L.wbase = off;
  off += ln_align(nw * 4, 16);
  L.sexp = off;
  off += ln_align(L.dcap * 2, 16);
  L.stok = off;
  off += ln_align(L.dcap * 4, 16);
  L.sg13 = off;                           // global scales of each slot's w13 and w2
  off += ln_align(L.dcap * 4, 16);
  L.sg2 = off;
  off += ln_align(L.dcap * 4, 16);
  L.unscale = off;
  off += 32 * 4;
  L.bars = off;                           // full[NS], empty[NS], redfull/redfree [groups][2]
  off += (2 * NS + 4 * kLnGroups) * 8;
  L.misc = off;                           // D, the groups' stored-tile counts, the go flag
  off += 32;
  L.total = off + 1024;                   // slack to align the dynamic base to 1024 bytes
  return L;
}

// Tensor maps (uint8) of the routed [0..3] and shared [4..7] experts: w13 rows, w13
// scales, w2 rows, w2 scales.
//   rows:   {128 B, 32-row group, row in group, 128-byte chunk}; a tile box {128, 4, 2, H/256}
//           takes rows 32 q + 2p + h (q < 4, h < 2) and lands as [chunk][h][q][128 B], so
//           the 16-byte units of MMA rows g and g + 1 are 64 bytes apart after the swizzle;
//           a down box {128, 4, 4, I/256} takes rows 32 q + 4p + i as [chunk][i][q][128 B];
//   scales: {512 B, kb4, 128-row block, ...}: a box takes one 32 (64)-byte piece per kb4.
struct LeanArgs {
  CUtensorMap maps[8];
  MoeArgs a;
  int NS;
};

namespace {

// Output row of down block b, MMA row r (0..15): the 16 rows share 64-byte scale pieces.
__device__ __forceinline__ int ln_down_row(int b, int r) {
  return (b >> 3) * 128 + (r >> 2) * 32 + 4 * (b & 7) + (r & 3);
}
// Act column of gate/up tile u (of a slot), MMA row g (0..7).
__device__ __forceinline__ int ln_up_col(int u, int g) {
  return (u >> 4) * 128 + (g >> 1) * 32 + 2 * (u & 15) + (g & 1);
}

// First tile of CTA c: [c W / G - (bytes of the down blocks of CTAs < c)] / p1 rounded,
// clamped to [0, T]; monotone in c and T at c = G (the tiles balance the down blocks, of
// d_bytes each, that CTA c owns: blocks c, c + G, ... of NB).
__device__ __forceinline__ int ln_tile_bound(int c, int G, int T, int NB, long long p1,
                                             long long d_bytes) {
  const long long q = NB / G, rm = NB % G;
  const long long blocks_before = q * c + (c < rm ? c : rm);
  const long long W = (long long)T * p1 + (long long)NB * d_bytes;
  long long num = (long long)c * W - (long long)G * d_bytes * blocks_before;
  const long long den = (long long)G * p1;
  if (num < 0) num = 0;
  long long v = (num + den / 2) / den;
  return (int)(v < T ? v : T);
}

}  // namespace

__global__ void __launch_bounds__(kLnThreads, 1) moe_lean_kernel(const __grid_constant__ LeanArgs A) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const MoeArgs& a = A.a;
  const int NS = A.NS;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int M = a.M, R = a.R, H = a.H, I = a.I, E = a.E;
  const int G = gridDim.x, cta = blockIdx.x;
  const LeanLayout L = lean_layout(M, R, E, H, I, NS, G);
  uint8_t* ring = smem + L.ring;
  uint8_t* xs = smem + L.xs;
  float4* red = reinterpret_cast<float4*>(smem + L.red);
  float* res = reinterpret_cast<float*>(smem + L.res);
  float* rw = reinterpret_cast<float*>(smem + L.rw);
  short* rslot = reinterpret_cast<short*>(smem + L.rslot);
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(smem + L.bitmap);
  int* wbase = reinterpret_cast<int*>(smem + L.wbase);
  short* sexp = reinterpret_cast<short*>(smem + L.sexp);
  uint32_t* stok = reinterpret_cast<uint32_t*>(smem + L.stok);
  float* sg13 = reinterpret_cast<float*>(smem + L.sg13);
  float* sg2 = reinterpret_cast<float*>(smem + L.sg2);
  float* unscale = reinterpret_cast<float*>(smem + L.unscale);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + NS;
  uint64_t* redfull = empty + NS;           // [group][buffer]
  uint64_t* redfree = redfull + 2 * kLnGroups;
  int* misc = reinterpret_cast<int*>(smem + L.misc);
  unsigned* cnt = a.cnt;                    // [0] tiles stored (layer), [1] CTAs done
  const int n = M * R;
  const int nw = (E + 31) / 32;
  const int sh = a.has_shared ? 1 : 0;

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kLnGroupWarps);
    }
    for (int b = 0; b < 2 * kLnGroups; ++b) {
      mbar_init(&redfull[b], kLnGroupWarps - 1);
      mbar_init(&redfree[b], 1);
    }
    mbar_fence_init();
    for (int g2 = 1; g2 <= kLnGroups; ++g2) misc[g2] = 0;
  }
  if (warp == 0 && lane == 0)
    for (int i = 0; i < 8; ++i)
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&A.maps[i])) : "memory");
  for (int i = tid; i < nw; i += kLnThreads) bitmap[i] = 0u;
  for (int i = tid; i < L.dcap; i += kLnThreads) stok[i] = 0u;
  // The routing, the activations and the counters are written by earlier kernels.
  pdl_wait();
  __syncthreads();

  // ---------------------------------------------------------------- routing decode
  for (int i = tid; i < n; i += kLnThreads) {
    const int id = __ldcg(a.ids + i);  // [M, R] row-major: entry i = t * R + r
    const int loc = id - a.e_lo;
    const bool ok = id >= 0 && loc >= 0 && loc < E;
    rslot[i] = (short)(ok ? loc : -1);
    rw[i] = __ldcg(a.wts + i);
    if (ok) atomicOr(&bitmap[loc >> 5], 1u << (loc & 31));
  }
  __syncthreads();
  if (warp == 0) {
    int running = 0;
    for (int base = 0; base < nw; base += 32) {
      const int w = base + lane;
      const int pc = w < nw ? __popc(bitmap[w]) : 0;
      int scan = pc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, scan, o);
        if (lane >= o) scan += v;
      }
      if (w < nw) wbase[w] = sh + running + scan - pc;
      running += __shfl_sync(0xffffffffu, scan, 31);
    }
    if (lane == 0) misc[0] = sh + running;
  }
  __syncthreads();
  for (int i = tid; i < n; i += kLnThreads) {
    const int e = rslot[i];
    if (e >= 0) {
      const int d = wbase[e >> 5] + __popc(bitmap[e >> 5] & ((1u << (e & 31)) - 1u));
      rslot[i] = (short)d;
      atomicOr(&stok[d], 1u << (i / R));
    }
  }
  for (int w = tid; w < nw; w += kLnThreads) {
    uint32_t m = bitmap[w];
    int d = wbase[w];
    while (m) {
      sexp[d++] = (short)(w * 32 + __ffs(m) - 1);
      m &= m - 1;
    }
  }
  if (sh && tid == 0) {
    sexp[0] = -1;
    stok[0] = (1u << M) - 1u;
  }
  __syncthreads();

  const int D = misc[0];
  const int T1 = I / 8;                    // tiles per slot
  const int T = D * T1;
  const int NB = H / 16;                   // down blocks
  const long long p1 = 16LL * (H / 2) + H;                        // bytes of one tile
  const long long d_bytes = (long long)D * (16LL * (I / 2) + I);  // one block, all slots
  const int t_lo = ln_tile_bound(cta, G, T, NB, p1, d_bytes);
  const int t_hi = ln_tile_bound(cta + 1, G, T, NB, p1, d_bytes);
  const int n1 = t_hi - t_lo;
  const int my_blocks = cta < NB ? (NB - cta + G - 1) / G : 0;
  const int ngrp = (D + kLnSlotsPerItem - 1) / kLnSlotsPerItem;
  const int n_items = n1 + my_blocks * ngrp;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    const uint64_t pol = policy_evict_first();
    int issued = 0;
    for (int j = 0; j < n_items; ++j) {
      const int s = j % NS;
      if (j >= NS && !mbar_wait(&empty[s], ((j / NS) & 1) ^ 1)) {
        if (lane == 0) record_error(a.err, ERR_WAIT_EMPTY);
        break;
      }
      uint8_t* st = ring + (size_t)s * L.stage;
      if (lane == 0) {
        if (j < n1) {
          const int tau = t_lo + j, d = tau / T1, u = tau - d * T1;
          const int e = sexp[d];
          const CUtensorMap* mw = &A.maps[e >= 0 ? 0 : 4];
          const CUtensorMap* ms = &A.maps[e >= 0 ? 1 : 5];
          const int ee = e >= 0 ? e : 0;
          mbar_arrive_expect_tx(&full[s], (uint32_t)L.tile1);
          const int rg = (ee * 2 * I + (u >> 4) * 128) / 32;  // up rows' first 32-row group
          tma_load_4d(st, mw, 0, rg, 2 * (u & 15), 0, &full[s], pol);
          tma_load_4d(st + L.pitch1, mw, 0, rg + I / 32, 2 * (u & 15), 0, &full[s], pol);
          tma_load_4d(st + 2 * L.pitch1, ms, 32 * (u & 15), 0, u >> 4, 2 * ee, &full[s], pol);
        } else {
          const int k = j - n1, bi = k / ngrp, grp = k - bi * ngrp;
          const int b = cta + bi * G;
          const int d0 = grp * kLnSlotsPerItem;
          const int ns = D - d0 < kLnSlotsPerItem ? D - d0 : kLnSlotsPerItem;
          mbar_arrive_expect_tx(&full[s], (uint32_t)(ns * (L.pitch2 + I)));
          for (int sl = 0; sl < ns; ++sl) {
            const int e = sexp[d0 + sl];
            const CUtensorMap* mw = &A.maps[e >= 0 ? 2 : 6];
            const CUtensorMap* ms = &A.maps[e >= 0 ? 3 : 7];
            const int ee = e >= 0 ? e : 0;
            uint8_t* dst = st + sl * L.slot2;
            tma_load_4d(dst, mw, 0, (ee * H + (b >> 3) * 128) / 32, 4 * (b & 7), 0, &full[s], pol);
            tma_load_3d(dst + L.pitch2, ms, 64 * (b & 7), 0, ee * (H / 128) + (b >> 3), &full[s], pol);
          }
        }
      }
      __syncwarp();
      issued = j + 1;
    }
    // no copy may still be landing when the CTA exits
    if (lane == 0)
      for (int j = issued > NS ? issued - NS : 0; j < issued; ++j)
        if (!mbar_wait(&full[j % NS], (j / NS) & 1)) record_error(a.err, ERR_DRAIN);
    __syncwarp();
  } else if (warp == kLnSignalWarp) {
    // ------------------------------------------------------------------ signaller
    // Each pass takes the tiles both groups have stored since the last pass, fences once
    // at GPU scope (cumulative: the consumers' act stores were ordered before their
    // CTA-scope counts, which this warp has read) and adds them to the layer's counter.
    volatile int* stored = &misc[1];
    int done = 0;
    const unsigned long long t0 = global_ns();
    while (done < n1) {
      int now = 0;
#pragma unroll
      for (int g2 = 0; g2 < kLnGroups; ++g2) now += stored[g2];
      if (now == done) {
        if (global_ns() - t0 > kWaitLimitNs) {
          if (lane == 0) record_error(a.err, ERR_WAIT_RED);
          break;
        }
        __nanosleep(20);
        continue;
      }
      __threadfence();
      if (lane == 0) atomicAdd(&cnt[0], (unsigned)(now - done));
      done = now;
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ consumers
    const int cw = warp - 1, grp = cw / kLnGroupWarps, wg = cw % kLnGroupWarps;
    const int g = lane >> 2, c = lane & 3;
    for (int d = tid - 32; d < D; d += kLnConsumers * 32) {  // visible after the staging
      const int e = sexp[d];
      sg13[d] = e >= 0 ? __ldg(a.g13 + (size_t)e * a.g13_stride) : __ldg(a.sh_g13);
      sg2[d] = e >= 0 ? __ldg(a.g2 + (size_t)e * a.g2_stride) : __ldg(a.sh_g2);
    }
    // x rows as fp16 scaled by each token's power of two, in the fragment order
    stage_rows_bulk<W_NVFP4, false>(xs, unscale, M, 0, H, reinterpret_cast<const __nv_bfloat16*>(a.x),
                                    a.ldx, NormGate{}, nullptr, a.err, true, 32, kLnConsumers * 32, 1);
    group_sync(1, kLnConsumers * 32);
    const int srow = stage_row_bytes(H);
    const int S = H / 128, s_lo = wg * S / kLnGroupWarps, s_hi = (wg + 1) * S / kLnGroupWarps;
    // ---------------------------------------------------------------- gate/up tiles
    // Warp wg of the group reduces k steps [s_lo, s_hi) of every tile.  Four accumulator
    // sets (16-byte word parity x MMA half) keep the MMAs of a step independent; they are
    // summed in a fixed order.  The warp that combines a tile's four
    // k quarters rotates with the tile, so the epilogue's work is spread over the group.
    const int sg = ((g & 1) << 2) | (g >> 1);  // box line of MMA row g within a chunk
    int ntile = 0;
    bool ok = true;
    for (int j = grp; j < n1; j += kLnGroups, ++ntile) {
      const int s = j % NS;
      const uint8_t* st = ring + (size_t)s * L.stage;
      const int tau = t_lo + j, d = tau / T1, u = tau - d * T1;
      if (!warp_all_wait(&full[s], (j / NS) & 1)) {
        if (lane == 0) record_error(a.err, ERR_WAIT_FULL);
        ok = false;
        break;
      }
      float acc[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
      const uint8_t* ra = st + sg * 128;
      const uint8_t* scu = st + 2 * L.pitch1 + 16 * (g & 1) + 4 * (g >> 1) + 2 * (c & 1);
      const uint8_t* scg = scu + (H / 64) * 32;
      const uint8_t* xg = xs + (size_t)(g < M ? g : 0) * srow + c * 16;
      for (int ks = s_lo; ks < s_hi; ++ks) {
        const int off = (ks >> 1) * 1024 + (((((ks & 1) << 2) | c) ^ sg) << 4);
        const uint4 va = lds128(ra + off), vb = lds128(ra + L.pitch1 + off);
        const int pc = 2 * ks + (c >> 1);
        const uint32_t fa = e4m3x2_to_f16x2(lds_u16(scu + pc * 32));
        const uint32_t fb = e4m3x2_to_f16x2(lds_u16(scg + pc * 32));
        uint4 x4[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          x4[q] = g < M ? lds128(xg + (ks * 4 + q) * 64) : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t wa[4] = {va.x, va.y, va.z, va.w}, wb[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {  // word q: k 8q .. 8q + 7 of this lane's 32
          uint32_t ha[4], hb[4];
          deq_e2m1_word(wa[q], ha);
          deq_e2m1_word(wb[q], hb);
          const uint32_t s_a = q < 2 ? bcast_lo(fa) : bcast_hi(fa);
          const uint32_t s_b = q < 2 ? bcast_lo(fb) : bcast_hi(fb);
#pragma unroll
          for (int h = 0; h < 2; ++h)
            mma_f16(acc[((q & 1) << 1) | h], hmul2(ha[2 * h], s_a), hmul2(hb[2 * h], s_b),
                    hmul2(ha[2 * h + 1], s_a), hmul2(hb[2 * h + 1], s_b), h ? x4[q].z : x4[q].x,
                    h ? x4[q].w : x4[q].y);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v.x += acc[i][0];
        v.y += acc[i][1];
        v.z += acc[i][2];
        v.w += acc[i][3];
      }
      // combine the four k quarters in the leader (warp ntile % 4 of the group)
      const int leader = ntile & (kLnGroupWarps - 1);
      const int rb_i = grp * 2 + (ntile & 1);
      const uint32_t rph = (ntile >> 1) & 1;
      float4* rbuf = red + (size_t)rb_i * kLnGroupWarps * 32;
      if (wg != leader) {
        if (ntile >= 2 && !warp_all_wait(&redfree[rb_i], rph ^ 1)) {
          if (lane == 0) record_error(a.err, ERR_WAIT_RFREE);
          ok = false;
          break;
        }
        rbuf[wg * 32 + lane] = v;
        __syncwarp();
        if (lane == 0) mbar_arrive(&redfull[rb_i]);
        continue;
      }
      if (!warp_all_wait(&redfull[rb_i], rph)) {
        if (lane == 0) record_error(a.err, ERR_WAIT_RED);
        ok = false;
        break;
      }
      float4 tot = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int w = 0; w < kLnGroupWarps; ++w) {  // the four k quarters, in k order
        const float4 p = w == wg ? v : rbuf[w * 32 + lane];
        tot.x += p.x;
        tot.y += p.y;
        tot.z += p.z;
        tot.w += p.w;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&redfree[rb_i]);
      // lane (g, c): up and gate of act column ln_up_col(u, g) for tokens 2c, 2c + 1
      const float gsc = sg13[d];
      const uint32_t tm = stok[d];
      const int col = ln_up_col(u, g);
      const float ov[4] = {tot.x, tot.y, tot.z, tot.w};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int t = 2 * c + h;
        if (t < M && ((tm >> t) & 1u)) {
          const float us = unscale[t];
          const float upv = ov[h] * us * gsc;
          const float gv = ov[2 + h] * us * gsc;
          reinterpret_cast<__nv_bfloat16*>(a.act)[((size_t)d * M + t) * I + col] =
              __float2bfloat16_rn(silu_f32(gv) * upv);
        }
      }
      __syncwarp();
      if (lane == 0) {
        __threadfence_block();
        atomicAdd(reinterpret_cast<unsigned*>(&misc[1 + grp]), 1u);  // tile stored
      }
    }
    // ---------------------------------------------------------------- down blocks
    uint8_t* acts = smem + L.acts;
    float* aun = reinterpret_cast<float*>(smem + L.aun);
    const int arow = stage_row_bytes(I);
    if (my_blocks > 0) {
      group_sync(2, kLnConsumers * 32);
      if (cw == 0) {  // every tile of the layer stored and published
        bool got = true;
        if (lane == 0) {
          const unsigned long long t0 = global_ns();
          while (ld_acquire_u32(&cnt[0]) < (unsigned)T) {
            if (global_ns() - t0 > kWaitLimitNs) {
              got = false;
              break;
            }
            __nanosleep(32);
          }
          if (!got) record_error(a.err, ERR_WAIT_EXPERT);
          misc[1 + kLnGroups] = got ? 1 : 0;
        }
        __syncwarp();
      }
      group_sync(2, kLnConsumers * 32);  // warp 1 lane 0's acquire orders the loads below
      if (misc[1 + kLnGroups] == 0) ok = false;
      // act rows (slot d, token t) -> scaled fp16 in the B-fragment order, one warp per row
      for (int r = cw; ok && r < D * M; r += kLnConsumers) {
        const int d = r / M, t = r - d * M;
        const bool has = (stok[d] >> t) & 1u;
        const uint8_t* src = a.act + (size_t)r * I * 2;
        uint4 v[kLnMaxIch];
        float m = 0.f;
#pragma unroll
        for (int q = 0; q < kLnMaxIch; ++q) {  // 8 values per unit, units lane + 32 q
          const int u = lane + 32 * q;
          v[q] = (has && u < I / 8) ? ldg_cg_u4(src + u * 16) : make_uint4(0u, 0u, 0u, 0u);
          m = fmaxf(m, bf16x8_absmax(v[q]));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const int e = stage_exponent(m);
#pragma unroll
        for (int q = 0; q < kLnMaxIch; ++q) {
          const int u = lane + 32 * q;
          if (u < I / 8)
            *reinterpret_cast<uint4*>(acts + (size_t)r * arow + stage_unit_offset<W_NVFP4>(8 * u)) =
                bf16x8_to_f16x8_scaled(v[q], e);
        }
        if (lane == 0) aun[r] = pow2f(-e);
      }
      group_sync(2, kLnConsumers * 32);
    }
    for (int j = n1 + ((grp - n1) % kLnGroups + kLnGroups) % kLnGroups; ok && j < n_items;
         j += kLnGroups) {
      const int s = j % NS;
      const uint8_t* st = ring + (size_t)s * L.stage;
      const int k = j - n1, bi = k / ngrp, gi = k - bi * ngrp;
      const int d = gi * kLnSlotsPerItem + wg;  // this warp's slot of the item
      const bool live = d < D;
      if (!warp_all_wait(&full[s], (j / NS) & 1)) {
        if (lane == 0) record_error(a.err, ERR_WAIT_FULL);
        ok = false;
        break;
      }
      float acc[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
      const uint32_t tm = live ? stok[d] : 0u;
      if (live) {
        // MMA row r = box line 16 chunk + 4 (r & 3) + (r >> 2); rows g and g + 8
        const uint8_t* tile = st + wg * L.slot2;
        const int la = ((g & 3) << 2) | (g >> 2), lb = la + 2;
        const uint8_t* sca = tile + L.pitch2 + 16 * (g & 3) + 4 * (g >> 2) + 2 * (c & 1);
        const bool hasb = g < M && ((tm >> g) & 1u);
        const uint8_t* xb = acts + (size_t)(d * M + (g < M ? g : 0)) * arow + c * 16;
#pragma unroll
        for (int ks = 0; ks < kLnMaxIch; ++ks) {
          if (ks >= I / 128) break;
          const int uu = ((ks & 1) << 2) | c;
          const uint8_t* cb = tile + (ks >> 1) * 2048;
          const uint4 va = lds128(cb + la * 128 + ((uu ^ (la & 7)) << 4));
          const uint4 vb = lds128(cb + lb * 128 + ((uu ^ (lb & 7)) << 4));
          const int pc = 2 * ks + (c >> 1);
          const uint32_t fa = e4m3x2_to_f16x2(lds_u16(sca + pc * 64));
          const uint32_t fb = e4m3x2_to_f16x2(lds_u16(sca + pc * 64 + 8));
          uint4 x4[4];
#pragma unroll
          for (int q = 0; q < 4; ++q)
            x4[q] = hasb ? lds128(xb + (ks * 4 + q) * 64) : make_uint4(0u, 0u, 0u, 0u);
          const uint32_t wa[4] = {va.x, va.y, va.z, va.w}, wb[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t ha[4], hb[4];
            deq_e2m1_word(wa[q], ha);
            deq_e2m1_word(wb[q], hb);
            const uint32_t s_a = q < 2 ? bcast_lo(fa) : bcast_hi(fa);
            const uint32_t s_b = q < 2 ? bcast_lo(fb) : bcast_hi(fb);
#pragma unroll
            for (int h = 0; h < 2; ++h)
              mma_f16(acc[((q & 1) << 1) | h], hmul2(ha[2 * h], s_a), hmul2(hb[2 * h], s_b),
                      hmul2(ha[2 * h + 1], s_a), hmul2(hb[2 * h + 1], s_b), h ? x4[q].z : x4[q].x,
                      h ? x4[q].w : x4[q].y);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (!live) continue;
      // lane (g, c): rows g and g + 8 of the block for tokens 2c, 2c + 1
      const float g2 = sg2[d];
      float ov[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) ov[r] = ((acc[0][r] + acc[1][r]) + acc[2][r]) + acc[3][r];
      float* rblk = res + (size_t)bi * M * (R + 1) * 16;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int t = 2 * c + h;
        if (t >= M || !((tm >> t) & 1u)) continue;
        const float un = aun[d * M + t];
        const float y0 = ov[h] * un, y1 = ov[2 + h] * un;
        float* rt = rblk + (size_t)t * (R + 1) * 16;
        for (int r = 0; r < R; ++r)
          if (rslot[t * R + r] == d) {
            const float f = g2 * rw[t * R + r];
            rt[r * 16 + g] = y0 * f;
            rt[r * 16 + g + 8] = y1 * f;
          }
        if (sh && d == 0) {
          const float f = g2 * 1.f;
          rt[R * 16 + g] = y0 * f;
          rt[R * 16 + g + 8] = y1 * f;
        }
      }
    }
    // ---------------------------------------------------------------- route sums
    group_sync(1, kLnConsumers * 32);
    const int ct = tid - 32;
    for (int bi = 0; bi < my_blocks; ++bi) {
      const int b = cta + bi * G;
      const float* rblk = res + (size_t)bi * M * (R + 1) * 16;
      for (int idx = ct; idx < M * 16; idx += kLnConsumers * 32) {
        const int t = idx >> 4, r16 = idx & 15;
        const float* rt = rblk + (size_t)t * (R + 1) * 16 + r16;
        float v = 0.f;
        for (int r = 0; r < R; ++r) v += rslot[t * R + r] >= 0 ? rt[r * 16] : 0.f;
        if (sh) v += rt[R * 16];
        const int nrow = ln_down_row(b, r16);
        if (a.out_f32)
          reinterpret_cast<float*>(a.out)[(size_t)t * a.ldo + nrow] = v;
        else
          reinterpret_cast<__nv_bfloat16*>(a.out)[(size_t)t * a.ldo + nrow] = __float2bfloat16_rn(v);
      }
    }
  }
  // ---------------------------------------------------------------- counters back to 0
  pdl_trigger();
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(&cnt[1], 1u);
    if (prev == (unsigned)G - 1) {  // every CTA is past its counter reads and adds
      __threadfence();
      atomicExch(&cnt[0], 0u);
      atomicExch(&cnt[1], 0u);
    }
  }
}

namespace {
constexpr size_t kLnMaxSmem = 227 * 1024;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver's tensor-map encoder, found through the runtime (no link against libcuda).
EncodeTiledFn lean_encoder() {
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

// One uint8 tensor map of `rank` dims (the inner dim contiguous).
bool lean_map(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims,
              const cuuint64_t* strides, const cuuint32_t* box, bool swizzle) {
  EncodeTiledFn enc = lean_encoder();
  if (!enc || !base) return false;
  const cuuint32_t es[5] = {1, 1, 1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, (cuuint32_t)rank, const_cast<void*>(base), dims, strides,
             box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
             swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The four maps of one expert bank of Et experts (layouts described at LeanArgs).
bool lean_bank_maps(CUtensorMap* m, const uint8_t* w13, const uint8_t* s13, const uint8_t* w2,
                    const uint8_t* s2, int Et, int H, int I) {
  const uint64_t rb1 = H / 2, rb2 = I / 2, kp1 = H / 16, kp2 = I / 16;
  {
    const cuuint64_t dims[4] = {128, (cuuint64_t)Et * 2 * I / 32, 32, rb1 / 128};
    const cuuint64_t str[3] = {32 * rb1, rb1, 128};
    const cuuint32_t box[4] = {128, 4, 2, (cuuint32_t)(rb1 / 128)};
    if (!lean_map(&m[0], w13, 4, dims, str, box, true)) return false;
  }
  {
    const cuuint64_t dims[4] = {512, kp1 / 4, (cuuint64_t)I / 128, (cuuint64_t)2 * Et};
    const cuuint64_t str[3] = {512, 128 * kp1, (uint64_t)(I / 128) * 128 * kp1};
    const cuuint32_t box[4] = {32, (cuuint32_t)(kp1 / 4), 1, 2};
    if (!lean_map(&m[1], s13, 4, dims, str, box, false)) return false;
  }
  {
    const cuuint64_t dims[4] = {128, (cuuint64_t)Et * H / 32, 32, rb2 / 128};
    const cuuint64_t str[3] = {32 * rb2, rb2, 128};
    const cuuint32_t box[4] = {128, 4, 4, (cuuint32_t)(rb2 / 128)};
    if (!lean_map(&m[2], w2, 4, dims, str, box, true)) return false;
  }
  {
    const cuuint64_t dims[3] = {512, kp2 / 4, (cuuint64_t)Et * H / 128};
    const cuuint64_t str[2] = {512, 128 * kp2};
    const cuuint32_t box[3] = {64, (cuuint32_t)(kp2 / 4), 1};
    if (!lean_map(&m[3], s2, 3, dims, str, box, false)) return false;
  }
  return true;
}

// Encoded maps are kept per (bank pointers, shape): a layer's weights do not move.
struct LeanMapKey {
  const void *w13, *s13, *w2, *s2;
  int Et, H, I;
  bool operator<(const LeanMapKey& o) const {
    return std::tie(w13, s13, w2, s2, Et, H, I) < std::tie(o.w13, o.s13, o.w2, o.s2, o.Et, o.H, o.I);
  }
};

bool lean_bank_maps_cached(CUtensorMap* m, const uint8_t* w13, const uint8_t* s13, const uint8_t* w2,
                           const uint8_t* s2, int Et, int H, int I) {
  static std::mutex mu;
  static std::map<LeanMapKey, std::array<CUtensorMap, 4>> cache;
  const LeanMapKey k{w13, s13, w2, s2, Et, H, I};
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(k);
    if (it != cache.end()) {
      memcpy(m, it->second.data(), 4 * sizeof(CUtensorMap));
      return true;
    }
  }
  if (!lean_bank_maps(m, w13, s13, w2, s2, Et, H, I)) return false;
  std::lock_guard<std::mutex> g(mu);
  if (cache.size() > 4096) cache.clear();
  std::array<CUtensorMap, 4> v;
  memcpy(v.data(), m, 4 * sizeof(CUtensorMap));
  cache[k] = v;
  return true;
}

}  // namespace

bool moe_lean_plan(int M, int R, int E, int H, int I, int grid, int& NS, size_t& smem) {
  // 128-byte chunks of whole rows (TMA boxes): H / 2 and I / 2 multiples of 128
  if (M < 1 || M > kLnMaxM || H % 256 || I % 256 || I / 128 > kLnMaxIch || H < 512 ||
      H / 128 > kLnGroupWarps * kLnMaxQ || E > 4096 || R < 1 || R > 32 || grid < 1)
    return false;
  const LeanLayout L0 = lean_layout(M, R, E, H, I, 0, grid);
  int ns = (int)(((long long)kLnMaxSmem - L0.total - 64) / (L0.stage + 16));
  if (ns > 12) ns = 12;
  ns -= ns % kLnGroups;  // every stage is consumed by one group
  if (ns < kLnGroups) return false;
  NS = ns;
  smem = (size_t)lean_layout(M, R, E, H, I, NS, grid).total;
  return smem <= kLnMaxSmem;
}

int64_t moe_lean_counters(int M, int R, int E) {
  (void)M;
  (void)R;
  (void)E;
  return 2;
}

int launch_moe_lean(const MoeArgs& a, int NS, int grid, size_t smem, cudaStream_t stream) {
  if (!prepare_kernel((const void*)moe_lean_kernel)) return 2;
  LeanArgs A;
  memset(&A, 0, sizeof(A));
  if (!lean_bank_maps_cached(&A.maps[0], a.w13, a.s13, a.w2, a.s2, a.E, a.H, a.I)) return 3;
  if (a.has_shared) {
    if (!lean_bank_maps_cached(&A.maps[4], a.sh_w13, a.sh_s13, a.sh_w2, a.sh_s2, 1, a.H, a.I)) return 3;
  } else {
    memcpy(&A.maps[4], &A.maps[0], 4 * sizeof(CUtensorMap));
  }
  A.a = a;
  A.NS = NS;
  return launch_with_pdl((const void*)moe_lean_kernel, A, grid, kLnThreads, smem, a.pdl, stream);
}

}  // namespace fnx
