// NVFP4 routed-MoE layer in ONE persistent launch (M <= 16 tokens).
//
// Replaces the reference's one-token Triton pair (patches/sglang/series/0112-...patch:
// 182-227 gate/up + SiLU, :229-287 down + route sum) and the three-launch form of
// moe_gemv.cu for the tilings it is compiled for.  Same weight contract and numerics:
//   act[t, r, :] = bf16( silu(g13 * <gate, x_t>) * g13 * <up, x_t> )         (0112:220-224)
//   out[t, :]    = bf16( sum_r w[t, r] * g2 * <W2, act[t, r]>  + shared expert )
// with the route sum in route order, then the shared expert (deterministic).
//
// Work items.  Distinct routed experts (and the always-on shared expert) are split into
// VIRTUAL experts of at most 8 routes each (one 8-column MMA block), so no route is ever
// dropped whatever the routing (repeated ids, many tokens on one expert).  A virtual
// expert contributes I / 8 gate/up TILES (16 weight rows: up and gate rows of 8 columns
// of I taken from the four 32-row quadrants of a 128-column block, whose swizzled scales
// are then contiguous 32-byte pieces) and H / 64 down HALF-BLOCKS (64 rows of H over I).
// Items are numbered tiles first (virtual-expert major), then half-blocks; CTA c takes
// items c, c + grid, ... and streams them through ONE shared-memory ring in that order,
// so a CTA's down weights are loaded while its own and the other CTAs' tiles compute.
//
// Roles: warp 0 issues the ring's bulk copies; NG groups of four consumer warps take the
// CTA's items round robin (group g: items g, g + NG, ...).
//  * tile: each warp of the group reduces one quarter of H (k slice) with mma.sync in
//    swap-AB form; warps 1..3 hand their partial C tile to warp 0 through shared memory;
//    warp 0 sums the four in order, applies the global scale and the per-token power of
//    two, SiLU(gate) * up, stores the bf16 act row (in the down projection's B-operand
//    order) and release-increments the virtual expert's tile counter.
//  * half-block: each warp waits (bounded) until its virtual expert's I / 8 tiles are
//    all done, loads that expert's act rows, converts its slots to fp16 scaled by a power
//    of two (exact) and folds 2^-e * g2 * route weight into one factor per slot; then
//    each warp streams one 16-row tile over all of I and stores its per-(token, route)
//    partials.  The group that completes a 64-row output block (the last of its V
//    contributions, counted by a release/acquire counter) sums that block's partials in
//    route order, then the shared expert's, rounds once, and resets the counter.
// Every counter returns to zero within the call (graph-replay safe, no memset).
//
// Every wait is an mbarrier or counter wait bounded by kWaitLimitNs; an expired wait
// records an error code in the workspace and ends the waiting role's loop.  The only
// named barrier runs once, before the loops, over all consumer warps.  The kernel
// relies on its CTAs running concurrently (one per SM, grid <= SMs): a half-block waits
// for tiles of other CTAs.
#include "fnx_common.cuh"
#include "fnx_kernels.h"

namespace fnx {

namespace {

struct FRoute {
  short* lid;        // [n] local expert id of route i = t * R + r, or -1
  uint32_t* bitmap;  // [nw] routed experts
  int* wbase;        // [nw] distinct slots before each bitmap word
  short* exp_of;     // [dcap] local expert of distinct slot d (ascending)
  short* cnt_of;     // [dcap] routes of distinct slot d
  short* vbase;      // [dcap] first virtual expert of distinct slot d
  uint8_t* ctab;     // [nchunk][dcap] routes of d in each 32-route chunk
  uint8_t* rrank;    // [n] rank of a route among its chunk's routes to the same expert
  short* rdist;      // [n] distinct slot of a route, or -1
  uint8_t* etok;     // [n] token of a route
  short* vexp;       // [vcap] local expert of virtual expert v, -1 = shared
  uint8_t* vnum;     // [vcap] routes of v (1..8)
  short* vent;       // [vcap][8] route entry of slot s (shared: -1 - token)
  int* misc;         // [0] distinct experts D, [1] virtual experts V
};

__device__ __forceinline__ FRoute froute_view(uint8_t* smem, const FusedLayout& L) {
  FRoute r;
  r.lid = reinterpret_cast<short*>(smem + L.lid);
  r.bitmap = reinterpret_cast<uint32_t*>(smem + L.bitmap);
  r.wbase = reinterpret_cast<int*>(smem + L.wbase);
  r.exp_of = reinterpret_cast<short*>(smem + L.exp_of);
  r.cnt_of = reinterpret_cast<short*>(smem + L.cnt_of);
  r.vbase = reinterpret_cast<short*>(smem + L.vbase);
  r.ctab = smem + L.ctab;
  r.rrank = smem + L.rrank;
  r.rdist = reinterpret_cast<short*>(smem + L.rdist);
  r.etok = smem + L.etok;
  r.vexp = reinterpret_cast<short*>(smem + L.vexp);
  r.vnum = smem + L.vnum;
  r.vent = reinterpret_cast<short*>(smem + L.vent);
  r.misc = reinterpret_cast<int*>(smem + L.misc);
  return r;
}

// The routing table, decoded by every CTA (CTA-wide, ends with __syncthreads): experts
// in ascending id order, each expert's routes in route order, cut into virtual experts of
// at most 8 routes; the shared expert (if any) comes first as ceil(M / 8) virtual experts.
__device__ void froute_decode(const MoeArgs& a, const FRoute& rt, int vcap) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nthreads = blockDim.x, nwarps = nthreads >> 5;
  const int R = a.R, M = a.M;
  const int n = M * R;
  const int nw = (a.E + 31) / 32;
  const int nchunk = (n + 31) / 32;
  const int dcap = a.E < n ? a.E : n;
  const int nsh = a.has_shared ? (M + kFusedSlots - 1) / kFusedSlots : 0;
  for (int i = tid; i < nw; i += nthreads) rt.bitmap[i] = 0u;
  for (int i = tid; i < nchunk * dcap; i += nthreads) rt.ctab[i] = 0;
  for (int i = tid; i < n; i += nthreads) {
    const int id = __ldcg(a.ids + i);  // [M, R] row-major: entry i = t * R + r
    const int loc = id - a.e_lo;
    rt.lid[i] = (short)((id >= 0 && loc >= 0 && loc < a.E) ? loc : -1);
    rt.etok[i] = (uint8_t)(i / R);
  }
  __syncthreads();
  for (int i = tid; i < n; i += nthreads) {
    const int e = rt.lid[i];
    if (e >= 0) atomicOr(&rt.bitmap[e >> 5], 1u << (e & 31));
  }
  __syncthreads();
  if (warp == 0) {
    int running = 0;
    for (int base = 0; base < nw; base += 32) {
      const int w = base + lane;
      const int pc = (w < nw) ? __popc(rt.bitmap[w]) : 0;
      int scan = pc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, scan, o);
        if (lane >= o) scan += v;
      }
      if (w < nw) rt.wbase[w] = running + scan - pc;
      running += __shfl_sync(0xffffffffu, scan, 31);
    }
    if (lane == 0) rt.misc[0] = running;
  }
  __syncthreads();
  for (int w = tid; w < nw; w += nthreads) {
    uint32_t m = rt.bitmap[w];
    int d = rt.wbase[w];
    while (m) {
      const int b = __ffs(m) - 1;
      rt.exp_of[d++] = (short)(w * 32 + b);
      m &= m - 1;
    }
  }
  for (int k = warp; k < nchunk; k += nwarps) {  // one warp per 32-route chunk
    const int i = k * 32 + lane;
    const int e = i < n ? rt.lid[i] : -1;
    int d = -1;
    if (e >= 0) d = rt.wbase[e >> 5] + __popc(rt.bitmap[e >> 5] & ((1u << (e & 31)) - 1u));
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (i < n) {
      rt.rrank[i] = (uint8_t)rank;
      rt.rdist[i] = (short)d;
    }
    if (e >= 0 && rank == 0) rt.ctab[k * dcap + d] = (uint8_t)__popc(peers);
  }
  __syncthreads();
  const int D = rt.misc[0];
  for (int d = tid; d < D; d += nthreads) {
    int cnt = 0;
    for (int k = 0; k < nchunk; ++k) cnt += rt.ctab[k * dcap + d];
    rt.cnt_of[d] = (short)cnt;
  }
  __syncthreads();
  if (warp == 0) {  // virtual experts: exclusive prefix sum of ceil(cnt / 8), after the shared ones
    int running = nsh;
    for (int base = 0; base < D; base += 32) {
      const int d = base + lane;
      const int nv = d < D ? (rt.cnt_of[d] + kFusedSlots - 1) / kFusedSlots : 0;
      int scan = nv;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, scan, o);
        if (lane >= o) scan += v;
      }
      if (d < D) rt.vbase[d] = (short)(running + scan - nv);
      running += __shfl_sync(0xffffffffu, scan, 31);
    }
    if (lane == 0) {
      if (running > vcap) {  // cannot happen for vcap = fused_vcap(M, R, E)
        record_error(a.err, ERR_ROUTES);
        running = 0;
      }
      rt.misc[1] = running;
    }
  }
  __syncthreads();
  if (rt.misc[1] == 0 && D + nsh > 0) return;  // table overflow: nothing is computed
  for (int i = tid; i < n; i += nthreads) {
    const int d = rt.rdist[i];
    if (d < 0) continue;
    int slot = rt.rrank[i];
    for (int k = 0; k < (i >> 5); ++k) slot += rt.ctab[k * dcap + d];
    const int v = rt.vbase[d] + slot / kFusedSlots;
    rt.vent[v * kFusedSlots + slot % kFusedSlots] = (short)i;
  }
  for (int d = tid; d < D; d += nthreads) {
    const int cnt = rt.cnt_of[d];
    for (int j = 0; j * kFusedSlots < cnt; ++j) {
      const int v = rt.vbase[d] + j;
      rt.vexp[v] = rt.exp_of[d];
      const int left = cnt - j * kFusedSlots;
      rt.vnum[v] = (uint8_t)(left < kFusedSlots ? left : kFusedSlots);
    }
  }
  for (int q = tid; q < nsh * kFusedSlots; q += nthreads) {
    const int v = q / kFusedSlots, s = q % kFusedSlots;
    if (s == 0) {
      rt.vexp[v] = -1;
      const int left = M - v * kFusedSlots;
      rt.vnum[v] = (uint8_t)(left < kFusedSlots ? left : kFusedSlots);
    }
    rt.vent[q] = (short)(-1 - q);
  }
  __syncthreads();
}

__device__ __forceinline__ int fentry_token(const FRoute& rt, int entry) {
  return entry < 0 ? -1 - entry : rt.etok[entry];
}

// (token, route) pair row of an entry in the partials: t * (R + 1) + r; shared: r = R.
__device__ __forceinline__ int fentry_pair(const FRoute& rt, int entry, int R) {
  return entry < 0 ? (-1 - entry) * (R + 1) + R : entry + rt.etok[entry];
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

}  // namespace

template <int CPW1, int CPW2>
__global__ void __launch_bounds__(kFusedThreads, 1) moe_fused_kernel(const MoeArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int Q = Geo<W_NVFP4>::Q;
  constexpr int kWF = kFusedProd;                       // first fetcher warp
  constexpr int kWE = kFusedProd + kFusedFetch;         // first epilogue warp
  constexpr int kW0 = kFusedProd + kFusedFetch + kFusedEpi;  // first consumer warp
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int M = a.M, R = a.R, H = a.H, I = a.I, NS = a.NS, NG = a.NG;
  if (NS % kFusedRing != 0 || NG != kFusedMaxGroups) {  // a ring the parity waits cannot order
    if (tid == 0) record_error(a.err, ERR_RING);
    return;
  }
  const FusedLayout L = fused_layout(M, R, a.E, H, I, NS, a.vcap);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + NS;
  uint64_t* xbar = empty + NS;
  uint64_t* afull = xbar + 1;
  uint64_t* aempty = afull + kFusedAct;
  uint64_t* rfull = aempty + kFusedAct;
  uint64_t* rfree = rfull + kFusedRes;
  uint8_t* stages = smem + L.stages;
  uint8_t* xs = smem + L.xs;
  float* unscale = reinterpret_cast<float*>(smem + L.unscale);
  const FRoute rt = froute_view(smem, L);
  const int KP1 = H / 16, KP2 = I / 16;
  const int J = KP1 / 4;                // 4-byte scale groups per row of a tile
  const int T1 = I / 8, T2 = H / 64;    // tiles and half-blocks per virtual expert
  const int P = M * (R + 1);
  const int srow = stage_row_bytes(H), brow = stage_row_bytes(I);
  const int g = lane >> 2, c = lane & 3;
  const int pg = phys_lo(g), pg8 = phys_hi(g);
  const int G = gridDim.x, cta = blockIdx.x;
  const int nsh = a.has_shared ? (M + kFusedSlots - 1) / kFusedSlots : 0;
  unsigned* done1 = a.cnt;                   // [vcap] finished tiles of virtual expert v
  unsigned* cnt2 = a.cnt + a.vcap;           // [H / 64] contributions to a 64-row block
  unsigned* cnt_all = cnt2 + T2;             // completed 64-row blocks

  int* lastk = reinterpret_cast<int*>(smem + L.lastk);
  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1 + 32);  // bulk-copy arrival + one cp.async arrival per lane
      mbar_init(&empty[s], 4);
      lastk[s] = -1;
    }
    mbar_init(xbar, 1);
    for (int q = 0; q < kFusedAct; ++q) {
      mbar_init(&afull[q], 1);
      mbar_init(&aempty[q], 4);
    }
    for (int q = 0; q < kFusedRes; ++q) {
      mbar_init(&rfull[q], 4);
      mbar_init(&rfree[q], 1);
    }
    mbar_fence_init();
  }
  __syncthreads();

  // Column index i (0..7) of gate/up tile u: column 128 (u / 16) + 32 (i / 2) + 2 (u % 16)
  // + i % 2 (two columns from each 32-row quadrant of a 128-column block).
  auto col_of = [&](int tile, int i) { return (tile >> 4) * 128 + (i >> 1) * 32 + 2 * (tile & 15) + (i & 1); };

  // ---- producer helpers (warp 0; every lane calls them) ----
  auto issue_tile = [&](int s, int e, int tile) {
    const uint64_t pol = policy_evict_first();
    const uint8_t* wq = e >= 0 ? a.w13 + (size_t)e * (2 * I) * L.ub1 : a.sh_w13;
    const uint8_t* sq = e >= 0 ? a.s13 + (size_t)e * (2 * I) * KP1 : a.sh_s13;
    uint8_t* st = stages + (size_t)s * L.stage_bytes;
    if (lane == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)(16 * L.ub1));
    __syncwarp();
    if (lane < 8) {  // lane = half * 4 + quadrant: the rows of column indices 2q, 2q + 1
      const int half = lane >> 2, q = lane & 3;
      const int row = half * I + col_of(tile, 2 * q);
      bulk_g2s(st + tile_row_offset(half * 8 + 2 * q, L.ub1), wq + (size_t)row * L.ub1,
               (uint32_t)(2 * L.ub1), &full[s], pol);
    }
    if (a.swizzled) {  // per half and 512-byte block j: rows 2p, 2p + 1, 16 bytes each
      const int blk = tile >> 4, r0 = 2 * (tile & 15);
      for (int half = 0; half < 2; ++half) {
        const uint8_t* src = sq + (size_t)(blk + half * (I / 128)) * 128 * KP1 + r0 * 16;
        for (int jj = lane; jj < 2 * J; jj += 32)
          cp_async16(st + L.soff1 + (half * J * 2 + jj) * 16, src + (jj >> 1) * 512 + (jj & 1) * 16);
      }
    } else {
      const int sp = dense_align(KP1, 16);
      for (int r = 0; r < 16; ++r) {
        const int m = (r >> 3) * I + col_of(tile, r & 7);
        for (int j = lane; j < KP1 / 8; j += 32)
          cp_async8(st + L.soff1 + r * sp + 8 * j, sq + (size_t)m * KP1 + 8 * j);
      }
    }
    if (lane == 0) cp_async4(st + L.foff1, e >= 0 ? a.g13 + (size_t)e * a.g13_stride : a.sh_g13);
    cp_async_arrive(&full[s]);
  };
  auto issue_half = [&](int s, int e, int hb) {
    const uint64_t pol = policy_evict_first();
    const uint8_t* wq = (e >= 0 ? a.w2 + (size_t)e * H * L.ub2 : a.sh_w2) + (size_t)hb * 64 * L.ub2;
    const uint8_t* sb = e >= 0 ? a.s2 + (size_t)e * H * KP2 : a.sh_s2;
    uint8_t* st = stages + (size_t)s * L.stage_bytes;
    const uint32_t sbytes = a.swizzled ? 128 * KP2 : 64 * KP2;
    if (lane == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)(64 * L.ub2) + sbytes);
    __syncwarp();
    if (lane < 8) {  // lane = tile * 2 + half: 8 contiguous rows
      const int t = lane >> 1, h = lane & 1;
      bulk_g2s(st + t * L.tb2 + tile_row_offset(8 * h, L.ub2), wq + (size_t)(16 * t + 8 * h) * L.ub2,
               (uint32_t)(8 * L.ub2), &full[s], pol);
    } else if (lane == 8) {
      const uint8_t* src = a.swizzled ? sb + (size_t)(hb >> 1) * 128 * KP2 : sb + (size_t)hb * 64 * KP2;
      bulk_g2s(st + L.soff2, src, sbytes, &full[s], pol);
    }
    cp_async_arrive(&full[s]);
  };

  // The shared expert's first tiles do not depend on the routing: a CTA whose first item
  // is one of them starts streaming it before the previous kernel has finished.
  const bool pre0 = warp == 0 && cta < nsh * T1;  // producer warp 0 owns item 0
  if (pre0) {
    issue_tile(0, -1, cta % T1);
    if (lane == 0) lastk[0] = 0;
  }

  pdl_wait();  // x and topk_ids come from earlier kernels
  if (tid == 0) issue_x_rows(xs, M, 0, H, reinterpret_cast<const __nv_bfloat16*>(a.x), a.ldx, xbar);
  froute_decode(a, rt, a.vcap);  // ends with __syncthreads
  // Every CTA of this grid has started here, so a dependent grid cannot take an SM that a
  // CTA of this one still needs: it may launch now.
  pdl_trigger();
  const int V = rt.misc[1];
  const int n1tot = V * T1;
  const int total = V * (T1 + T2);
  const int my = cta < total ? (total - cta + G - 1) / G : 0;
  const int n1 = cta < n1tot ? (n1tot - cta + G - 1) / G : 0;  // this CTA's tiles come first

  if (V == 0 || my == 0) {
    if (V == 0) {  // no route reaches this expert slice and there is no shared expert
      for (int q = cta * blockDim.x + tid; q < M * H; q += G * blockDim.x) {
        const int t = q / H, nn = q - t * H;
        if (a.out_f32) reinterpret_cast<float*>(a.out)[(size_t)t * a.ldo + nn] = 0.f;
        else reinterpret_cast<__nv_bfloat16*>(a.out)[(size_t)t * a.ldo + nn] = __float2bfloat16_rn(0.f);
      }
    }
    if (tid == 0 && !mbar_wait(xbar, 0)) record_error(a.err, ERR_DRAIN);  // x copy landed
    return;
  }

  if (warp < kWF) {
    // ---------------------------------------------------------------- producers
    // producer warp p issues items p, p + kFusedProd, ... (in ring order per warp)
    for (int k = warp + ((pre0 && warp == 0) ? kFusedProd : 0); k < my; k += kFusedProd) {
      const int s = k % NS;
      if (k >= NS && !mbar_wait(&empty[s], ((k / NS) & 1) ^ 1)) {
        record_error(a.err, ERR_WAIT_EMPTY);
        break;
      }
      const int idx = cta + k * G;
      if (lane == 0) lastk[s] = k;
      if (idx < n1tot) {
        const int v = idx / T1;
        issue_tile(s, rt.vexp[v], idx - v * T1);
      } else {
        const int j = idx - n1tot, v = j / T2;
        issue_half(s, rt.vexp[v], j - v * T2);
      }
    }
    // Nothing may land after the CTA exits: once every producer warp is done issuing, wait
    // for the last item issued into each stage (earlier ones landed before their stage
    // was reused).  A stage that never received an item holds -1.
    group_sync(2, kFusedProd * 32);
    if (warp == 0)
      for (int st = lane; st < NS; st += 32) {
        const int k = lastk[st];
        if (k >= 0 && !mbar_wait(&full[st], (k / NS) & 1)) record_error(a.err, ERR_DRAIN);
      }
    return;
  }

  if (warp < kWE) {
    // ---------------------------------------------------------------- act fetchers
    // Half-block j of this CTA (fetcher j % kFusedFetch): wait until its virtual expert's
    // tiles have all stored their act values, load its route rows (bf16, B-operand order),
    // convert each to fp16 scaled by 2^e (max |act| in [2^14, 2^15), exact) into act slot
    // j % kFusedAct, with the row's factor 2^-e * g2 * route weight after it.
    const int f = warp - kWF;
    constexpr int kU = 4;  // 16-byte units per lane per row (I <= 1024)
    for (int j = f; n1 + j < my; j += kFusedFetch) {
      const int idx = cta + (n1 + j) * G;
      const int jj = idx - n1tot, v = jj / T2;
      const int vn = rt.vnum[v], e = rt.vexp[v];
      const int as = j % kFusedAct;
      if (!mbar_wait(&aempty[as], ((j / kFusedAct) & 1) ^ 1)) {
        record_error(a.err, ERR_WAIT_EMPTY);
        break;
      }
      bool ok = true;
      if (lane == 0) {
        const unsigned long long t0 = global_ns();
        while (ld_acquire_gpu(&done1[v]) < (unsigned)T1) {
          if (global_ns() - t0 > kWaitLimitNs) {
            ok = false;
            break;
          }
          __nanosleep(32);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);  // lane 0's acquire orders the loads below
      if (!ok) {
        record_error(a.err, ERR_WAIT_EXPERT);
        break;
      }
      uint8_t* dst0 = smem + L.act + (size_t)as * L.act_bytes;
      const uint8_t* src0 = a.act + (size_t)v * kFusedSlots * brow;
      for (int s0 = 0; s0 < vn; s0 += 2) {  // two rows at a time: all their loads in flight
        uint4 u[2][kU];
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
          for (int q = 0; q < kU; ++q) {
            const int k8 = lane + 32 * q;
            u[r][q] = (s0 + r < vn && k8 < I / 8)
                          ? ldg_cg_u4(src0 + (size_t)(s0 + r) * brow + stage_unit_offset<W_NVFP4>(8 * k8))
                          : make_uint4(0u, 0u, 0u, 0u);
          }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          if (s0 + r >= vn) break;
          float m = 0.f;
#pragma unroll
          for (int q = 0; q < kU; ++q) m = fmaxf(m, bf16x8_absmax(u[r][q]));
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          const int ex = stage_exponent(m);
          uint8_t* dst = dst0 + (size_t)(s0 + r) * brow;
#pragma unroll
          for (int q = 0; q < kU; ++q) {
            const int k8 = lane + 32 * q;
            if (k8 < I / 8)
              *reinterpret_cast<uint4*>(dst + stage_unit_offset<W_NVFP4>(8 * k8)) =
                  bf16x8_to_f16x8_scaled(u[r][q], ex);
          }
          if (lane == 0) {
            const int entry = rt.vent[v * kFusedSlots + s0 + r];
            const float g2 = e >= 0 ? __ldg(a.g2 + (size_t)e * a.g2_stride) : __ldg(a.sh_g2);
            const float wr = entry >= 0 ? __ldg(a.wts + entry) : 1.f;
            *reinterpret_cast<float*>(dst + 2 * I) = pow2f(-ex) * (g2 * wr);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[as]);
    }
    return;
  }

  if (warp < kW0) {
    // ---------------------------------------------------------------- epilogue warps
    // Epilogue warp e takes the results of items e, e + kFusedEpi, ...  Its global stores
    // are released in batches: the results that are ready are stored, then one fence and
    // one counter update per item of the batch (lane i updates item i's counter), so a
    // fence's latency is paid once per batch, not once per item.  A batch closes when the
    // warp's next result is not ready yet, after 8 items, or when the item kind changes.
    const int ew = warp - kWE;
    int pend = -1;   // lane i: the virtual expert (tiles) or 64-row block (down) of item i
    int np = 0, ptype = 0;
    auto reduce_block = [&](int hb) {
      // the last contribution to rows [64 hb, 64 hb + 64): sum each token's route
      // partials in route order, then the shared expert's, and round once
      const float* base = a.part + (size_t)hb * P * 64;
      for (int q = lane; q < M * 16; q += 32) {
        const int t = q >> 4, r4 = (q & 15) * 4;
        const float* pb = base + (size_t)t * (R + 1) * 64 + r4;
        float4 acc4 = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r0 = 0; r0 <= R; r0 += 8) {  // 8 loads in flight, then sums in route order
          float4 pv[8];
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            const int r = r0 + jj;
            const bool live = r < R ? rt.lid[t * R + r] >= 0 : (r == R && a.has_shared);
            pv[jj] = live ? __ldcg(reinterpret_cast<const float4*>(pb + (size_t)r * 64))
                          : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            acc4.x += pv[jj].x;
            acc4.y += pv[jj].y;
            acc4.z += pv[jj].z;
            acc4.w += pv[jj].w;
          }
        }
        const int n0 = hb * 64 + r4;
        if (a.out_f32) {
          float* o32 = reinterpret_cast<float*>(a.out) + (size_t)t * a.ldo + n0;
          o32[0] = acc4.x;
          o32[1] = acc4.y;
          o32[2] = acc4.z;
          o32[3] = acc4.w;
        } else {
          __nv_bfloat16* o16 = reinterpret_cast<__nv_bfloat16*>(a.out) + (size_t)t * a.ldo + n0;
          o16[0] = __float2bfloat16_rn(acc4.x);
          o16[1] = __float2bfloat16_rn(acc4.y);
          o16[2] = __float2bfloat16_rn(acc4.z);
          o16[3] = __float2bfloat16_rn(acc4.w);
        }
      }
    };
    auto flush = [&]() {
      if (np == 0) return;
      __threadfence();  // this warp's act / partial stores, before any counter update
      __syncwarp();
      if (ptype == 1) {
        if (lane < np) atomicAdd(&done1[pend], 1u);  // tiles: release, no reply needed
      } else {
        const unsigned prev = lane < np ? atom_add_acq_rel_gpu(&cnt2[pend], 1u) : 0u;
        unsigned lastmask = __ballot_sync(0xffffffffu, lane < np && prev == (unsigned)(V - 1));
        while (lastmask) {
          const int l = __ffs(lastmask) - 1;
          lastmask &= lastmask - 1;
          const int hb = __shfl_sync(0xffffffffu, pend, l);
          __threadfence();
          reduce_block(hb);
          __syncwarp();
          if (lane == 0) {
            cnt2[hb] = 0u;
            // the last of all blocks: every half-block has read its act rows, so the tile
            // counters return to zero for the next call
            if (atom_add_acq_rel_gpu(cnt_all, 1u) == (unsigned)(T2 - 1)) {
              for (int q = 0; q < V; ++q) done1[q] = 0u;
              *cnt_all = 0u;
            }
          }
        }
      }
      np = 0;
      pend = -1;
    };
    for (int k = ew; k < my; k += kFusedEpi) {
      const int idx = cta + k * G;
      const int rs = k % kFusedRes;
      const int type = idx < n1tot ? 1 : 2;
      if (np > 0 && type != ptype) flush();
      if (!mbar_wait(&rfull[rs], (k / kFusedRes) & 1)) {
        record_error(a.err, ERR_WAIT_RED);
        break;
      }
      const float* res = reinterpret_cast<const float*>(smem + L.res + (size_t)rs * L.res_bytes);
      int key;
      if (type == 1) {
        // gate/up tile: sum the four k slices in order, then silu(g * gate) * (g * up)
        const int v = idx / T1, tile = idx - v * T1;
        const int vn = rt.vnum[v];
        float4 o = *reinterpret_cast<const float4*>(res + lane * 4);
#pragma unroll
        for (int w = 1; w < 4; ++w) {
          const float4 p = *reinterpret_cast<const float4*>(res + (w * 32 + lane) * 4);
          o.x += p.x;
          o.y += p.y;
          o.z += p.z;
          o.w += p.w;
        }
        const float gsc = res[4 * 32 * 4];
        __syncwarp();
        if (lane == 0) mbar_arrive(&rfree[rs]);
        const float ov[4] = {o.x, o.y, o.z, o.w};
        // MMA row g is physical row pg: the up row of column g for even g, the gate row
        // for odd g; MMA row g + 8 is the other one (0112-...patch:220-224).
        const bool odd = g & 1;
        const int col = col_of(tile, g);
        const int col_off = stage_unit_offset<W_NVFP4>(col & ~7) + (col & 7) * 2;
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const int sl = 2 * c + p;
          if (sl >= vn) continue;
          const int t = fentry_token(rt, rt.vent[v * kFusedSlots + sl]);
          const float us = unscale[t];
          const float upv = (odd ? ov[2 + p] : ov[p]) * us * gsc;
          const float gv = (odd ? ov[p] : ov[2 + p]) * us * gsc;
          *reinterpret_cast<__nv_bfloat16*>(a.act + (size_t)(v * kFusedSlots + sl) * brow + col_off) =
              __float2bfloat16_rn(silu_f32(gv) * upv);
        }
        key = v;
      } else {
        // down half-block: the four warps' 16-row tiles, already multiplied by the route
        // factors; store the per-(token, route) partials
        const int jj = idx - n1tot, v = jj / T2, hb = jj - v * T2;
        const int vn = rt.vnum[v];
        float ov[4][4];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const float4 p = *reinterpret_cast<const float4*>(res + (w * 32 + lane) * 4);
          ov[w][0] = p.x;
          ov[w][1] = p.y;
          ov[w][2] = p.z;
          ov[w][3] = p.w;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&rfree[rs]);
        float* base = a.part + (size_t)hb * P * 64;
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const int sl = 2 * c + p;
          if (sl >= vn) continue;
          const int pr = fentry_pair(rt, rt.vent[v * kFusedSlots + sl], R);
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            st_cg_f32(base + (size_t)pr * 64 + 16 * w + pg, ov[w][p]);
            st_cg_f32(base + (size_t)pr * 64 + 16 * w + pg8, ov[w][2 + p]);
          }
        }
        key = hb;
      }
      if (lane == np) pend = key;
      ++np;
      ptype = type;
      const int kn = k + kFusedEpi;
      const bool next_ready =
          kn < my && mbar_test(&rfull[kn % kFusedRes], (kn / kFusedRes) & 1);
      if (np == kFusedBatch || !next_ready) flush();
    }
    flush();
    return;
  }

  // ------------------------------------------------------------------ consumers
  const int ct0 = kW0 * 32, cnth = 4 * NG * 32;
  stage_rows_bulk<W_NVFP4, false>(xs, unscale, M, 0, H, reinterpret_cast<const __nv_bfloat16*>(a.x),
                                  a.ldx, NormGate{}, xbar, a.err, false, ct0, cnth, 1);
  group_sync(1, cnth);
  const int gi = (warp - kW0) >> 2, wg = (warp - kW0) & 3;
  if (gi >= NG) return;
  const int sp1 = dense_align(KP1, 16);

  for (int k = gi; k < my; k += NG) {
    const int idx = cta + k * G;
    const int s = k % NS, ph = (k / NS) & 1;
    const int rs = k % kFusedRes;
    const uint8_t* st = stages + (size_t)s * L.stage_bytes;
    float* res = reinterpret_cast<float*>(smem + L.res + (size_t)rs * L.res_bytes);
    float o[4];
    if (idx < n1tot) {
      // ------------------------------------------------------------ gate/up tile
      const int v = idx / T1;
      const int vn = rt.vnum[v];
      const int tok = g < vn ? fentry_token(rt, rt.vent[v * kFusedSlots + g]) : -1;
      if (!mbar_wait(&full[s], ph)) {
        record_error(a.err, ERR_WAIT_FULL);
        break;
      }
      // scale bytes (kb = 8 ch + 2 c, + 1) of physical row rho: swizzled stage layout
      // [half][j][row of pair][quadrant][4], linear [rho][KP1 padded]
      auto soff_of = [&](int rho) {
        if (!a.swizzled) return L.soff1 + rho * sp1 + c * 2;
        const int half = rho >> 3, i = rho & 7;
        return L.soff1 + ((half * J + (c >> 1)) * 2 + (i & 1)) * 16 + (i >> 1) * 4 + (c & 1) * 2;
      };
      const int offa = tile_row_offset(pg, L.ub1) + c * 16, offb = tile_row_offset(pg8, L.ub1) + c * 16;
      const int soffa = soff_of(pg), soffb = soff_of(pg8);
      const int sstep = a.swizzled ? 64 : 8;
      float acc[4][1][4];
#pragma unroll
      for (int h = 0; h < 4; ++h)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[h][0][r] = 0.f;
#pragma unroll
      for (int cc = 0; cc < CPW1; ++cc) {
        const int ch = wg * CPW1 + cc;
        const uint4 va = lds128(st + offa + ch * 64);
        const uint4 vb = lds128(st + offb + ch * 64);
        const uint32_t sa = *reinterpret_cast<const unsigned short*>(st + soffa + ch * sstep);
        const uint32_t sb = *reinterpret_cast<const unsigned short*>(st + soffb + ch * sstep);
        uint4 xf[1][Q];
#pragma unroll
        for (int q = 0; q < Q; ++q)
          xf[0][q] = tok >= 0 ? lds128(xs + (size_t)tok * srow + ((ch * Q + q) * 4 + c) * 16)
                              : make_uint4(0u, 0u, 0u, 0u);
        chunk_mma<W_NVFP4, 1>(acc[(2 * cc) % 4], acc[(2 * cc + 1) % 4], va, vb, sa, sb, xf, 1);
      }
      const float gsc = (wg == 0 && lane == 0) ? *reinterpret_cast<const float*>(st + L.foff1) : 0.f;
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
      for (int r = 0; r < 4; ++r) o[r] = (acc[0][0][r] + acc[1][0][r]) + (acc[2][0][r] + acc[3][0][r]);
      if (!mbar_wait(&rfree[rs], ((k / kFusedRes) & 1) ^ 1)) {
        record_error(a.err, ERR_WAIT_RFREE);
        break;
      }
      if (wg == 0 && lane == 0) res[4 * 32 * 4] = gsc;
    } else {
      // ------------------------------------------------------------ down half-block
      const int j = k - n1;  // this CTA's half-block ordinal (act slot j % kFusedAct)
      const int jj = idx - n1tot, v = jj / T2, hb = jj - v * T2;
      const int vn = rt.vnum[v];
      const int as = j % kFusedAct;
      const uint8_t* actb = smem + L.act + (size_t)as * L.act_bytes;
      if (!mbar_wait(&afull[as], (j / kFusedAct) & 1)) {
        record_error(a.err, ERR_WAIT_X);
        break;
      }
      if (!mbar_wait(&full[s], ph)) {
        record_error(a.err, ERR_WAIT_FULL);
        break;
      }
      // this warp's 16-row tile wg of the half-block, over all of I
      auto soff_of = [&](int r) {
        if (!a.swizzled) return L.soff2 + r * KP2 + c * 2;
        const int m = 64 * (hb & 1) + r;  // row within the 128-row scale block
        return L.soff2 + (c >> 1) * 512 + (m & 31) * 16 + (m >> 5) * 4 + (c & 1) * 2;
      };
      const int soffa = soff_of(16 * wg + pg), soffb = soff_of(16 * wg + pg8);
      const int sstep = a.swizzled ? 1024 : 8;
      const int offa = wg * L.tb2 + tile_row_offset(pg, L.ub2) + c * 16;
      const int offb = wg * L.tb2 + tile_row_offset(pg8, L.ub2) + c * 16;
      float acc[4][1][4];
#pragma unroll
      for (int h = 0; h < 4; ++h)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[h][0][r] = 0.f;
#pragma unroll
      for (int ch = 0; ch < CPW2; ++ch) {
        const uint4 va = lds128(st + offa + ch * 64);
        const uint4 vb = lds128(st + offb + ch * 64);
        const uint32_t sa = *reinterpret_cast<const unsigned short*>(st + soffa + ch * sstep);
        const uint32_t sb = *reinterpret_cast<const unsigned short*>(st + soffb + ch * sstep);
        uint4 xf[1][Q];
#pragma unroll
        for (int q = 0; q < Q; ++q)
          xf[0][q] = g < vn ? lds128(actb + (size_t)g * brow + ((ch * Q + q) * 4 + c) * 16)
                            : make_uint4(0u, 0u, 0u, 0u);
        chunk_mma<W_NVFP4, 1>(acc[(2 * ch) % 4], acc[(2 * ch + 1) % 4], va, vb, sa, sb, xf, 1);
      }
      float f[2];
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const int sl = 2 * c + p;
        f[p] = sl < vn ? *reinterpret_cast<const float*>(actb + (size_t)sl * brow + 2 * I) : 0.f;
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&empty[s]);
        mbar_arrive(&aempty[as]);
      }
#pragma unroll
      for (int r = 0; r < 4; ++r) o[r] = (acc[0][0][r] + acc[1][0][r]) + (acc[2][0][r] + acc[3][0][r]);
      o[0] *= f[0];
      o[1] *= f[1];
      o[2] *= f[0];
      o[3] *= f[1];
      if (!mbar_wait(&rfree[rs], ((k / kFusedRes) & 1) ^ 1)) {
        record_error(a.err, ERR_WAIT_RFREE);
        break;
      }
    }
    *reinterpret_cast<float4*>(res + (wg * 32 + lane) * 4) = make_float4(o[0], o[1], o[2], o[3]);
    __syncwarp();
    if (lane == 0) mbar_arrive(&rfull[rs]);
  }
}

namespace {

using FusedKernel = void (*)(const MoeArgs);

FusedKernel fused_ptr(int H, int I) {
  const int c1 = H / 512, c2 = I / 128;
  if (H % 512 || I % 128) return nullptr;
  if (c1 == 4 && c2 == 4) return moe_fused_kernel<4, 4>;   // H = 2048, I = 512
  if (c1 == 5 && c2 == 5) return moe_fused_kernel<5, 5>;   // H = 2560, I = 640
  if (c1 == 2 && c2 == 2) return moe_fused_kernel<2, 2>;   // H = 1024, I = 256
  if (c1 == 4 && c2 == 8) return moe_fused_kernel<4, 8>;   // H = 2048, I = 1024
  return nullptr;
}

}  // namespace

bool moe_fused_has(int H, int I) { return fused_ptr(H, I) != nullptr; }

int launch_moe_fused(const MoeArgs& a, int grid, size_t smem, cudaStream_t stream) {
  FusedKernel k = fused_ptr(a.H, a.I);
  if (!k) return 1;
  if (!prepare_kernel((const void*)k)) return 2;
  return launch_with_pdl((const void*)k, a, grid,
                         (kFusedProd + kFusedFetch + kFusedEpi + 4 * a.NG) * 32, smem, a.pdl, stream);
}

}  // namespace fnx
