// NVFP4 routed-MoE expert GEMV for M <= 16 tokens (decode and speculative verify).
//
// Replaces the reference's one-token Triton pair
//   _draft_moe_up_gate_kernel  patches/sglang/series/0112-...patch:182-227  (k1)
//   _draft_moe_down_kernel     0112-...patch:229-287                        (k2)
// and generalises it to M <= 16 with bf16 activations (W4A16), where the reference
// switches to FlashInfer's CUTLASS W4A4 chain.
//
// Weight contract (what ModelOptNvFp4FusedMoEMethod hands over, 0112-...patch:68-76):
//   w13 [E, 2I, H/2] uint8, rows [0, I) up and [I, 2I) gate, low nibble = even k;
//   w13 block scales e4m3 [E, 2I, H/16], 128x4 swizzled (or linear);
//   g13 = w13_weight_scale_2[e, 0] for both halves; w2 [E, H, I/2], scales, g2[e].
//
// Routing table.  Every CTA decodes topk_ids itself (an expert bitmap, a prefix count,
// and per distinct expert the list of routes that chose it, in route order), which
// costs a few hundred cycles and no extra launch.  Each distinct expert's rows are then
// streamed ONCE for all tokens routed to it: the tokens are the B operand of the
// tensor-core MMA, so verify widths cost D distinct experts, not M * top_k routes.
// Route ids < 0 (and ids outside this launch's expert slice) are skipped
// (0112-...patch:205, :259).
//
// k1 and k2 are persistent and warp-specialised like the dense GEMV: warp 0 stages each
// unit's weight rows (bulk copies) and its block scales and scalars in a shared-memory
// ring; consumer warps dequantise and run the MMAs.  Unit positions advance without
// integer division.
//
// k1 unit: (distinct expert, 8 columns of I) taken from the four 32-row quadrants of a
// 128-column block, so the swizzled scales of the unit are contiguous 32-byte pieces.
// MMA rows 0..7 are up rows, 8..15 the matching gate rows, so one epilogue lane holds
// both and applies silu(gate * g) * (up * g) (0112-...patch:220-224), rounding act to
// bf16.  Two epilogue warps take alternate units.  The act row of route slot s of
// distinct expert d is row d * 16 + s of the act buffer, stored in the down kernel's
// B-operand order; k1 needs no cross-CTA synchronisation.
// k2 unit: (distinct expert, 128-row block of H): weights and scales are one bulk copy
// each, the expert's act rows a third.  A converter warp finds each act row's max
// |act|, rewrites the row in place as fp16 scaled by a power of two (exact), and folds
// the inverse power of two, g2 and the route weight into one factor per route
// (0112-...patch:268-269).  Each consumer warp owns a 16-row tile over all of I and
// stores its scaled fp32 partial per (token, route) directly.
// k3 sums each token's route partials in route order, then the shared expert's, and
// rounds once to bf16: deterministic, no float atomics.  k2 and k3 are chained with
// programmatic dependent launch.
#include "fnx_common.cuh"
#include "fnx_kernels.h"

namespace fnx {

namespace {

constexpr int kSlotCap = kMoeSlotCap;

struct Routing {
  int* ids;          // [M*R] local expert id or -1
  uint32_t* bitmap;  // [nw]
  int* wbase;        // [nw]
  int* exp_of;       // [dcap] local expert id of distinct slot d (ascending)
  int* cnt_of;       // [dcap] routes of slot d
  short* ent;        // [dcap][16] route entries (t * R + r), ascending
  int* misc;         // misc[0] = D (distinct routed experts)
  uint8_t* ctab;     // [ceil(M*R / 32)][dcap] routes of slot d in each 32-route chunk
  uint8_t* rrank;    // [M*R] rank of a route among its chunk's routes to the same expert
  short* rdist;      // [M*R] distinct slot of a route, or -1
  uint8_t* etok;     // [M*R] token of a route entry
  short* epair;      // [M*R + M] (token, route) pair row of an entry; shared: M*R + t
};

__device__ inline Routing routing_view(uint8_t* smem, const MoeLayout& L) {
  Routing r;
  r.ids = reinterpret_cast<int*>(smem + L.ids);
  r.bitmap = reinterpret_cast<uint32_t*>(smem + L.bitmap);
  r.wbase = reinterpret_cast<int*>(smem + L.wbase);
  r.exp_of = reinterpret_cast<int*>(smem + L.exp_of);
  r.cnt_of = reinterpret_cast<int*>(smem + L.cnt_of);
  r.ent = reinterpret_cast<short*>(smem + L.ent);
  r.misc = reinterpret_cast<int*>(smem + L.misc);
  r.ctab = smem + L.ctab;
  r.rrank = smem + L.rrank;
  r.rdist = reinterpret_cast<short*>(smem + L.rdist);
  r.etok = smem + L.etok;
  r.epair = reinterpret_cast<short*>(smem + L.epair);
  return r;
}

// Build the routing table (CTA-wide; ends with __syncthreads).  Every step is a
// constant number of passes over the routes: a bitmap of the routed experts, its prefix
// count (the distinct slot d of each expert, ascending), then per 32-route chunk each
// route's rank among the chunk's routes to the same expert (__match_any_sync) and the
// chunk's per-slot counts; a route's slot inside its expert is its rank plus the counts
// of the earlier chunks, so slots follow route order.
__device__ void route_decode(const MoeArgs& a, const Routing& rt) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nthreads = blockDim.x, nwarps = nthreads >> 5;
  const int R = a.R, M = a.M;
  const int n = M * R;
  const int nw = (a.E + 31) / 32;
  const int nchunk = (n + 31) / 32;
  const int dcap = (a.E < n ? a.E : n) + 1;
  for (int i = tid; i < nw; i += nthreads) rt.bitmap[i] = 0u;
  for (int i = tid; i < nchunk * dcap; i += nthreads) rt.ctab[i] = 0;
  for (int i = tid; i < n; i += nthreads) {
    const int id = __ldcg(a.ids + i);  // [M, R] row-major: entry i = t * R + r
    const int loc = id - a.e_lo;
    rt.ids[i] = (id >= 0 && loc >= 0 && loc < a.E) ? loc : -1;
    const int t = i / R;
    rt.etok[i] = (uint8_t)t;
    rt.epair[i] = (short)(i + t);  // t * (R + 1) + r
  }
  for (int t = tid; t < M; t += nthreads) rt.epair[n + t] = (short)(t * (R + 1) + R);
  __syncthreads();
  for (int i = tid; i < n; i += nthreads) {
    const int e = rt.ids[i];
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
      rt.exp_of[d++] = w * 32 + b;
      m &= m - 1;
    }
  }
  // per chunk (one warp each): rank among same-expert routes, chunk counts
  for (int k = warp; k < nchunk; k += nwarps) {
    const int i = k * 32 + lane;
    const int e = i < n ? rt.ids[i] : -1;
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
  for (int i = tid; i < n; i += nthreads) {
    const int d = rt.rdist[i];
    if (d < 0) continue;
    int slot = rt.rrank[i];
    for (int k = 0; k < (i >> 5); ++k) slot += rt.ctab[k * dcap + d];
    if (slot < kSlotCap) rt.ent[d * kSlotCap + slot] = (short)i;
  }
  const int cap = a.NT == 2 ? kSlotCap : kSlotCap / 2;  // B columns of one unit
  for (int d = tid; d < D; d += nthreads) {
    int cnt = 0;
    for (int k = 0; k < nchunk; ++k) cnt += rt.ctab[k * dcap + d];
    // more routes on one expert than one unit's B columns: the surplus routes would be
    // dropped; report it (the fused form splits such experts instead)
    if (cnt > cap && blockIdx.x == 0) record_error(a.err, ERR_ROUTES);
    rt.cnt_of[d] = cnt < kSlotCap ? cnt : kSlotCap;
  }
  __syncthreads();
}

// Routes of the unit's expert: count, and the route entry (t * R + r) of slot s.
struct UnitRoutes {
  int n;           // live B columns (<= 8 * NT)
  bool shared;
  int d;
};

__device__ __forceinline__ int slot_entry(const Routing& rt, const UnitRoutes& ur, int s) {
  return ur.shared ? -1 - s : rt.ent[ur.d * kSlotCap + s];  // shared: -1 - token
}

// (token, route) pair row of a slot entry; the shared expert is route R of its token.
__device__ __forceinline__ int pair_of(const Routing& rt, int entry, int n) {
  return entry < 0 ? rt.epair[n - 1 - entry] : rt.epair[entry];
}

__device__ __forceinline__ int token_of(const Routing& rt, int entry) {
  return entry < 0 ? -1 - entry : rt.etok[entry];
}

}  // namespace

// ------------------------------------------------------------------------------------
// k1: act[d * 16 + s, j] = bf16(silu(g * <gate_j, x_t>) * g * <up_j, x_t>)
// ------------------------------------------------------------------------------------
template <int NT, int CPW>
__global__ void __launch_bounds__(kMoeUpThreads, 1) moe_up_kernel(const MoeArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int Q = Geo<W_NVFP4>::Q;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int M = a.M, R = a.R, H = a.H, I = a.I, W = a.W, NS = a.NS, RS = a.RS, EW = a.EW;
  const MoeLayout L = moe_layout(1, M, R, a.E, H, I, W, NS, RS, NT, 1);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + 2 * NS;
  uint64_t* rfull = empty + NS;
  uint64_t* rfree = rfull + RS;
  uint64_t* xbar = rfree + RS;  // bulk copy of the activation rows
  uint8_t* stages = smem + L.stages;
  uint8_t* xs = smem + L.xs;
  float* unscale = reinterpret_cast<float*>(smem + L.unscale);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* sred = reinterpret_cast<float*>(smem + L.sred);
  const Routing rt = routing_view(smem, L);
  const int srow = stage_row_bytes(H);
  const int KP = H / 16;
  const int UB = H / 2;
  const int g = lane >> 2, c = lane & 3;
  const int pg = phys_lo(g), pg8 = phys_hi(g);

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1 + 32);  // bulk-copy arrival + one cp.async arrival per lane
      mbar_init(&empty[s], W);
    }
    for (int r = 0; r < RS; ++r) {
      mbar_init(&rfull[r], W);
      mbar_init(&rfree[r], 1);
    }
    mbar_init(xbar, 1);
    mbar_fence_init();
  }
  // x and topk_ids come from earlier kernels.
  pdl_wait();
  // the activation rows travel by bulk copy while the routing table is decoded
  if (tid == 0) issue_x_rows(xs, M, 0, H, reinterpret_cast<const __nv_bfloat16*>(a.x), a.ldx, xbar);
  route_decode(a, rt);  // ends with __syncthreads (also publishes the barrier inits)
  // Every CTA is resident (the grid is one wave): the down kernel may launch now and take
  // each SM as this grid's CTA there exits, decoding its routes and prefetching W2 while
  // the other CTAs finish (it reads the act rows only after its griddepcontrol.wait).
  pdl_trigger();
  const int D = rt.misc[0];
  const int tiles = I / 8;
  const int n_units = (D + a.has_shared) * tiles;
  const int stride = gridDim.x, first = blockIdx.x;
  const int my_units = first < n_units ? (n_units - first + stride - 1) / stride : 0;

  auto routes_of = [&](int d) {
    UnitRoutes ur;
    ur.d = d;
    ur.shared = d >= D;
    const int n = ur.shared ? M : rt.cnt_of[d];
    ur.n = n < 8 * NT ? n : 8 * NT;
    return ur;
  };
  auto expert_id = [&](int d) { return d < D ? rt.exp_of[d] : -1; };
  // Unit tile u (0 .. I/8 - 1) covers 8 columns taken from the four 32-row quadrants of
  // one 128-column block: block b = u / 16, pair p = u % 16, and column index i (0..7)
  // is column 128 b + 32 (i / 2) + 2 p + i % 2.  In the 128x4 swizzled scale layout the
  // scales of rows {32 q + r} of a block sit together (16 bytes per r), so a unit's scales
  // are contiguous 32-byte pieces.  Physical rows 0..7 are the up rows of column indices
  // 0..7, rows 8..15 the gate rows (I + column).
  auto col_of = [&](int tile, int i) { return (tile >> 4) * 128 + (i >> 1) * 32 + 2 * (tile & 15) + (i & 1); };
  const int J = KP / 4;  // 4-byte scale groups per row (512-byte blocks per 128 rows)

  // Producer: eight 2-row weight blocks (up and gate rows of each quadrant pair) by bulk
  // copy; the unit's block scales and the expert's global scale by cp.async; all
  // complete on full[s].
  auto issue = [&](const UnitCursor& cu) {
    const uint64_t pol = policy_evict_first();
    const int s = cu.s, d = cu.q, tile = cu.r;
    const int e = expert_id(d);
    const uint8_t* wq = e >= 0 ? a.w13 + (size_t)e * (2 * I) * UB : a.sh_w13;
    const uint8_t* sq = e >= 0 ? a.s13 + (size_t)e * (2 * I) * KP : a.sh_s13;
    uint8_t* st = stages + (size_t)s * L.stage_bytes;
    if (lane == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)(16 * UB));
    __syncwarp();
    if (lane < 8) {  // lane = half * 4 + quadrant: rows of column indices 2q, 2q + 1
      const int half = lane >> 2, q = lane & 3;
      const int row = half * I + col_of(tile, 2 * q);
      bulk_g2s(st + tile_row_offset(half * 8 + 2 * q, UB), wq + (size_t)row * UB,
               (uint32_t)(2 * UB), &full[s], pol);
    }
    if (a.swizzled) {
      // per half and 512-byte block j: rows r = 2p, 2p + 1 of the block, 16 bytes each
      const int blk = tile >> 4, r0 = 2 * (tile & 15);
      for (int half = 0; half < 2; ++half) {
        const uint8_t* src = sq + (size_t)(blk + half * (I / 128)) * 128 * KP + r0 * 16;
        for (int jj = lane; jj < 2 * J; jj += 32)  // jj = 2 j + row
          cp_async16(st + L.soff + (half * J * 2 + jj) * 16, src + (jj >> 1) * 512 + (jj & 1) * 16);
      }
    } else {
      for (int r = 0; r < 16; ++r) {
        const int m = (r >> 3) * I + col_of(tile, r & 7);
        for (int j = lane; j < KP / 8; j += 32)
          cp_async8(st + L.soff + r * L.spitch + 8 * j, sq + (size_t)m * KP + 8 * j);
      }
    }
    if (lane == 0)
      cp_async4(st + L.foff, e >= 0 ? a.g13 + (size_t)e * a.g13_stride : a.sh_g13);
    cp_async_arrive(&full[s]);
  };

  UnitCursor pc;
  pc.init(first, stride, tiles, NS);
  if (warp == 0) {
    const int pre = my_units < NS ? my_units : NS;
    for (int i = 0; i < pre; ++i, pc.next()) issue(pc);
  }
  // The other warps stage the activations meanwhile; the producer never waits for them.
  if (warp > 0) {
    stage_rows_bulk<W_NVFP4, false>(xs, unscale, M, 0, H,
                                    reinterpret_cast<const __nv_bfloat16*>(a.x), a.ldx,
                                    NormGate{}, xbar, a.err, false, 32, blockDim.x - 32, 1);
    group_sync(1, blockDim.x - 32);
  }

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    int issued = my_units < NS ? my_units : NS;
    for (int i = NS; i < my_units; ++i, pc.next()) {
      if (!mbar_wait(&empty[pc.s], pc.ph ^ 1)) {
        record_error(a.err, ERR_WAIT_EMPTY);
        break;
      }
      issue(pc);
      issued = i + 1;
    }
    for (int j = issued > NS ? issued - NS : 0; j < issued; ++j)
      if (!mbar_wait(&full[j % NS], (j / NS) & 1)) record_error(a.err, ERR_DRAIN);
  } else if (warp > EW) {
    // ---------------------------------------------------------------- consumers
    const int cw = warp - 1 - EW;  // k slice of the unit
    const int offa = tile_row_offset(pg, UB) + c * 16;
    const int offb = tile_row_offset(pg8, UB) + c * 16;
    // scale bytes (kb = 8 ch + 2 c, +1) of physical row rho: swizzled stage layout
    // [half][j][row of pair][quadrant][4], linear [rho][KP]
    auto soff_of = [&](int rho) {
      if (!a.swizzled) return L.soff + rho * L.spitch + c * 2;
      const int half = rho >> 3, i = rho & 7;
      return L.soff + ((half * J + (c >> 1)) * 2 + (i & 1)) * 16 + (i >> 1) * 4 + (c & 1) * 2;
    };
    const int soffa = soff_of(pg), soffb = soff_of(pg8);
    const int sstep = a.swizzled ? 64 : 8;  // per 64-byte chunk (two 4-byte groups)
    UnitCursor cu;
    cu.init(first, stride, tiles, NS);
    int rs = 0, rph = 0;
    for (int i = 0; i < my_units; ++i, cu.next()) {
      const UnitRoutes ur = routes_of(cu.q);
      int tok[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int sl = nt * 8 + g;
        tok[nt] = sl < ur.n ? token_of(rt, slot_entry(rt, ur, sl)) : -1;
      }
      if (!mbar_wait(&full[cu.s], cu.ph)) {
        record_error(a.err, ERR_WAIT_FULL);
        break;
      }
      const uint8_t* st = stages + (size_t)cu.s * L.stage_bytes;
      constexpr int NC = NT == 1 ? 4 : 2;
      float acc[NC][NT][4];
#pragma unroll
      for (int h = 0; h < NC; ++h)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int r = 0; r < 4; ++r) acc[h][nt][r] = 0.f;
#pragma unroll
      for (int cc = 0; cc < CPW; ++cc) {
        const int ch = cw * CPW + cc;
        const uint4 va = lds128(st + offa + ch * 64);
        const uint4 vb = lds128(st + offb + ch * 64);
        const uint32_t sa = *reinterpret_cast<const unsigned short*>(st + soffa + ch * sstep);
        const uint32_t sb = *reinterpret_cast<const unsigned short*>(st + soffb + ch * sstep);
        uint4 xf[NT][Q];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int q = 0; q < Q; ++q)
            xf[nt][q] = tok[nt] >= 0
                            ? lds128(xs + (size_t)tok[nt] * srow + ((ch * Q + q) * 4 + c) * 16)
                            : make_uint4(0u, 0u, 0u, 0u);
        chunk_mma<W_NVFP4, NT>(acc[(2 * cc) % NC], acc[(2 * cc + 1) % NC], va, vb, sa, sb, xf,
                               ur.n > 8 ? 2 : 1);
      }
      const float gsc = (cw == 0 && lane == 0) ? *reinterpret_cast<const float*>(st + L.foff) : 0.f;
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[cu.s]);
      if (!mbar_wait(&rfree[rs], rph ^ 1)) {
        record_error(a.err, ERR_WAIT_RFREE);
        break;
      }
      float* dst = red + ((size_t)(rs * W + cw) * 32 + lane) * NT * 4;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float o[4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
          o[r] = NC == 4 ? (acc[0][nt][r] + acc[1][nt][r]) + (acc[2 % NC][nt][r] + acc[3 % NC][nt][r])
                         : acc[0][nt][r] + acc[1][nt][r];
        *reinterpret_cast<float4*>(dst + nt * 4) = make_float4(o[0], o[1], o[2], o[3]);
      }
      if (cw == 0 && lane == 0) sred[rs * 64] = gsc;
      __syncwarp();
      if (lane == 0) mbar_arrive(&rfull[rs]);
      if (++rs == RS) {
        rs = 0;
        rph ^= 1;
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue warps
    const int ew = warp - 1;
    const int bpitch = L.bpitch;
    UnitCursor cu;  // units ew, ew + EW, ... of this CTA; reduction slot ew
    cu.init(first + ew * stride, EW * stride, tiles, 1);
    for (int i = ew; i < my_units; i += EW, cu.next()) {
      const UnitRoutes ur = routes_of(cu.q);
      const int tile = cu.r;
      const int rs = ew;
      if (!mbar_wait(&rfull[rs], cu.ph)) {
        record_error(a.err, ERR_WAIT_RED);
        break;
      }
      const float gs = sred[rs * 64];
      float v[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float4 s0 = make_float4(0.f, 0.f, 0.f, 0.f), s1 = s0;
        int w = 0;
        for (; w + 1 < W; w += 2) {
          const float4 p = *reinterpret_cast<const float4*>(red + ((size_t)(rs * W + w) * 32 + lane) * NT * 4 + nt * 4);
          const float4 q = *reinterpret_cast<const float4*>(red + ((size_t)(rs * W + w + 1) * 32 + lane) * NT * 4 + nt * 4);
          s0.x += p.x; s0.y += p.y; s0.z += p.z; s0.w += p.w;
          s1.x += q.x; s1.y += q.y; s1.z += q.z; s1.w += q.w;
        }
        if (w < W) {
          const float4 p = *reinterpret_cast<const float4*>(red + ((size_t)(rs * W + w) * 32 + lane) * NT * 4 + nt * 4);
          s0.x += p.x; s0.y += p.y; s0.z += p.z; s0.w += p.w;
        }
        v[nt][0] = s0.x + s1.x;
        v[nt][1] = s0.y + s1.y;
        v[nt][2] = s0.z + s1.z;
        v[nt][3] = s0.w + s1.w;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&rfree[rs]);
      // MMA row g is physical row pg: the up row of column g for even g, the gate row
      // for odd g; MMA row g + 8 is the other one.
      const bool odd = g & 1;
      const int col = col_of(tile, g);  // column index g of the unit
      const int col_off = stage_unit_offset<W_NVFP4>(col & ~7) + (col & 7) * 2;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const int sl = nt * 8 + 2 * c + p;
          if (sl >= ur.n) continue;
          const int t = token_of(rt, slot_entry(rt, ur, sl));
          const float us = unscale[t];
          const float upv = (odd ? v[nt][2 + p] : v[nt][p]) * us * gs;
          const float gv = (odd ? v[nt][p] : v[nt][2 + p]) * us * gs;
          *reinterpret_cast<__nv_bfloat16*>(a.act + (size_t)(ur.d * kSlotCap + sl) * bpitch + col_off) =
              __float2bfloat16_rn(silu_f32(gv) * upv);
        }
    }
  }
}

// ------------------------------------------------------------------------------------
// k2: part[t, r, n] = w_{t,r} * g2_{e_r} * <W2[e_r, n], act_{t,r}>  (and the shared expert)
// ------------------------------------------------------------------------------------
// A unit is (distinct expert, 128-row block of H): its 128 weight rows are one
// contiguous bulk copy, and so are the block's scales in both layouts (the 128x4
// swizzled block, or 128 linear rows).  Each of the 8 consumer warps owns one 16-row
// tile over all of I, so its accumulators are final: it multiplies each route column by
// the route's factor and stores the partials itself, 32-byte pieces per (route, 8 rows).
// Partials live at part[((b * P + pair) * 128) + row], P = M * (R + 1).
template <int NT, int CPW>
__global__ void __launch_bounds__(kMoeDownThreads, 1) moe_down_kernel(const MoeArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int Q = Geo<W_NVFP4>::Q;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int M = a.M, R = a.R, H = a.H, I = a.I, NS = a.NS;
  const MoeLayout L = moe_layout(2, M, R, a.E, H, I, 8, NS, 0, NT, 8);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* cvt = full + NS;
  uint64_t* empty = cvt + NS;
  uint8_t* stages = smem + L.stages;
  const Routing rt = routing_view(smem, L);
  const int KP = I / 16;
  const int UB = I / 2;
  const int P = M * (R + 1);
  const int bpitch = L.bpitch;
  const int g = lane >> 2, c = lane & 3;

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1 + 32);
      mbar_init(&cvt[s], 1);
      mbar_init(&empty[s], 8);
    }
    mbar_fence_init();
  }
  // The route-sum kernel that follows may be scheduled now; it waits for this grid.
  pdl_trigger();
  // topk_ids were written before k1 started, and k1 lets this grid launch only after
  // its own griddepcontrol.wait, so they are visible here; the act rows are read after
  // this kernel's pdl_wait().
  route_decode(a, rt);
  const int D = rt.misc[0];
  const int Dtot = D + a.has_shared;
  const int blocks = H / 128;
  const int n_units = Dtot * blocks;
  const int stride = gridDim.x, first = blockIdx.x;
  const int my_units = first < n_units ? (n_units - first + stride - 1) / stride : 0;

  auto routes_of = [&](int d) {
    UnitRoutes ur;
    ur.d = d;
    ur.shared = d >= D;
    const int n = ur.shared ? M : rt.cnt_of[d];
    ur.n = n < 8 * NT ? n : 8 * NT;
    return ur;
  };
  auto expert_id = [&](int d) { return d < D ? rt.exp_of[d] : -1; };

  // Weights, block scales and the expert's scalars of a unit (valid before k1 ends);
  // the B rows follow after pdl_wait().  Everything completes on full[s].
  auto issue_weights = [&](const UnitCursor& cu, int brows) {
    const uint64_t pol = policy_evict_first();
    const int s = cu.s, d = cu.q, blk = cu.r;
    const int e = expert_id(d);
    const uint8_t* wq = (e >= 0 ? a.w2 + (size_t)e * H * UB : a.sh_w2) + (size_t)blk * 128 * UB;
    const uint8_t* sq = (e >= 0 ? a.s2 + (size_t)e * H * KP : a.sh_s2) + (size_t)blk * 128 * KP;
    uint8_t* st = stages + (size_t)s * L.stage_bytes;
    const UnitRoutes ur = routes_of(d);
    float* f = reinterpret_cast<float*>(st + L.foff);
    // plain stores first: lane 0's arrival below releases them to the stage's readers
    if (lane < ur.n && ur.shared) f[lane] = 1.f;
    __syncwarp();
    if (lane == 0) {
      mbar_arrive_expect_tx(&full[s], (uint32_t)(128 * UB + 128 * KP + brows * bpitch));
      bulk_g2s(st, wq, (uint32_t)(128 * UB), &full[s], pol);
      bulk_g2s(st + L.soff, sq, (uint32_t)(128 * KP), &full[s], pol);
    }
    // route weights [0, n) (the shared expert's are 1.0) and the global scale at [16]
    if (lane < ur.n && !ur.shared) cp_async4(f + lane, a.wts + slot_entry(rt, ur, lane));
    if (lane == 0) cp_async4(f + 16, e >= 0 ? a.g2 + (size_t)e * a.g2_stride : a.sh_g2);
    cp_async_arrive(&full[s]);
  };
  auto issue_brows = [&](const UnitCursor& cu) {
    const uint64_t pol = policy_evict_first();
    const UnitRoutes ur = routes_of(cu.q);
    if (lane == 0 && ur.n > 0)
      bulk_g2s(stages + (size_t)cu.s * L.stage_bytes + L.boff,
               a.act + (size_t)(ur.d * kSlotCap) * bpitch, (uint32_t)(ur.n * bpitch),
               &full[cu.s], pol);
  };

  const int pre = my_units < NS ? my_units : NS;
  UnitCursor pc;
  pc.init(first, stride, blocks, NS);
  if (warp == 0) {
    UnitCursor c0 = pc;
    for (int i = 0; i < pre; ++i, c0.next()) issue_weights(c0, routes_of(c0.q).n);
  }
  pdl_wait();  // the act rows may be read from here on

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    for (int i = 0; i < pre; ++i, pc.next()) issue_brows(pc);
    int issued = pre;
    for (int i = NS; i < my_units; ++i, pc.next()) {
      if (!mbar_wait(&empty[pc.s], pc.ph ^ 1)) {
        record_error(a.err, ERR_WAIT_EMPTY);
        break;
      }
      issue_weights(pc, routes_of(pc.q).n);
      issue_brows(pc);
      issued = i + 1;
    }
    for (int j = issued > NS ? issued - NS : 0; j < issued; ++j)
      if (!mbar_wait(&full[j % NS], (j / NS) & 1)) record_error(a.err, ERR_DRAIN);
  } else if (warp == 1) {
    // ---------------------------------------------------------------- converter
    // Each B row (bf16 act of one route) becomes fp16 scaled by 2^e (its max |act| in
    // [2^14, 2^15)); factor[s] = 2^-e * g2 * w_route.
    UnitCursor cu;
    cu.init(first, stride, blocks, NS);
    for (int i = 0; i < my_units; ++i, cu.next()) {
      const UnitRoutes ur = routes_of(cu.q);
      if (!mbar_wait(&full[cu.s], cu.ph)) {
        record_error(a.err, ERR_WAIT_FULL);
        break;
      }
      uint8_t* st = stages + (size_t)cu.s * L.stage_bytes;
      float* f = reinterpret_cast<float*>(st + L.foff);
      const float g2 = f[16];
      for (int sl = 0; sl < ur.n; ++sl) {
        uint8_t* row = st + L.boff + sl * bpitch;
        float m = 0.f;
        for (int k8 = lane; k8 < I / 8; k8 += 32)
          m = fmaxf(m, bf16x8_absmax(*reinterpret_cast<const uint4*>(row + stage_unit_offset<W_NVFP4>(8 * k8))));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const int ex = stage_exponent(m);
        for (int k8 = lane; k8 < I / 8; k8 += 32) {
          uint4* u = reinterpret_cast<uint4*>(row + stage_unit_offset<W_NVFP4>(8 * k8));
          *u = bf16x8_to_f16x8_scaled(*u, ex);
        }
        if (lane == 0) f[sl] = pow2f(-ex) * (g2 * f[sl]);
      }
      fence_proxy_async_smem();  // the stage is rewritten by bulk copies later
      __syncwarp();
      if (lane == 0) mbar_arrive(&cvt[cu.s]);
    }
  } else if (warp < 10) {
    // ---------------------------------------------------------------- consumers
    const int rtile = warp - 2;  // rows 16 rtile .. 16 rtile + 15 of the block
    const int ra = rtile * 16 + g, rb = ra + 8;
    const int offa = ra * UB + c * 16, offb = rb * UB + c * 16;
    // scale bytes (kb = 8 ch + 2 c, +1) of block rows ra / rb: the 128x4 swizzled block
    // (row m at (kb / 4) * 512 + (m % 32) * 16 + (m / 32) * 4 + kb % 4) or linear rows
    auto soff_of = [&](int m) {
      if (!a.swizzled) return L.soff + m * KP + c * 2;
      return L.soff + (c >> 1) * 512 + (m & 31) * 16 + (m >> 5) * 4 + (c & 1) * 2;
    };
    const int soffa = soff_of(ra), soffb = soff_of(rb);
    const int sstep = a.swizzled ? 1024 : 8;  // per 64-byte chunk
    UnitCursor cu;
    cu.init(first, stride, blocks, NS);
    for (int i = 0; i < my_units; ++i, cu.next()) {
      const UnitRoutes ur = routes_of(cu.q);
      if (!mbar_wait(&cvt[cu.s], cu.ph)) {
        record_error(a.err, ERR_WAIT_FULL);
        break;
      }
      const uint8_t* st = stages + (size_t)cu.s * L.stage_bytes;
      const uint8_t* bst = st + L.boff;
      constexpr int NC = NT == 1 ? 4 : 2;
      float acc[NC][NT][4];
#pragma unroll
      for (int h = 0; h < NC; ++h)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int r = 0; r < 4; ++r) acc[h][nt][r] = 0.f;
#pragma unroll
      for (int ch = 0; ch < CPW; ++ch) {
        const uint4 va = lds128(st + offa + ch * 64);
        const uint4 vb = lds128(st + offb + ch * 64);
        const uint32_t sa = *reinterpret_cast<const unsigned short*>(st + soffa + ch * sstep);
        const uint32_t sb = *reinterpret_cast<const unsigned short*>(st + soffb + ch * sstep);
        uint4 xf[NT][Q];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int sl = nt * 8 + g;
#pragma unroll
          for (int q = 0; q < Q; ++q)
            xf[nt][q] = sl < ur.n ? lds128(bst + (size_t)sl * bpitch + ((ch * Q + q) * 4 + c) * 16)
                                  : make_uint4(0u, 0u, 0u, 0u);
        }
        chunk_mma<W_NVFP4, NT>(acc[(2 * ch) % NC], acc[(2 * ch + 1) % NC], va, vb, sa, sb, xf,
                               ur.n > 8 ? 2 : 1);
      }
      // route factors of this lane's columns, read before the stage is released
      float fac[NT][2];
      int pr[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const int sl = nt * 8 + 2 * c + p;
          const bool live = sl < ur.n;
          fac[nt][p] = live ? reinterpret_cast<const float*>(st + L.foff)[sl] : 0.f;
          pr[nt][p] = live ? pair_of(rt, slot_entry(rt, ur, sl), M * R) : -1;
        }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[cu.s]);
      float* base = a.part + (size_t)cu.r * P * 128 + rtile * 16 + g;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          if (pr[nt][p] < 0) continue;
          float o[4];
#pragma unroll
          for (int r = 0; r < 4; ++r)
            o[r] = NC == 4 ? (acc[0][nt][r] + acc[1][nt][r]) + (acc[2 % NC][nt][r] + acc[3 % NC][nt][r])
                           : acc[0][nt][r] + acc[1][nt][r];
          float* dst = base + (size_t)pr[nt][p] * 128;
          st_cg_f32(dst, o[p] * fac[nt][p]);          // row ra
          st_cg_f32(dst + 8, o[2 + p] * fac[nt][p]);  // row rb
        }
    }
  }
}

// ------------------------------------------------------------------------------------
// k3: out[t, n] = sum of token t's route partials in route order, then the shared
// expert's; one rounding.  One thread per (token, 4 rows).
// ------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) moe_sum_kernel(const MoeArgs a) {
  const int M = a.M, R = a.R, H = a.H;
  const int P = M * (R + 1);
  pdl_wait();  // k2's partials
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q < M * H / 4) {
    const int t = q / (H / 4), n = (q - t * (H / 4)) * 4;
    const int blk = n >> 7, row = n & 127;
    const float* base = a.part + ((size_t)blk * P + t * (R + 1)) * 128 + row;
    const int nr = R + 1;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r0 = 0; r0 < nr; r0 += 8) {  // 8 loads in flight, then sums in route order
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int r = r0 + j;
        bool live = false;
        if (r < R) {
          const int id = __ldg(a.ids + t * R + r), loc = id - a.e_lo;
          live = id >= 0 && loc >= 0 && loc < a.E;
        } else {
          live = r == R && a.has_shared;
        }
        v[j] = live ? __ldcg(reinterpret_cast<const float4*>(base + (size_t)r * 128))
                    : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        s.x += v[j].x;
        s.y += v[j].y;
        s.z += v[j].z;
        s.w += v[j].w;
      }
    }
    if (a.out_f32) {
      float* o = reinterpret_cast<float*>(a.out) + (size_t)t * a.ldo + n;
      o[0] = s.x;
      o[1] = s.y;
      o[2] = s.z;
      o[3] = s.w;
    } else {
      __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(a.out) + (size_t)t * a.ldo + n;
      o[0] = __float2bfloat16_rn(s.x);
      o[1] = __float2bfloat16_rn(s.y);
      o[2] = __float2bfloat16_rn(s.z);
      o[3] = __float2bfloat16_rn(s.w);
    }
  }
  pdl_trigger();
}

namespace {

using MoeKernel = void (*)(const MoeArgs);

MoeKernel moe_up_ptr(int nt, int cpw) {
  if (nt == 1) return cpw == 1 ? moe_up_kernel<1, 1> : cpw == 2 ? moe_up_kernel<1, 2> : cpw == 4 ? moe_up_kernel<1, 4> : nullptr;
  if (nt == 2) return cpw == 1 ? moe_up_kernel<2, 1> : cpw == 2 ? moe_up_kernel<2, 2> : cpw == 4 ? moe_up_kernel<2, 4> : nullptr;
  return nullptr;
}

MoeKernel moe_down_ptr(int nt, int cpw) {
#define FNX_DOWN(NT_)                                                                   \
  switch (cpw) {                                                                        \
    case 1: return moe_down_kernel<NT_, 1>;                                             \
    case 2: return moe_down_kernel<NT_, 2>;                                             \
    case 4: return moe_down_kernel<NT_, 4>;                                             \
    case 5: return moe_down_kernel<NT_, 5>;                                             \
    case 8: return moe_down_kernel<NT_, 8>;                                             \
    default: return nullptr;                                                            \
  }
  if (nt == 1) { FNX_DOWN(1) }
  if (nt == 2) { FNX_DOWN(2) }
#undef FNX_DOWN
  return nullptr;
}

int occupancy_of(MoeKernel k, int threads, size_t smem) {
  if (!k || !prepare_kernel((const void*)k)) return 0;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, threads, smem) != cudaSuccess) return 0;
  return n;
}

}  // namespace

int moe_up_occupancy(int nt, int cpw, int threads, size_t smem) {
  return occupancy_of(moe_up_ptr(nt, cpw), threads, smem);
}
int moe_down_occupancy(int nt, int cpw, int threads, size_t smem) {
  return occupancy_of(moe_down_ptr(nt, cpw), threads, smem);
}

int launch_moe_up(const MoeArgs& a, int nt, int grid, size_t smem, cudaStream_t stream) {
  MoeKernel k = moe_up_ptr(nt, a.CPW);
  if (!k) return 1;
  if (!prepare_kernel((const void*)k)) return 2;
  return launch_with_pdl((const void*)k, a, grid, (a.W + 1 + a.EW) * 32, smem, a.pdl, stream);
}

int launch_moe_down(const MoeArgs& a, int nt, int grid, size_t smem, cudaStream_t stream) {
  MoeKernel k = moe_down_ptr(nt, a.CPW);
  if (!k) return 1;
  if (!prepare_kernel((const void*)k)) return 2;
  return launch_with_pdl((const void*)k, a, grid, 10 * 32, smem, a.pdl, stream);
}

int launch_moe_sum(const MoeArgs& a, cudaStream_t stream) {
  const int n = a.M * a.H / 4;
  return launch_with_pdl((const void*)moe_sum_kernel, a, (n + 255) / 256, 256, 0, 1, stream);
}

}  // namespace fnx
