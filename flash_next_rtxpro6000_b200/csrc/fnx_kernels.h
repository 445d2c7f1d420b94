// Internal launch interface between the C ABI (fnx_api.cu) and the kernels.
// Argument blocks are plain structs of device pointers and sizes.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "fnx_common.cuh"

namespace fnx {

// The greedy top-1 draft chain step applied to each token's argmax row (the finalize of
// draft_topk1_postprocess, patches/sglang/series/0016-…patch:46-73): the row is mapped to
// a full-vocabulary token through token_map (hot-vocabulary draft heads), written to
// topk_index and to column draft_col of draft_tokens, topk_p is set to 1 and the
// token's position advanced.  Every pointer may be null (that part is skipped).
struct DraftChain {
  const int64_t* token_map;  // [rows] int64, or null (token = row)
  int64_t* topk_index;       // [M]
  float* topk_p;             // [M]
  int64_t* draft_tokens;     // [M, draft_ld]
  int64_t draft_ld;
  int draft_col;
  int64_t* positions;        // [M], incremented
};

// Not inlined: it sits on the argmax path of every dense GEMV instance, where its code
// would otherwise grow the kernels for a step only the draft head uses.  Arguments by
// value (taking the address of a kernel's parameter block would copy it to the stack).
static __device__ __noinline__ void draft_chain_store_v(const int64_t* token_map,
                                                        int64_t* topk_index, float* topk_p,
                                                        int64_t* draft_tokens, int64_t draft_ld,
                                                        int draft_col, int64_t* positions, int m,
                                                        int64_t row) {
  const int64_t tok = token_map ? token_map[row] : row;
  if (topk_index) topk_index[m] = tok;
  if (topk_p) topk_p[m] = 1.f;
  if (draft_tokens) draft_tokens[(size_t)m * draft_ld + draft_col] = tok;
  if (positions) positions[m] += 1;
}

__device__ __forceinline__ void draft_chain_store(const DraftChain& c, int m, int64_t row) {
  draft_chain_store_v(c.token_map, c.topk_index, c.topk_p, c.draft_tokens, c.draft_ld,
                      c.draft_col, c.positions, m, row);
}

// Peer exchange of argmax keys for vocab-sharded heads (one process per GPU): every rank
// holds one buffer (FNX_PEER_BUFFER_BYTES, zeroed at allocation) laid out as
//   [0, 2048)     keys [2 (epoch parity)][8 ranks][16 tokens] u64, written by the ranks
//   [2048, 2560)  flags [8 ranks][16 tokens] u32: the last epoch rank r published token m
//   [2560, 2564)  epoch u32: this rank's call counter
//   [2624, ...)   PeerDesc: every rank's buffer as mapped in this process, world, rank
constexpr int kPeerFlagsOff = 2048, kPeerEpochOff = 2560, kPeerDescOff = 2624;
struct PeerDesc {
  unsigned char* buf[8];
  int world, rank;
  unsigned long long wait_ns;  // limit of the wait for the other ranks (0: kWaitLimitNs)
};

// The exchange step, done by one warp of the last CTA: lane m < M holds this rank's key of
// token m and returns the maximum over all ranks (the global greedy key).  Lane m writes
// its key into every rank's buffer (slot of this call's epoch parity), fences at system
// scope once and writes the epoch into every rank's flag of (this rank, token m) (a
// release pattern: the fence orders its key stores before the flags); it then polls its
// own buffer's flags of token m with acquire loads until every rank has published this
// epoch or the next one, and reads the keys.  No cross-lane ordering is needed: each lane
// pairs its own stores and loads.  In step, a rank can run at most one call ahead of
// another (it needs the other's flags to finish a call), so two key slots suffice.
// Failures keep this rank's own key and record an error code:
//  * ERR_WAIT_PEER: a rank did not publish within the wait limit (2 s by default);
//  * ERR_PEER_DESYNC: a rank is two or more calls ahead (the ranks' call sequences
//    diverged, e.g. after an expired wait), so its key slot may hold a later call's key.
static __device__ __noinline__ unsigned long long peer_key_max(unsigned char* pbuf,
                                                               unsigned long long key, int M,
                                                               int* err) {
  const int lane = threadIdx.x & 31;
  const PeerDesc* d = reinterpret_cast<const PeerDesc*>(pbuf + kPeerDescOff);
  const int world = d->world, rank = d->rank;
  const unsigned long long limit = d->wait_ns ? d->wait_ns : kWaitLimitNs;
  unsigned* epoch_p = reinterpret_cast<unsigned*>(pbuf + kPeerEpochOff);
  const unsigned e = *epoch_p + 1u;
  const int par = e & 1u;
  unsigned long long best = key;
  bool ok = true, desync = false;
  if (lane < M) {
    for (int r = 0; r < world; ++r) {
      unsigned long long* dst =
          reinterpret_cast<unsigned long long*>(d->buf[r]) + (par * 8 + rank) * 16 + lane;
      asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(dst), "l"(key) : "memory");
    }
    // one system-scope fence, then plain (relaxed) flag stores: a release pattern that
    // orders this lane's key stores before every flag at the cost of a single fence
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    for (int r = 0; r < world; ++r) {
      unsigned* f = reinterpret_cast<unsigned*>(d->buf[r] + kPeerFlagsOff) + rank * 16 + lane;
      asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(f), "r"(e) : "memory");
    }
    const unsigned long long t0 = global_ns();
    for (int r = 0; r < world && ok; ++r) {
      if (r == rank) continue;
      const unsigned* f = reinterpret_cast<const unsigned*>(pbuf + kPeerFlagsOff) + r * 16 + lane;
      for (;;) {
        unsigned v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
        const int ahead = (int)(v - e);
        if (ahead >= 2) {
          ok = false;
          desync = true;
          break;
        }
        if (ahead >= 0) break;
        if (global_ns() - t0 > limit) {
          ok = false;
          break;
        }
        __nanosleep(32);
      }
      if (ok) {
        unsigned long long k;
        const unsigned long long* src =
            reinterpret_cast<const unsigned long long*>(pbuf) + (par * 8 + r) * 16 + lane;
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(k) : "l"(src) : "memory");
        best = k > best ? k : best;
      }
    }
    if (!ok) best = key;
  }
  const bool any_desync = __any_sync(0xffffffffu, desync);
  if (!__all_sync(0xffffffffu, ok) && lane == 0)
    record_error(err, any_desync ? ERR_PEER_DESYNC : ERR_WAIT_PEER);
  if (lane == 0) *epoch_p = e;
  return best;
}

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
  float* ws;              // split-K partials [tile_groups * ksplit * RT * 256]
  unsigned int* ws_cnt;   // split-K counters [tile_groups] (zero between calls)
  int* err;               // device error flag (first error code wins), or null
  int M, N, K;            // N = output columns (fused SiLU: H, weight rows 2H)
  int ksplit;             // k splits of a tile group (separate work units)
  int silu;
  int W;                  // consumer warps per CTA
  int RT;                 // 16-row tiles per work unit
  int NS;                 // shared-memory stages in the weight ring
  int RS;                 // reduction slots between consumers and the epilogue warp
  int UB;                 // weight bytes per row per unit
  int TILE;               // shared-memory bytes of one 16-row tile (tile_bytes(UB))
  int E;                  // epilogue warps (units alternate between them)
  int nch_u;              // 64-byte chunks per row per unit
  int row_tiles;          // 16-row (SiLU: 8-output) tiles
  int tile_groups;        // ceil(row_tiles / RT)
  int n_units;            // tile_groups * ksplit
  int pdl;
  int xslice;             // 1: gridDim.x % ksplit == 0, so each CTA stages (and sizes)
                          // only its k split of the activations
  DraftChain chain;       // greedy draft-chain step on the argmax (all null: off)
  unsigned char* peerbuf; // this rank's peer-exchange buffer (vocab shards), or null
  NormGate norm;          // gated RMSNorm on the activation load (norm.G > 0), else off;
                          // with xslice the unit k extent is a multiple of norm.G
};

// One stage of the dense weight ring: RT tiles of weights, then the unit's row scales
// (RT * 16 values, raw bf16 or fp32), then (NVFP4) the unit's e4m3 block scales,
// RT * 16 rows of sbr bytes.
struct DenseStage {
  int rsoff, bsoff, sbr, bytes;
};

__host__ __device__ inline int dense_align(int v, int a) { return (v + a - 1) / a * a; }

__host__ __device__ inline DenseStage dense_stage(int nvfp4, int RT, int tile, int nch_u) {
  DenseStage d;
  d.rsoff = RT * tile;
  d.bsoff = d.rsoff + RT * 64;
  d.sbr = dense_align(nch_u * 8, 16);
  d.bytes = dense_align(d.bsoff + (nvfp4 ? RT * 16 * d.sbr : 0), 128);
  return d;
}

// Shared-memory layout of the dense kernel (host and device use the same function).
struct DenseLayout {
  int bars, stages, xs, unscale, red, sred, total;
};

__host__ __device__ inline DenseLayout dense_layout(int M, int K, int W, int NS, int RS, int NT,
                                                    int stage_bytes) {
  DenseLayout L;
  int off = 0;
  L.bars = off;
  off = dense_align(off + (2 * NS + 2 * RS + 1) * 8, 128);  // + the activation barrier
  L.stages = off;
  off += NS * stage_bytes;
  L.xs = dense_align(off, 128);
  off = L.xs + M * (2 * K + 64);
  L.unscale = dense_align(off, 16);
  off = L.unscale + 32 * 4;  // 16 unscale factors + 16 row maxima (stage_rows)
  L.red = dense_align(off, 16);
  off = L.red + RS * W * 32 * NT * 16;
  L.sred = off;                       // per slot: 64 floats of row scales (RT x 16)
  off += RS * 64 * 4;
  L.total = dense_align(off, 128);
  return L;
}

// Block sizes the kernels are compiled for (registers per thread = 65536 / threads):
// the MoE kernels run at most 14 (k1) and exactly 10 (k2) warps, so they may keep more
// of each chunk's operands in flight than a 20-warp bound would allow.
constexpr int kMoeUpThreads = 14 * 32;
constexpr int kMoeDownThreads = 10 * 32;
constexpr int kDenseThreadsMax = 20 * 32;  // producer + up to 3 epilogue + 16 consumer warps

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
  // [e_lo, e_lo + E) are skipped; weight tensors hold the local experts only.
  int e_lo;
  // scratch (caller-owned; counters zero between calls)
  uint8_t* act;           // [dcap * 16] rows of 2I + 64 B: the SiLU-mul activations in bf16,
                          //   row d * 16 + s = route slot s of distinct expert d, in the
                          //   B-operand order of the down kernel (k1 -> k2)
  float* part;            // fp32 [H / 128][M * (R + 1)][128]  k2 route partials
  int* err;
  // output: bf16 [M, H] (or fp32 partial sums when out_f32, for cross-rank reduction)
  void* out;
  int64_t ldo;
  int out_f32;
  // launch geometry (EW: k1 epilogue warps)
  int W, CPW, NS, RS, NT, EW;
  int pdl;
  // fused single-launch form (moe_fused.cu): counters [vcap + H / 64 + 1] (zero between
  // calls, left at zero), the virtual-expert capacity and the consumer groups
  unsigned* cnt;
  int vcap, NG;
};

// Shared-memory layout of the MoE kernels.  A stage holds the unit's weight tiles, its
// e4m3 block scales (row-major, spitch bytes per row), for k2 the B rows of its routes
// (bpitch bytes each), and a small float area: k1 the expert's global scale; k2 the
// route weights [0, 16) and the global scale [16], replaced by the route factors.
struct MoeLayout {
  int bars, stages, xs, unscale, red, sred, ids, bitmap, wbase, exp_of, cnt_of, ent, misc;
  int ctab, rrank, rdist, etok, epair, total;
  int stage_bytes, wpitch, soff, spitch, boff, bpitch, foff;
};

constexpr int kMoeSlotCap = 16;  // routes of one distinct expert handled by one unit

__host__ __device__ inline MoeLayout moe_layout(int kernel /*1 = up, 2 = down*/, int M, int R,
                                                int E, int H, int I, int W, int NS, int RS,
                                                int NT, int RT) {
  MoeLayout L;
  const int nw = (E + 31) / 32;
  const int dcap = (E < M * R ? E : M * R) + 1;
  const int K = kernel == 1 ? H : I;
  L.bpitch = 2 * I + 64;
  if (kernel == 1) {  // one 16-row tile (two 8-row halves), scales of 16 rows
    L.wpitch = tile_bytes(K / 2);
    L.spitch = dense_align(K / 16, 16);  // linear scales: one padded row per weight row
    L.soff = L.wpitch;
    L.boff = dense_align(L.soff + 16 * L.spitch, 128);  // >= swizzled 16 * K/16
  } else {            // 128 contiguous rows, then the 128 rows' scales as one block
    L.wpitch = 16 * (K / 2);
    L.spitch = K / 16;
    L.soff = 8 * L.wpitch;
    L.boff = dense_align(L.soff + 128 * L.spitch, 128);
  }
  L.foff = L.boff + (kernel == 2 ? 8 * NT * L.bpitch : 0);
  L.stage_bytes = dense_align(L.foff + 80, 128);
  int off = 0;
  L.bars = off;
  // full, converted, empty; rfull, rfree; the activation rows' barrier
  off = dense_align(off + (3 * NS + 2 * RS + 1) * 8, 128);
  L.stages = off;
  off += NS * L.stage_bytes;
  L.xs = off;
  off += kernel == 1 ? M * (2 * H + 64) : 0;
  L.unscale = dense_align(off, 16);
  off = L.unscale + 32 * 4;  // 16 unscale factors + 16 row maxima (stage_rows)
  L.red = dense_align(off, 16);
  off = L.red + RS * W * 32 * NT * 16;
  L.sred = off;               // per slot: 64 floats handed to the epilogue
  off += RS * 64 * 4;
  L.ids = off;
  off += dense_align(M * R, 4) * 4;
  L.bitmap = off;
  off += dense_align(nw, 4) * 4;
  L.wbase = off;
  off += dense_align(nw, 4) * 4;
  L.exp_of = off;
  off += dense_align(dcap, 4) * 4;
  L.cnt_of = off;
  off += dense_align(dcap, 4) * 4;
  L.ent = off;
  off += dense_align(dcap * kMoeSlotCap * 2, 16);
  L.misc = off;
  off += 16;
  const int n = M * R;
  L.ctab = off;
  off += dense_align(((n + 31) / 32) * dcap, 16);
  L.rrank = off;
  off += dense_align(n, 16);
  L.rdist = off;
  off += dense_align(2 * n, 16);
  L.etok = off;
  off += dense_align(n, 16);
  L.epair = off;
  off += dense_align(2 * (n + M), 16);
  L.total = dense_align(off, 128);
  return L;
}

// ------------------------------------------------------------------------------------
// Fused MoE layer (moe_fused.cu): one persistent launch, one CTA per SM.
// ------------------------------------------------------------------------------------
constexpr int kFusedSlots = 8;     // route slots of one virtual expert (MMA N = 8)
constexpr int kFusedProd = 2;      // producer warps (items round robin; a bulk copy takes
                                   // ~70 cycles to issue, warps issue in parallel)
constexpr int kFusedFetch = 2;     // act fetcher warps
constexpr int kFusedEpi = 8;       // epilogue warps (each release of stores costs its warp
                                   // ~0.5-1 us, so several run side by side)
constexpr int kFusedRes = 8;       // result slots (consumers -> epilogue warps)
constexpr int kFusedBatch = 1;     // items whose stores one epilogue release covers
constexpr int kFusedAct = 2;       // act ring slots (fetchers -> consumers)
constexpr int kFusedMaxGroups = 2; // consumer groups of 4 warps
constexpr int kFusedThreads = (kFusedProd + kFusedFetch + kFusedEpi + 4 * kFusedMaxGroups) * 32;
// The rings use parity waits, which are only correct when one warp (producer side) and
// one consumer group (consumer side) see every use of a slot in order, so that a slot's
// barrier is never more than one phase behind the waiter.  Items go round robin to the
// producer warps and to the consumer groups, so the stage count must be a multiple of
// both: kFusedRing.  (Stage counts that broke this let a wait pass a phase early: a stage
// was refilled while it was being read, and the exit drain could miss a copy in flight.)
constexpr int kFusedRing = kFusedProd * kFusedMaxGroups /
                           (kFusedProd % kFusedMaxGroups == 0   ? kFusedMaxGroups
                            : kFusedMaxGroups % kFusedProd == 0 ? kFusedProd
                                                                : 1);
static_assert(kFusedRing % kFusedProd == 0 && kFusedRing % kFusedMaxGroups == 0,
              "kFusedRing must be a common multiple of producers and consumer groups");
static_assert(kFusedRes % kFusedEpi == 0 && kFusedRes % kFusedMaxGroups == 0,
              "each result slot must belong to one epilogue warp and one consumer group");
static_assert(kFusedAct % kFusedFetch == 0 && kFusedAct % kFusedMaxGroups == 0,
              "each act slot must belong to one fetcher warp and one consumer group");

// Capacity of the virtual-expert table for n = M * R routes over E experts: every
// virtual expert holds 1..8 routes of one expert, so there are at most
// min(E, n) + n / 8 of them, and never more than n; plus two shared-expert halves.
__host__ __device__ inline int fused_vcap(int M, int R, int E) {
  const int n = M * R;
  const int d = E < n ? E : n;
  const int v = d + n / 8;
  return (v < n ? v : n) + 2;
}

// Shared-memory layout of the fused kernel (identical on host and device).  A ring stage
// holds one work item: a gate/up tile (16 weight rows over H: the up and gate rows of 8
// columns of I; their block scales; the expert's global scale) or a down half-block
// (64 weight rows over I as four 16-row tiles; the 128-row block's scales).  An act slot
// holds the 8 route rows of one virtual expert as scaled fp16, each followed by its
// factor; a result slot holds the four consumer warps' C fragments of one item.
struct FusedLayout {
  int ub1, tb1, soff1, foff1;   // gate/up tile: row bytes, tile bytes, scale / scalar offsets
  int ub2, tb2, soff2;          // down half-block
  int stage_bytes, act_bytes, res_bytes;
  int bars, stages, xs, act, res, unscale;
  int lid, bitmap, wbase, exp_of, cnt_of, vbase, ctab, rrank, rdist, etok, vexp, vnum, vent,
      misc, lastk, total;
};

__host__ __device__ inline FusedLayout fused_layout(int M, int R, int E, int H, int I, int NS,
                                                    int vcap) {
  FusedLayout L;
  L.ub1 = H / 2;
  L.tb1 = tile_bytes(L.ub1);
  L.soff1 = L.tb1;
  const int sc1 = 16 * dense_align(H / 16, 16);  // >= the swizzled 2 x 2 x (H / 64) x 16 B
  L.foff1 = L.soff1 + sc1;
  L.ub2 = I / 2;
  L.tb2 = tile_bytes(L.ub2);
  L.soff2 = 4 * L.tb2;
  const int sc2 = 128 * (I / 16);                // the whole 128-row block (swizzled)
  const int e1 = L.foff1 + 16, e2 = L.soff2 + sc2;
  L.stage_bytes = dense_align(e1 > e2 ? e1 : e2, 128);
  L.act_bytes = kFusedSlots * stage_row_bytes(I);  // factor of row s at s * row + 2I
  L.res_bytes = 4 * 32 * 16 + 16;                  // + the expert's global scale (tiles)
  const int n = M * R;
  const int nw = (E + 31) / 32;
  const int dcap = E < n ? E : n;
  const int nchunk = (n + 31) / 32;
  int off = 0;
  L.bars = off;  // full, empty [NS]; xbar; afull, aempty [kFusedAct]; rfull, rfree [kFusedRes]
  off = dense_align(off + (2 * NS + 1 + 2 * kFusedAct + 2 * kFusedRes) * 8, 128);
  L.stages = off;
  off += NS * L.stage_bytes;
  L.xs = off;
  off += M * stage_row_bytes(H);
  L.act = dense_align(off, 128);
  off = L.act + kFusedAct * L.act_bytes;
  L.res = dense_align(off, 16);
  off = L.res + kFusedRes * L.res_bytes;
  L.unscale = dense_align(off, 16);
  off = L.unscale + 32 * 4;
  L.lid = off;
  off += dense_align(2 * n, 16);
  L.bitmap = off;
  off += dense_align(4 * nw, 16);
  L.wbase = off;
  off += dense_align(4 * nw, 16);
  L.exp_of = off;
  off += dense_align(2 * dcap, 16);
  L.cnt_of = off;
  off += dense_align(2 * dcap, 16);
  L.vbase = off;
  off += dense_align(2 * dcap, 16);
  L.ctab = off;
  off += dense_align(nchunk * dcap, 16);
  L.rrank = off;
  off += dense_align(n, 16);
  L.rdist = off;
  off += dense_align(2 * n, 16);
  L.etok = off;
  off += dense_align(n, 16);
  L.vexp = off;
  off += dense_align(2 * vcap, 16);
  L.vnum = off;
  off += dense_align(vcap, 16);
  L.vent = off;
  off += dense_align(2 * kFusedSlots * vcap, 16);
  L.misc = off;
  off += 16;
  L.lastk = off;  // [NS] last item issued into each ring stage
  off += dense_align(4 * NS, 16);
  L.total = dense_align(off, 128);
  return L;
}

// MoE router: x . W^T (+ bias) into fp32 logits, then (topk > 0) the softmax top-k of
// every row, run by the CTA that finishes last (router.cu).
struct RouterArgs {
  const __nv_bfloat16* x;  // [M, K], row stride ldx elements, rows 16-byte aligned
  int64_t ldx;
  const __nv_bfloat16* w;  // [N, K] router weight, row stride ldw elements
  int64_t ldw;
  const __nv_bfloat16* bias;  // [N] or null
  float* logits;           // [M, ldl] fp32
  int64_t ldl;
  float* out_w;            // [M, ldk] routing weights (topk > 0)
  int32_t* out_ids;        // [M, ldk] expert ids
  int64_t ldk;
  unsigned* counter;       // CTA arrival counter, zero between calls (topk > 0)
  int M, N, K, topk, renorm, pdl;
};

// Softmax top-k of given logits (bf16 or fp32 [M, lds]) plus an optional fp32 bias.
struct TopkArgs {
  const void* scores;
  int64_t lds;
  int scores_f32;
  const float* bias;
  float* out_w;
  int32_t* out_ids;
  int64_t ldk;
  int M, N, topk, renorm, pdl;
};

int launch_router(const RouterArgs& a, cudaStream_t stream);

// Greedy top-1 of given logits rows (fp32 or bf16 [M, ldl], V columns) with the draft
// chain step (topk1.cu): split over CTAs, keys combined with atomicMax, the last CTA
// applies the chain and leaves keys and counter at zero.
struct Top1Args {
  const void* logits;
  int64_t ldl;
  int logits_f32;
  int M, V, splits, pdl;
  unsigned long long* keys;  // [M], zero between calls
  unsigned* count;           // zero between calls
  DraftChain chain;
};

int launch_top1(const Top1Args& a, cudaStream_t stream);
int launch_softmax_topk(const TopkArgs& a, cudaStream_t stream);

// Compiled forms of the dense kernel: whole activation rows staged; each CTA staging
// only its k split (xslice); the fused gated RMSNorm (xslice or not, at run time).
enum DenseMode : int { DENSE_PLAIN = 0, DENSE_SLICE = 1, DENSE_NORM = 2 };

inline int dense_mode(const DenseArgs& a) {
  return a.norm.G > 0 ? DENSE_NORM : (a.xslice ? DENSE_SLICE : DENSE_PLAIN);
}

int launch_dense(const DenseArgs& a, int wtype, int nt, int cpw, int grid, size_t smem,
                 cudaStream_t stream);
int launch_moe_up(const MoeArgs& a, int nt, int grid, size_t smem, cudaStream_t stream);
int launch_moe_down(const MoeArgs& a, int nt, int grid, size_t smem, cudaStream_t stream);
int launch_moe_sum(const MoeArgs& a, cudaStream_t stream);
// The fused layer for the (H, I) tilings it is compiled for: 1 = no instance.
int launch_moe_fused(const MoeArgs& a, int grid, size_t smem, cudaStream_t stream);
// Decode-width MoE layer in one launch (moe_lean.cu): M = 1, swizzled scales, H and I
// multiples of 256 (H <= 2048, I <= 512).  moe_lean_plan picks the ring depth and shared memory for a
// grid of `grid` CTAs (all resident, one per SM); the launch needs moe_lean_counters(M, R,
// E) zeroed counters in a.cnt and (min(E, M R) + 1) M I bf16 act values in a.act, and
// returns 3 when the weights' tensor maps cannot be encoded.
bool moe_lean_plan(int M, int R, int E, int H, int I, int grid, int& NS, size_t& smem);
int64_t moe_lean_counters(int M, int R, int E);
int launch_moe_lean(const MoeArgs& a, int NS, int grid, size_t smem, cudaStream_t stream);
bool moe_fused_has(int H, int I);
int launch_argmax_decode(const unsigned long long* keys, int64_t* out, int M,
                         cudaStream_t stream);

// NVFP4 load-time codec (nvfp4_codec.cu).  scratch: one u32 (cleared here).
int launch_nvfp4_quantize(const void* w, int64_t ldw, int w_f32, int N, int K, uint8_t* wq,
                          int64_t ldwq, uint8_t* bs, int64_t ldbs, float* gscale,
                          unsigned* scratch, cudaStream_t stream);
int launch_nvfp4_dequantize(const uint8_t* wq, int64_t ldwq, const uint8_t* bs, int64_t ldbs,
                            const float* gscale, int per_row, void* out, int64_t ldo, int out_f32,
                            int N, int K, cudaStream_t stream);

int dense_occupancy(int wtype, int nt, int cpw, int mode, int threads, size_t smem);
int moe_up_occupancy(int nt, int cpw, int threads, size_t smem);
int moe_down_occupancy(int nt, int cpw, int threads, size_t smem);

// Tensor-core (tcgen05) dense GEMV (dense_tc.cu): int8 / fp8 weights, K a multiple of
// 128, plain mode.  dense_tc_plan picks the ring depth and shared memory (false: not
// available for this weight type / K); the launch needs dense_tc_partial_floats(grid)
// partial floats and dense_tc_counters(grid) zeroed counters.
bool dense_tc_plan(int wt, int K, int& NS, size_t& smem);
int dense_tc_grid(int N, int K);
int64_t dense_tc_partial_floats(int grid);
int64_t dense_tc_counters(int grid);
int launch_dense_tc(const DenseArgs& d, int wt, int grid, size_t smem, float* part, unsigned* pcnt,
                    cudaStream_t stream);

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
