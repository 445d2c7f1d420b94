// C ABI of the GEMV library (include/fnx_gemv.h): argument validation mirroring the
// reference's Python wrappers, the launch planner, and the kernel launches.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstddef>
#include <cstring>
#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/fnx_gemv.h"
#include "fnx_common.cuh"
#include "fnx_kernels.h"

#include <mutex>
#include <set>
#include <utility>

namespace fnx {

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

bool prepare_kernel(const void* func) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({func, dev})) return true;
  int optin = 0;
  if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
    return false;
  if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, optin) !=
      cudaSuccess)
    return false;
  done.insert({func, dev});
  return true;
}

}  // namespace fnx

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_fail(const char* what) {
  const cudaError_t e = cudaGetLastError();
  return fail(FNX_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int chunk_k(int wt) {
  switch (wt) {
    case FNX_W_BF16: return 32;
    case FNX_W_NVFP4: return 128;
    default: return 64;
  }
}

constexpr size_t kMaxSmem = 227 * 1024;

// Dense GEMV form (fnx_set_dense_path): by default the tensor-core form serves M > kTcMinM.
// Measured on the int8 lm_head (151,936 x 2,048) on B200: M = 9 / 16 tcgen05 70.2 / 74.0 us
// against mma.sync 77.6 / 79.7 us; M = 1 / 8 mma.sync 51.8 / 57.0 us against 66.3 / 69.7.
std::atomic<int> g_dense_path{FNX_DENSE_PATH_AUTO};
// MoE layer form (fnx_set_moe_path): by default the decode-width kernel serves M <= 8.
std::atomic<int> g_moe_path{FNX_MOE_PATH_AUTO};
constexpr int kTcMinM = 8;

// Geometry of one dense call.  A work unit is RT 16-row tiles x (K / ksplit); each of
// the W consumer warps streams CPW 64-byte chunks of every row of one tile; the weight
// ring has NS stages of RT tiles of TILE bytes (two 8-row halves, see tile_half_offset).
struct DensePlan {
  int ksplit, W, RT, CPW, NS, E, UB, TILE, nch_u, row_tiles, tile_groups, n_units, wt;
  int xslice;  // each CTA stages only its k split (needs a grid that is a multiple of ksplit)
  size_t smem;
};

bool layout_fits(int M, int K, int NT, DensePlan& p);

// Fill in the derived fields and the ring depth; false when two stages do not fit.
bool layout_plan(int M, int K, int NT, DensePlan& p) {
  // three epilogue warps where the threads and shared memory allow (the epilogue shares
  // the issue slots with up to 16 consumer warps), else two
  for (int e = 3; e >= 2; --e) {
    p.E = e;
    if (p.W + 1 + e > 20) continue;
    if (layout_fits(M, K, NT, p)) return true;
  }
  return false;
}

bool layout_fits(int M, int K, int NT, DensePlan& p) {
  p.UB = p.nch_u * 64;
  p.TILE = fnx::tile_bytes(p.UB);
  p.tile_groups = (p.row_tiles + p.RT - 1) / p.RT;
  p.n_units = p.tile_groups * p.ksplit;
  const int stage = fnx::dense_stage(p.wt == FNX_W_NVFP4, p.RT, p.TILE, p.nch_u).bytes;
  const int kx = p.xslice ? p.nch_u * chunk_k(p.wt) : K;  // staged activation columns
  const fnx::DenseLayout L0 = fnx::dense_layout(M, kx, p.W, 0, p.E, NT, stage);
  if ((size_t)L0.total + 2 * (size_t)stage + 256 > kMaxSmem) return false;
  const int ns = (int)((kMaxSmem - L0.total - 256) / stage);
  p.NS = std::max(2, std::min(ns, 8));
  p.smem = fnx::dense_layout(M, kx, p.W, p.NS, p.E, NT, stage).total;
  return true;
}

int finish_plan(int M, int K, int NT, DensePlan& p) {
  if (!layout_plan(M, K, NT, p))
    return fail(FNX_EUNSUPPORTED, "shared memory: M=%d K=%d leaves no room for 2 stages", M, K);
  return FNX_OK;
}

int plan_dense(int M, int N, int K, int wt, int silu, const fnx_gemv_cfg* req, DensePlan& p) {
  const int CH = chunk_k(wt);
  if (K <= 0 || K % CH)
    return fail(FNX_EUNSUPPORTED, "K=%d must be a positive multiple of %d for this weight type",
                K, CH);
  const int nch = K / CH;
  const int NT = M > 8 ? 2 : 1;
  p.wt = wt;
  p.row_tiles = silu ? (N + 7) / 8 : (N + 15) / 16;
  if (req) {
    p.ksplit = req->ksplit;
    p.W = req->warps;
    p.CPW = req->chunks_per_warp;
    p.RT = std::max(1, req->groups);
    if (p.ksplit < 1 || nch % p.ksplit)
      return fail(FNX_EINVAL, "ksplit=%d must divide K/%d = %d", p.ksplit, CH, nch);
    p.nch_u = nch / p.ksplit;
    p.xslice = p.ksplit > 1 ? 1 : 0;  // run_dense drops it where the grid does not allow it
    if (p.W < 1 || p.W > 16 || p.RT > 4 || p.W % p.RT ||
        (p.CPW != 1 && p.CPW != 2 && p.CPW != 4 && p.CPW != 8) || (p.W / p.RT) * p.CPW != p.nch_u)
      return fail(FNX_EINVAL,
                  "need warps <= 16, row tiles <= 4 dividing warps, chunks_per_warp in {1,2,4,8} "
                  "and (warps / row_tiles) * chunks_per_warp == %d chunks per unit", p.nch_u);
    return finish_plan(M, K, NT, p);
  }
  const int sms = fnx::num_sms();
  // Mid-size problems (fewer than 8 row tiles per SM) are latency-bound.  Measured on
  // B200 over 1024..16384 rows x 2048..8192 columns (int8, fp8, NVFP4; M = 1, 4, 16),
  // the best tilings take one row tile per unit, the fewest k splits that keep a unit
  // within nu_max chunks (the staged activations and a deep ring must fit; a split-K
  // fix-up costs more than a longer unit), and about 8 consumer warps at M = 1, 16 above.
  if ((int64_t)p.row_tiles < 8LL * sms) {
    const int nu_max = M <= 1 ? 96 : (M <= 8 ? 64 : 32);
    const int wt = M <= 1 ? 8 : 16;
    for (int k = 1; k <= nch && k <= sms; ++k) {
      if (nch % k || nch / k > nu_max) continue;
      const int nu = nch / k;
      int cpw = 1;
      while (cpw < 8 && nu % (2 * cpw) == 0 && nu / cpw > wt) cpw *= 2;
      if (nu / cpw > 16) continue;
      DensePlan q = p;
      q.ksplit = k;
      q.nch_u = nu;
      q.W = nu / cpw;
      q.CPW = cpw;
      q.RT = 1;
      q.xslice = k > 1 ? 1 : 0;
      if (layout_plan(M, K, NT, q)) {
        p = q;
        return FNX_OK;
      }
    }
  }
  // Large problems at M > 8 (two 8-token column blocks per tile): one row tile per unit
  // and 8 consumer warps, which leaves shared memory for a deeper weight ring.  Measured
  // on the int8 lm_head (151,936 x 2,048) at M = 16: 8 warps x 4 chunks x 1 tile 78.6 us,
  // 16 x 4 x 2 (the cost model's pick) 92.6 us; at M <= 8 the cost model's pick is best.
  if (NT == 2 && nch % 8 == 0 && nch / 8 <= 8 && ((nch / 8) & (nch / 8 - 1)) == 0) {
    DensePlan q = p;
    q.ksplit = 1;
    q.nch_u = nch;
    q.W = 8;
    q.CPW = nch / 8;
    q.RT = 1;
    q.xslice = 0;
    if (layout_plan(M, K, NT, q)) {
      p = q;
      return FNX_OK;
    }
  }
  // Search (k split, row tiles per unit RT, chunks per consumer warp CPW) with a cost
  // model of one CTA's time: rounds of units x the unit's chunk rows, plus a per-unit
  // overhead of each consumer warp (about 1.5 chunks) and of the split-K fix-up; fewer
  // than 12 consumer warps hide latency less well.  Measured on lm_head (151936 x 2048
  // int8, M = 1): 16 warps x 4 chunks x 2 tiles runs at 96 % of the copy bandwidth,
  // 16 x 2 x 1 at 80 %.
  double best_cost = 1e30;
  DensePlan best = p;
  bool found = false;
  for (int k = 1; k <= nch && k <= sms; ++k) {  // k <= sms: the grid rounds to a multiple
    if (nch % k) continue;
    const int nu = nch / k;
    for (int rt : {1, 2, 4}) {
      for (int cpw : {1, 2, 4, 8}) {
        if (nu % cpw) continue;
        const int ksl = nu / cpw, w = rt * ksl;
        if (w > 16) continue;
        DensePlan q = p;
        q.ksplit = k;
        q.nch_u = nu;
        q.W = w;
        q.CPW = cpw;
        q.RT = rt;
        q.xslice = k > 1 ? 1 : 0;
        if (!layout_plan(M, K, NT, q)) continue;
        // several tiles per unit only while every SM still gets two units or more:
        // small problems are latency-bound and want the most parallel units
        if (rt > 1 && (int64_t)q.tile_groups * k < 2LL * sms) continue;
        const int64_t units = q.n_units;
        const int64_t grid = std::min<int64_t>(units, sms);
        const int64_t rounds = (units + grid - 1) / grid;
        double cost = (double)rounds * rt * (nu + 1.5 * ksl + (k > 1 ? 2.0 : 0.0));
        if (w < 12) cost *= 1.25;
        if (w < 4) cost *= 2.0;
        if (cost < best_cost - 1e-9) {
          best_cost = cost;
          best = q;
          found = true;
        }
      }
    }
  }
  if (!found) return fail(FNX_EUNSUPPORTED, "no tiling of K=%d (%d chunks) fits M=%d", K, nch, M);
  p = best;
  return FNX_OK;
}

struct DenseCall {
  const void* x;
  int64_t ldx;
  const void* w;
  int64_t ldw;
  int wt;
  const void* bs;
  int64_t ldbs;
  const void* scale;
  int scale_kind;
  void* y;
  int64_t ldy;
  void* y2;
  int64_t ldy2;
  int64_t split_n;
  int out_f32;
  int64_t* argmax_out;
  unsigned long long* argmax_key_out;
  int64_t row_offset;
  int M, N, K;
  int silu;
  const fnx_gemv_cfg* cfg;
  const fnx_workspace* ws;
  int pdl;
  cudaStream_t stream;
  fnx::NormGate norm;  // gated RMSNorm on the activation load (norm.G > 0)
  fnx::DraftChain chain;  // draft chain step on the argmax (all null: off)
  unsigned char* peerbuf = nullptr;  // peer key exchange (vocab shards)
};

int run_dense(const DenseCall& c) {
  g_err.clear();
  if (c.M < 0 || c.M > FNX_MAX_M) return fail(FNX_EINVAL, "M=%d must be in [0, 16]", c.M);
  if (c.N < 0 || c.K <= 0) return fail(FNX_EINVAL, "bad shape N=%d K=%d", c.N, c.K);
  if (c.M == 0 || c.N == 0) return FNX_OK;
  if (!c.x || !c.w || !c.y) return fail(FNX_EINVAL, "null x, w or y");
  if (!aligned(c.x, 16) || (c.ldx * 2) % 16 || c.ldx < c.K)
    return fail(FNX_EINVAL, "x rows must be 16-byte aligned with ldx >= K");
  const int64_t row_bytes = c.wt == FNX_W_NVFP4 ? c.K / 2 : (c.wt == FNX_W_BF16 ? 2LL * c.K : c.K);
  if (!aligned(c.w, 16) || c.ldw % 16 || c.ldw < row_bytes)
    return fail(FNX_EINVAL, "weight rows must be 16-byte aligned, ldw=%lld < %lld bytes or not a "
                "multiple of 16", (long long)c.ldw, (long long)row_bytes);
  if (c.wt == FNX_W_NVFP4) {
    if (!c.bs || c.ldbs < c.K / 16 || c.ldbs % 8 || !aligned(c.bs, 8))
      return fail(FNX_EINVAL, "block scales must be [N, K/16], 8-byte aligned rows");
  }
  if (c.scale_kind < FNX_SCALE_NONE || c.scale_kind > FNX_SCALE_BF16_ROW)
    return fail(FNX_EINVAL, "bad scale kind %d", c.scale_kind);
  if (c.scale_kind != FNX_SCALE_NONE && !c.scale) return fail(FNX_EINVAL, "null scale");
  if (c.silu && (c.y2 || c.argmax_out || c.argmax_key_out || c.out_f32))
    return fail(FNX_EINVAL, "the fused SiLU form has a single bf16 destination");
  if (c.y2) {
    if (!(c.split_n > 0 && c.split_n < c.N))
      return fail(FNX_EINVAL, "split_n must be in (0, %d); got %lld", c.N, (long long)c.split_n);
    if (c.ldy2 < c.N - c.split_n) return fail(FNX_EINVAL, "ldy2 too small");
    if (c.ldy < c.split_n) return fail(FNX_EINVAL, "ldy too small");
  } else if (c.ldy < c.N) {
    return fail(FNX_EINVAL, "ldy=%lld < N=%d", (long long)c.ldy, c.N);
  }
  if (c.row_offset < 0 || c.row_offset + c.N > 0xFFFFFFFFLL)
    return fail(FNX_EINVAL, "row ids must fit in 32 bits");

  const bool chain_on = c.chain.topk_index || c.chain.topk_p || c.chain.draft_tokens ||
                        c.chain.positions;
  const bool want_argmax = c.argmax_out || c.argmax_key_out || chain_on || c.peerbuf;
  if (want_argmax && (!c.ws || !c.ws->argmax_keys || !c.ws->argmax_count))
    return fail(FNX_EINVAL, "argmax needs the workspace's argmax_keys/argmax_count");

  // The tensor-core form (tcgen05, A dequantised into tensor memory) at the verify widths:
  // int8 / fp8 weights, no fused SiLU / norm / draft chain, the planner's own tiling, and
  // a workspace for the partial sums of the blocks that CTAs share.
  const int path = g_dense_path.load(std::memory_order_relaxed);
  if (path != FNX_DENSE_PATH_MMA && !c.cfg && !c.silu && c.norm.G == 0 && !chain_on &&
      (c.wt == FNX_W_INT8 || c.wt == FNX_W_FP8_E4M3) &&
      (path == FNX_DENSE_PATH_TCGEN05 || c.M > kTcMinM)) {
    int ns = 0;
    size_t smem = 0;
    const int grid = fnx::dense_tc_grid(c.N, c.K);
    if (fnx::dense_tc_plan(c.wt, c.K, ns, smem) && c.ws && c.ws->partials && c.ws->counters &&
        c.ws->partial_floats >= fnx::dense_tc_partial_floats(grid) &&
        c.ws->n_counters >= fnx::dense_tc_counters(grid)) {
      fnx::DenseArgs a = {};
      a.x = c.x;
      a.ldx = c.ldx;
      a.w = static_cast<const uint8_t*>(c.w);
      a.ldw = c.ldw;
      a.scale = c.scale;
      a.scale_kind = c.scale_kind;
      a.y = c.y;
      a.ldy = c.ldy;
      a.y2 = c.y2;
      a.ldy2 = c.ldy2;
      a.split_n = c.y2 ? c.split_n : 0;
      a.out_f32 = c.out_f32;
      a.am_keys = want_argmax ? c.ws->argmax_keys : nullptr;
      a.am_count = want_argmax ? c.ws->argmax_count : nullptr;
      a.am_out = c.argmax_out;
      a.am_key_out = c.argmax_key_out;
      a.row_offset = c.row_offset;
      a.err = c.ws->error_flag;
      a.M = c.M;
      a.N = c.N;
      a.K = c.K;
      a.NS = ns;
      a.pdl = c.pdl;
      a.peerbuf = c.peerbuf;
      const int rc = fnx::launch_dense_tc(a, c.wt, grid, smem, c.ws->partials, c.ws->counters,
                                          c.stream);
      if (rc == 0) return FNX_OK;
      if (rc == 2) return cuda_fail("tensor-core GEMV launch");
      if (path == FNX_DENSE_PATH_TCGEN05 && rc == 3)
        return fail(FNX_EUNSUPPORTED, "tensor map of the weights could not be encoded");
      // otherwise (no tensor-map encoder, no instance) the mma.sync form below
    } else if (path == FNX_DENSE_PATH_TCGEN05 && !fnx::dense_tc_plan(c.wt, c.K, ns, smem)) {
      return fail(FNX_EUNSUPPORTED, "tensor-core GEMV: K=%d does not fit", c.K);
    }
  }

  DensePlan p;
  int rc = plan_dense(c.M, c.N, c.K, c.wt, c.silu, c.cfg, p);
  if (rc) return rc;
  const int NT = c.M > 8 ? 2 : 1;
  if (p.ksplit > 1) {
    const int64_t need = (int64_t)p.tile_groups * p.ksplit * p.RT * 256;
    if (!c.ws || !c.ws->partials || !c.ws->counters)
      return fail(FNX_EINVAL, "ksplit=%d needs a workspace", p.ksplit);
    if (c.ws->partial_floats < need || c.ws->n_counters < p.tile_groups)
      return fail(FNX_EINVAL, "workspace too small: need %lld floats and %d counters",
                  (long long)need, p.tile_groups);
  }
  // xslice (each CTA stages only its k split) needs a grid that is a multiple of ksplit
  // and, with the fused norm, a unit k extent that holds whole norm groups; otherwise
  // the full rows are staged (same tiling and workspace, larger shared memory).
  const int user_grid = c.cfg && c.cfg->grid > 0 ? c.cfg->grid : 0;
  auto full_rows = [&]() -> int {
    p.xslice = 0;
    if (!layout_plan(c.M, c.K, NT, p))
      return fail(FNX_EUNSUPPORTED, "shared memory: M=%d K=%d leaves no room for 2 stages",
                  c.M, c.K);
    return FNX_OK;
  };
  if (p.xslice && ((c.norm.G > 0 && (p.nch_u * chunk_k(c.wt)) % c.norm.G) ||
                   (user_grid > 0 && user_grid % p.ksplit)))
    if (int e = full_rows()) return e;
  int grid = user_grid;
  if (grid <= 0) {
    for (int pass = 0; pass < 2; ++pass) {
      const int mode = c.norm.G > 0 ? fnx::DENSE_NORM
                                    : (p.xslice ? fnx::DENSE_SLICE : fnx::DENSE_PLAIN);
      const int occ = fnx::dense_occupancy(c.wt, NT, p.CPW, mode, (p.W + 1 + p.E) * 32, p.smem);
      if (occ <= 0)
        return fail(FNX_EUNSUPPORTED, "kernel does not fit on an SM (smem %zu)", p.smem);
      grid = (int)std::min<int64_t>(p.n_units, (int64_t)fnx::num_sms() * occ);
      if (!p.xslice) break;
      if (grid > p.ksplit) grid -= grid % p.ksplit;  // n_units is a multiple of ksplit
      if (grid % p.ksplit == 0) break;
      if (int e = full_rows()) return e;  // fewer resident CTAs than k splits
    }
  }

  fnx::DenseArgs a = {};
  a.x = c.x;
  a.ldx = c.ldx;
  a.w = static_cast<const uint8_t*>(c.w);
  a.ldw = c.ldw;
  a.bs = static_cast<const uint8_t*>(c.bs);
  a.ldbs = c.ldbs;
  a.scale = c.scale;
  a.scale_kind = c.scale_kind;
  a.y = c.y;
  a.ldy = c.ldy;
  a.y2 = c.y2;
  a.ldy2 = c.ldy2;
  a.split_n = c.y2 ? c.split_n : 0;
  a.out_f32 = c.out_f32;
  a.am_keys = want_argmax ? c.ws->argmax_keys : nullptr;
  a.am_count = want_argmax ? c.ws->argmax_count : nullptr;
  a.am_out = c.argmax_out;
  a.am_key_out = c.argmax_key_out;
  a.row_offset = c.row_offset;
  a.ws = c.ws ? c.ws->partials : nullptr;
  a.ws_cnt = c.ws ? c.ws->counters : nullptr;
  a.err = c.ws ? c.ws->error_flag : nullptr;
  a.M = c.M;
  a.N = c.N;
  a.K = c.K;
  a.ksplit = p.ksplit;
  a.silu = c.silu;
  a.W = p.W;
  a.RT = p.RT;
  a.NS = p.NS;
  a.RS = p.E;
  a.UB = p.UB;
  a.TILE = p.TILE;
  a.E = p.E;
  a.nch_u = p.nch_u;
  a.row_tiles = p.row_tiles;
  a.tile_groups = p.tile_groups;
  a.n_units = p.n_units;
  a.pdl = c.pdl;
  a.norm = c.norm;
  a.chain = c.chain;
  a.peerbuf = c.peerbuf;
  a.xslice = p.xslice;
  rc = fnx::launch_dense(a, c.wt, NT, p.CPW, grid, p.smem, c.stream);
  if (rc == 1) return fail(FNX_EUNSUPPORTED, "no kernel instance for this configuration");
  if (rc) return cuda_fail("dense GEMV launch");
  return FNX_OK;
}

}  // namespace

// Launch geometry of the two MoE kernels for M tokens x R routes over E experts.
struct MoeGeo {
  int NT, w1, cpw1, ns1, cpw2, ns2, EW;
  size_t smem1, smem2;
};

// k1 (gate/up) tiling: H / 128 chunks per row split over W consumer warps of CPW chunks;
// two chunks per warp preferred (fewer per-unit hand-overs), 4 to 11 warps.
bool up_tiling(int H, int& W, int& CPW) {
  const int ch1 = H / 128;
  for (int c : {2, 1, 4})  // producer + 2 epilogue warps + W <= kMoeUpThreads / 32
    if (ch1 % c == 0 && ch1 / c >= 4 && ch1 / c + 3 <= fnx::kMoeUpThreads / 32) {
      CPW = c;
      W = ch1 / c;
      return true;
    }
  return false;
}

int moe_geometry(int M, int R, int E, int H, int I, MoeGeo& g) {
  if (H % 128 || I % 128 || H <= 0 || I <= 0)
    return fail(FNX_EUNSUPPORTED, "H=%d and I=%d must be multiples of 128", H, I);
  g.NT = M > 8 ? 2 : 1;
  g.EW = 2;
  if (!up_tiling(H, g.w1, g.cpw1)) return fail(FNX_EUNSUPPORTED, "H=%d: no gate/up tiling", H);
  // k2: each consumer warp streams one 16-row tile over all of I (I / 128 chunks)
  g.cpw2 = I / 128;
  if (g.cpw2 != 1 && g.cpw2 != 2 && g.cpw2 != 4 && g.cpw2 != 5 && g.cpw2 != 8)
    return fail(FNX_EUNSUPPORTED, "I=%d: the down kernel takes I in {128, 256, 512, 640, 1024}", I);
  auto stages_for = [&](int kernel, int W, int RS, int nbar) {
    const fnx::MoeLayout L0 = fnx::moe_layout(kernel, M, R, E, H, I, W, 0, RS, g.NT, 8);
    const int64_t ns = ((int64_t)kMaxSmem - L0.total - 256) / (L0.stage_bytes + 8 * nbar);
    return (int)std::min<int64_t>(ns, 8);
  };
  g.ns1 = stages_for(1, g.w1, g.EW, 2);
  g.ns2 = stages_for(2, 8, 0, 3);
  if (g.ns1 < 2 || g.ns2 < 2)
    return fail(FNX_EUNSUPPORTED, "MoE shared memory too small for M=%d, H=%d, I=%d", M, H, I);
  g.smem1 = fnx::moe_layout(1, M, R, E, H, I, g.w1, g.ns1, g.EW, g.NT, 8).total;
  g.smem2 = fnx::moe_layout(2, M, R, E, H, I, 8, g.ns2, 0, g.NT, 8).total;
  return FNX_OK;
}

// ---- workspace-free variant ------------------------------------------------------
// Some callers hold no device allocator of their own: a host program that binds the
// C ABI directly (cgo, JNI, a ctypes script) owns the weights and activations it
// passes in, but has no memory pool to carve a scratch buffer from for every shape.
// For them the scratch lives in one static array per device, laid out as
//   [0, 128)      argmax keys (16 x u64)        cleared before each launch
//   [256, 260)    argmax counter (u32)          cleared before each launch
//   [512, 516)    device error word (i32)       cleared before each launch
//   [4096, ...)   split-K counters (the ones a launch uses are cleared before it), then
//                 split-K partial floats
static __device__ __align__(256) unsigned char g_static_scratch[FNX_STATIC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
void* g_static_ptr[kMaxDevices] = {};

// Address of the current device's array, resolved once per device.
int static_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cuda_fail("cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(FNX_EUNSUPPORTED, "device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (!g_static_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || !p)
      return cuda_fail("cudaGetSymbolAddress(static scratch)");
    g_static_ptr[dev] = p;
  }
  *out = g_static_ptr[dev];
  return FNX_OK;
}
}  // namespace

extern "C" {

int fnx_set_dense_path(int path, int* previous) {
  g_err.clear();
  if (path != FNX_DENSE_PATH_AUTO && path != FNX_DENSE_PATH_MMA && path != FNX_DENSE_PATH_TCGEN05)
    return fail(FNX_EINVAL, "dense path %d must be FNX_DENSE_PATH_AUTO, _MMA or _TCGEN05", path);
  const int prev = g_dense_path.exchange(path);
  if (previous) *previous = prev;
  return FNX_OK;
}

int fnx_set_moe_path(int path, int* previous) {
  g_err.clear();
  if (path != FNX_MOE_PATH_AUTO && path != FNX_MOE_PATH_FUSED)
    return fail(FNX_EINVAL, "MoE path %d must be FNX_MOE_PATH_AUTO or _FUSED", path);
  const int prev = g_moe_path.exchange(path);
  if (previous) *previous = prev;
  return FNX_OK;
}

int fnx_plan_gemv(int M, int N, int K, int w_dtype, int fused_silu, int argmax,
                  fnx_gemv_cfg* out) {
  (void)argmax;
  g_err.clear();
  if (!out) return fail(FNX_EINVAL, "null out");
  if (M < 1 || M > FNX_MAX_M) return fail(FNX_EINVAL, "M=%d must be in [1, 16]", M);
  if (w_dtype < FNX_W_INT8 || w_dtype > FNX_W_NVFP4) return fail(FNX_EINVAL, "bad w_dtype");
  DensePlan p;
  const int rc = plan_dense(M, N, K, w_dtype, fused_silu, nullptr, p);
  if (rc) return rc;
  out->warps = p.W;
  out->chunks_per_warp = p.CPW;
  out->groups = p.RT;
  out->ksplit = p.ksplit;
  out->grid = 0;
  return FNX_OK;
}

int fnx_gemv_workspace_need(int M, int N, int K, int w_dtype, int fused_silu,
                            const fnx_gemv_cfg* cfg, int64_t* partial_floats,
                            int64_t* n_counters) {
  g_err.clear();
  DensePlan p;
  const int rc = plan_dense(M, N, K, w_dtype, fused_silu, cfg, p);
  if (rc) return rc;
  if (partial_floats)
    *partial_floats = p.ksplit > 1 ? (int64_t)p.tile_groups * p.ksplit * p.RT * 256 : 0;
  if (n_counters) *n_counters = p.ksplit > 1 ? p.tile_groups : 0;
  return FNX_OK;
}

int fnx_w8a16_gemv(const void* x, int64_t ldx, const void* w, int64_t ldw, int w_dtype,
                   const void* scale, int scale_kind, void* y, int64_t ldy, void* y2,
                   int64_t ldy2, int64_t split_n, int out_f32, int64_t* argmax_out,
                   unsigned long long* argmax_key_out, int64_t row_offset, int M, int N,
                   int K, const fnx_gemv_cfg* cfg, const fnx_workspace* ws, int pdl,
                   fnx_stream_t stream) {
  if (w_dtype != FNX_W_INT8 && w_dtype != FNX_W_FP8_E4M3 && w_dtype != FNX_W_BF16)
    return fail(FNX_EINVAL, "fnx_w8a16_gemv: w_dtype must be int8, fp8_e4m3 or bf16");
  DenseCall c = {x, ldx, w, ldw, w_dtype, nullptr, 0, scale, scale_kind, y, ldy, y2, ldy2,
                 split_n, out_f32, argmax_out, argmax_key_out, row_offset, M, N, K, 0,
                 cfg, ws, pdl, static_cast<cudaStream_t>(stream)};
  return run_dense(c);
}

int fnx_w8a16_gemv_static_ws(const void* x, int64_t ldx, const void* w, int64_t ldw,
                             int w_dtype, const void* scale, int scale_kind, void* y,
                             int64_t ldy, void* y2, int64_t ldy2, int64_t split_n, int out_f32,
                             int64_t* argmax_out, unsigned long long* argmax_key_out,
                             int64_t row_offset, int M, int N, int K, const fnx_gemv_cfg* cfg,
                             int pdl, fnx_stream_t stream) {
  g_err.clear();
  if (w_dtype != FNX_W_INT8 && w_dtype != FNX_W_FP8_E4M3 && w_dtype != FNX_W_BF16)
    return fail(FNX_EINVAL, "fnx_w8a16_gemv_static_ws: w_dtype must be int8, fp8_e4m3 or bf16");
  if (M < 1 || M > FNX_MAX_M) return fail(FNX_EINVAL, "M=%d must be in [1, 16]", M);
  DensePlan p;
  if (int rc = plan_dense(M, N, K, w_dtype, 0, cfg, p)) return rc;
  const int64_t floats = p.ksplit > 1 ? (int64_t)p.tile_groups * p.ksplit * p.RT * 256 : 0;
  const int64_t counters = p.ksplit > 1 ? p.tile_groups : 0;
  if (floats > FNX_STATIC_PARTIAL_FLOATS || counters > FNX_STATIC_COUNTERS)
    return fail(FNX_EUNSUPPORTED,
                "static scratch too small: the plan needs %lld partial floats and %lld counters; "
                "it holds %d and %d (use fnx_w8a16_gemv with a workspace)",
                (long long)floats, (long long)counters, FNX_STATIC_PARTIAL_FLOATS,
                FNX_STATIC_COUNTERS);
  void* base = nullptr;
  if (int rc = static_scratch(&base)) return rc;
  unsigned char* b = static_cast<unsigned char*>(base);
  fnx_workspace ws;
  ws.argmax_keys = reinterpret_cast<unsigned long long*>(b);
  ws.argmax_count = reinterpret_cast<unsigned int*>(b + 256);
  ws.error_flag = reinterpret_cast<int*>(b + 512);
  ws.counters = reinterpret_cast<unsigned int*>(b + 4096);
  ws.n_counters = FNX_STATIC_COUNTERS;
  ws.partials = reinterpret_cast<float*>(b + 4096 + 4 * FNX_STATIC_COUNTERS);
  ws.partial_floats = FNX_STATIC_PARTIAL_FLOATS;
  // The array keeps whatever the previous call left; a call that ended early (a wait
  // that gave up) may have left keys or counters set, or the error word.  Clear what this
  // launch needs at zero, on the caller's stream, before it runs (one contiguous memset of
  // keys, counter and error word; a memset allocates nothing).
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(b, 0, 516, st) != cudaSuccess ||
      (counters > 0 && cudaMemsetAsync(b + 4096, 0, (size_t)counters * 4, st) != cudaSuccess))
    return cuda_fail("clearing the static scratch");
  DenseCall c = {x, ldx, w, ldw, w_dtype, nullptr, 0, scale, scale_kind, y, ldy, y2, ldy2,
                 split_n, out_f32, argmax_out, argmax_key_out, row_offset, M, N, K, 0,
                 cfg, &ws, pdl, static_cast<cudaStream_t>(stream)};
  return run_dense(c);
}

int fnx_static_ws_error(int clear, fnx_stream_t stream, int* code) {
  g_err.clear();
  if (!code) return fail(FNX_EINVAL, "null code");
  void* base = nullptr;
  if (int rc = static_scratch(&base)) return rc;
  int* word = reinterpret_cast<int*>(static_cast<unsigned char*>(base) + 512);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int v = 0;
  if (cudaMemcpyAsync(&v, word, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return cuda_fail("reading the static scratch's error word");
  if (clear && v != 0 &&
      (cudaMemsetAsync(word, 0, sizeof(int), st) != cudaSuccess ||
       cudaStreamSynchronize(st) != cudaSuccess))
    return cuda_fail("clearing the static scratch's error word");
  *code = v;
  return FNX_OK;
}

int fnx_w8a16_gemv_silu_mul(const void* x, int64_t ldx, const void* w, int64_t ldw,
                            int w_dtype, const void* scale, int scale_kind, void* y,
                            int64_t ldy, int M, int H, int K, const fnx_gemv_cfg* cfg,
                            const fnx_workspace* ws, int pdl, fnx_stream_t stream) {
  if (w_dtype != FNX_W_INT8 && w_dtype != FNX_W_FP8_E4M3 && w_dtype != FNX_W_BF16)
    return fail(FNX_EINVAL, "fnx_w8a16_gemv_silu_mul: w_dtype must be int8, fp8_e4m3 or bf16");
  if (scale_kind != FNX_SCALE_F32_ROW && scale_kind != FNX_SCALE_BF16_ROW &&
      !(w_dtype == FNX_W_BF16 && scale_kind == FNX_SCALE_NONE))
    return fail(FNX_EINVAL, "the fused gate_up needs a per-channel scale");
  DenseCall c = {x, ldx, w, ldw, w_dtype, nullptr, 0, scale, scale_kind, y, ldy, nullptr, 0,
                 0, 0, nullptr, nullptr, 0, M, H, K, 1, cfg, ws, pdl,
                 static_cast<cudaStream_t>(stream)};
  return run_dense(c);
}

int fnx_w8a16_gemv_norm_gated(const void* x, int64_t ldx, const void* z, int64_t ldz,
                              const void* norm_weight, int norm_weight_f32, int group_size,
                              float eps, int sigmoid_gate, const void* w, int64_t ldw,
                              int w_dtype, const void* scale, int scale_kind, void* y,
                              int64_t ldy, int out_f32, int M, int N, int K,
                              const fnx_gemv_cfg* cfg, const fnx_workspace* ws, int pdl,
                              fnx_stream_t stream) {
  g_err.clear();
  if (w_dtype != FNX_W_INT8 && w_dtype != FNX_W_FP8_E4M3 && w_dtype != FNX_W_BF16)
    return fail(FNX_EINVAL, "fnx_w8a16_gemv_norm_gated: w_dtype must be int8, fp8_e4m3 or bf16");
  const int G = group_size;
  if (G <= 0 || K <= 0 || K % (G > 0 ? G : 1))
    return fail(FNX_EINVAL, "K=%d must be a positive multiple of group_size=%d", K, G);
  if (G < 8 || G > 256 || (G & (G - 1)))
    return fail(FNX_EUNSUPPORTED, "group_size=%d: the fused norm takes powers of two in [8, 256]",
                G);
  if (!z || !aligned(z, 16) || (ldz * 2) % 16 || ldz < K)
    return fail(FNX_EINVAL, "z rows must be 16-byte aligned with ldz >= K");
  if (!norm_weight || !aligned(norm_weight, 16))
    return fail(FNX_EINVAL, "norm_weight must be a 16-byte aligned [group_size] vector");
  if (!(eps >= 0.f)) return fail(FNX_EINVAL, "eps must be >= 0");
  DenseCall c = {x, ldx, w, ldw, w_dtype, nullptr, 0, scale, scale_kind, y, ldy, nullptr, 0,
                 0, out_f32, nullptr, nullptr, 0, M, N, K, 0, cfg, ws, pdl,
                 static_cast<cudaStream_t>(stream)};
  c.norm.z = static_cast<const __nv_bfloat16*>(z);
  c.norm.ldz = ldz;
  c.norm.w = norm_weight;
  c.norm.w_f32 = norm_weight_f32 ? 1 : 0;
  c.norm.G = G;
  c.norm.eps = eps;
  c.norm.sigmoid = sigmoid_gate ? 1 : 0;
  return run_dense(c);
}

int fnx_router_gemv_topk(const void* x, int64_t ldx, const void* w, int64_t ldw,
                         const void* bias, float* logits, int64_t ldl, float* topk_weights,
                         int32_t* topk_ids, int64_t ldk, int M, int N, int K, int topk,
                         int renormalize, const fnx_workspace* ws, int pdl,
                         fnx_stream_t stream) {
  g_err.clear();
  // router_gemv.py:60-80 (same conditions, same order of checks where they overlap)
  if (M < 1 || M > FNX_MAX_M) return fail(FNX_EINVAL, "router GEMV requires 1 <= M <= 16");
  if (K <= 0 || K % 128 || N <= 0 || N % 32)
    return fail(FNX_EINVAL, "router GEMV requires matching K %% 128 == 0 and N %% 32 == 0");
  if (!x || !w) return fail(FNX_EINVAL, "null x or weight");
  if (!aligned(x, 16) || !aligned(w, 16) || ldx < K || ldw < K || ldx % 8 || ldw % 8)
    return fail(FNX_EINVAL, "x and weight rows must be 16-byte aligned with ld >= K");
  if (bias && !aligned(bias, 2)) return fail(FNX_EINVAL, "misaligned bias");
  if (topk < 0 || topk > 32 || topk > N)
    return fail(topk > 32 ? FNX_EUNSUPPORTED : FNX_EINVAL,
                "topk=%d must be in [0, min(N, 32)]", topk);
  if (topk > 0 && N > 512)
    return fail(FNX_EUNSUPPORTED, "the fused top-k takes at most 512 experts (N=%d)", N);
  if (topk > 0 && (!topk_weights || !topk_ids || ldk < topk))
    return fail(FNX_EINVAL, "topk outputs must be [M, >= topk]");
  if (topk > 0 && (!ws || !ws->counters || ws->n_counters < 1))
    return fail(FNX_EINVAL, "the fused top-k needs a workspace counter");
  float* lg = logits;
  int64_t ld = ldl;
  if (!lg) {
    if (topk == 0) return fail(FNX_EINVAL, "null logits");
    if (!ws->partials || ws->partial_floats < (int64_t)M * N)
      return fail(FNX_EINVAL, "no logits buffer and the workspace holds fewer than M*N floats");
    lg = ws->partials;
    ld = N;
  } else if (ldl < N) {
    return fail(FNX_EINVAL, "ldl=%lld < N=%d", (long long)ldl, N);
  }
  fnx::RouterArgs a = {};
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.ldx = ldx;
  a.w = static_cast<const __nv_bfloat16*>(w);
  a.ldw = ldw;
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.logits = lg;
  a.ldl = ld;
  a.out_w = topk_weights;
  a.out_ids = topk_ids;
  a.ldk = ldk;
  a.counter = topk > 0 ? ws->counters : nullptr;
  a.M = M;
  a.N = N;
  a.K = K;
  a.topk = topk;
  a.renorm = renormalize ? 1 : 0;
  a.pdl = pdl;
  if (fnx::launch_router(a, static_cast<cudaStream_t>(stream))) return cuda_fail("router launch");
  return FNX_OK;
}

int fnx_softmax_topk(const void* scores, int64_t lds, int scores_f32, const float* bias,
                     float* topk_weights, int32_t* topk_ids, int64_t ldk, int M, int N,
                     int topk, int renormalize, int pdl, fnx_stream_t stream) {
  g_err.clear();
  if (M < 0 || N < 1 || N > 512)
    return fail(N > 512 ? FNX_EUNSUPPORTED : FNX_EINVAL, "need M >= 0 and 1 <= N <= 512");
  if (topk < 1 || topk > N || topk > 32)
    return fail(topk > 32 && topk <= N ? FNX_EUNSUPPORTED : FNX_EINVAL,
                "topk=%d must be in [1, min(N, 32)]", topk);
  if (M == 0) return FNX_OK;
  if (!scores || !topk_weights || !topk_ids || lds < N || ldk < topk)
    return fail(FNX_EINVAL, "null or too narrow scores / outputs");
  fnx::TopkArgs a = {};
  a.scores = scores;
  a.lds = lds;
  a.scores_f32 = scores_f32 ? 1 : 0;
  a.bias = bias;
  a.out_w = topk_weights;
  a.out_ids = topk_ids;
  a.ldk = ldk;
  a.M = M;
  a.N = N;
  a.topk = topk;
  a.renorm = renormalize ? 1 : 0;
  a.pdl = pdl;
  if (fnx::launch_softmax_topk(a, static_cast<cudaStream_t>(stream)))
    return cuda_fail("softmax top-k launch");
  return FNX_OK;
}

namespace {

// The draft chain arguments of fnx_draft_topk1 / fnx_draft_head_topk1.
int make_chain(int M, const int64_t* hot_token_id, int64_t* positions, int64_t* draft_tokens,
               int64_t ld_draft, int draft_col, int64_t* topk_index, float* topk_p,
               fnx::DraftChain& c) {
  if (draft_tokens && (draft_col < 0 || ld_draft <= draft_col))
    return fail(FNX_EINVAL, "draft_token_column=%d outside a row of %lld", draft_col,
                (long long)ld_draft);
  if (!topk_index && !topk_p && !draft_tokens && !positions)
    return fail(FNX_EINVAL, "no output of the draft step given");
  c.token_map = hot_token_id;
  c.topk_index = topk_index;
  c.topk_p = topk_p;
  c.draft_tokens = draft_tokens;
  c.draft_ld = ld_draft;
  c.draft_col = draft_col;
  c.positions = positions;
  (void)M;
  return FNX_OK;
}

}  // namespace

int fnx_draft_topk1(const void* logits, int64_t ldl, int logits_f32, int M, int V,
                    const int64_t* hot_token_id, int64_t* positions, int64_t* draft_tokens,
                    int64_t ld_draft, int draft_col, int64_t* topk_index, float* topk_p,
                    const fnx_workspace* ws, int pdl, fnx_stream_t stream) {
  g_err.clear();
  if (M < 0 || M > FNX_MAX_M) return fail(FNX_EUNSUPPORTED, "M=%d must be in [0, 16]", M);
  if (V < 1 || ldl < V) return fail(FNX_EINVAL, "bad logits shape V=%d ldl=%lld", V, (long long)ldl);
  if (M == 0) return FNX_OK;
  if (!logits) return fail(FNX_EINVAL, "null logits");
  if (!ws || !ws->argmax_keys || !ws->argmax_count)
    return fail(FNX_EINVAL, "the top-1 needs the workspace's argmax_keys/argmax_count");
  fnx::Top1Args a = {};
  if (int rc = make_chain(M, hot_token_id, positions, draft_tokens, ld_draft, draft_col,
                          topk_index, topk_p, a.chain))
    return rc;
  a.logits = logits;
  a.ldl = ldl;
  a.logits_f32 = logits_f32 ? 1 : 0;
  a.M = M;
  a.V = V;
  // slices of >= 4096 columns, about two CTAs per SM over all rows
  const int want = std::max(1, (2 * fnx::num_sms()) / M);
  a.splits = std::max(1, std::min(want, (V + 4095) / 4096));
  a.pdl = pdl;
  a.keys = ws->argmax_keys;
  a.count = ws->argmax_count;
  if (fnx::launch_top1(a, static_cast<cudaStream_t>(stream))) return cuda_fail("top-1 launch");
  return FNX_OK;
}

int fnx_draft_head_topk1(const void* x, int64_t ldx, const void* w, int64_t ldw, int w_dtype,
                         const void* scale, int scale_kind, void* logits, int64_t ldl,
                         int out_f32, int M, int N, int K, const int64_t* hot_token_id,
                         int64_t* positions, int64_t* draft_tokens, int64_t ld_draft,
                         int draft_col, int64_t* topk_index, float* topk_p,
                         const fnx_gemv_cfg* cfg, const fnx_workspace* ws, int pdl,
                         fnx_stream_t stream) {
  g_err.clear();
  if (w_dtype != FNX_W_INT8 && w_dtype != FNX_W_FP8_E4M3 && w_dtype != FNX_W_BF16 &&
      w_dtype != FNX_W_NVFP4)
    return fail(FNX_EINVAL, "fnx_draft_head_topk1: bad w_dtype");
  if (w_dtype == FNX_W_NVFP4)
    return fail(FNX_EINVAL, "NVFP4 heads: use fnx_w4a16_nvfp4_gemv with argmax_out");
  DenseCall c = {x, ldx, w, ldw, w_dtype, nullptr, 0, scale, scale_kind, logits, ldl, nullptr,
                 0, 0, out_f32, nullptr, nullptr, 0, M, N, K, 0, cfg, ws, pdl,
                 static_cast<cudaStream_t>(stream)};
  if (int rc = make_chain(M, hot_token_id, positions, draft_tokens, ld_draft, draft_col,
                          topk_index, topk_p, c.chain))
    return rc;
  return run_dense(c);
}

int fnx_peer_alloc(void** buf) {
  g_err.clear();
  if (!buf) return fail(FNX_EINVAL, "null output");
  void* p = nullptr;
  if (cudaMalloc(&p, FNX_PEER_BUFFER_BYTES) != cudaSuccess) return cuda_fail("cudaMalloc");
  if (cudaMemset(p, 0, FNX_PEER_BUFFER_BYTES) != cudaSuccess) {
    cudaFree(p);
    return cuda_fail("cudaMemset");
  }
  *buf = p;
  return FNX_OK;
}

int fnx_peer_free(void* buf) {
  g_err.clear();
  if (buf && cudaFree(buf) != cudaSuccess) return cuda_fail("cudaFree");
  return FNX_OK;
}

int fnx_ipc_get_handle(void* buf, void* handle) {
  g_err.clear();
  if (!buf || !handle) return fail(FNX_EINVAL, "null argument");
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, buf) != cudaSuccess) return cuda_fail("cudaIpcGetMemHandle");
  static_assert(sizeof(h) == FNX_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  return FNX_OK;
}

int fnx_ipc_open(const void* handle, void** buf) {
  g_err.clear();
  if (!handle || !buf) return fail(FNX_EINVAL, "null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return cuda_fail("cudaIpcOpenMemHandle");
  *buf = p;
  return FNX_OK;
}

int fnx_ipc_close(void* buf) {
  g_err.clear();
  if (buf && cudaIpcCloseMemHandle(buf) != cudaSuccess) return cuda_fail("cudaIpcCloseMemHandle");
  return FNX_OK;
}

int fnx_peer_setup(void* local, void* const* bufs, int world, int rank) {
  g_err.clear();
  if (!local || !bufs || world < 1 || world > FNX_MAX_PEERS || rank < 0 || rank >= world)
    return fail(FNX_EINVAL, "bad peer set (world=%d, rank=%d; at most %d ranks)", world, rank,
                FNX_MAX_PEERS);
  if (bufs[rank] != local) return fail(FNX_EINVAL, "bufs[rank] must be this rank's buffer");
  fnx::PeerDesc d = {};
  for (int r = 0; r < world; ++r) {
    if (!bufs[r]) return fail(FNX_EINVAL, "null buffer of rank %d", r);
    d.buf[r] = static_cast<unsigned char*>(bufs[r]);
  }
  d.world = world;
  d.rank = rank;
  if (cudaMemcpy(static_cast<unsigned char*>(local) + fnx::kPeerDescOff, &d, sizeof(d),
                 cudaMemcpyHostToDevice) != cudaSuccess)
    return cuda_fail("writing the peer table");
  return FNX_OK;
}

int fnx_peer_set_wait_limit(void* local, int64_t wait_ns) {
  g_err.clear();
  if (!local || wait_ns < 0) return fail(FNX_EINVAL, "null buffer or negative limit");
  const unsigned long long v = (unsigned long long)wait_ns;
  if (cudaMemcpy(static_cast<unsigned char*>(local) + fnx::kPeerDescOff +
                     offsetof(fnx::PeerDesc, wait_ns),
                 &v, sizeof(v), cudaMemcpyHostToDevice) != cudaSuccess)
    return cuda_fail("writing the wait limit");
  return FNX_OK;
}

int fnx_w8a16_gemv_vocab_sharded(const void* x, int64_t ldx, const void* w, int64_t ldw,
                                 int w_dtype, const void* scale, int scale_kind, void* y,
                                 int64_t ldy, int out_f32, int64_t* argmax_out,
                                 int64_t row_offset, int M, int N, int K, void* peer_buf,
                                 const fnx_gemv_cfg* cfg, const fnx_workspace* ws, int pdl,
                                 fnx_stream_t stream) {
  g_err.clear();
  if (w_dtype != FNX_W_INT8 && w_dtype != FNX_W_FP8_E4M3 && w_dtype != FNX_W_BF16)
    return fail(FNX_EINVAL, "fnx_w8a16_gemv_vocab_sharded: w_dtype must be int8, fp8_e4m3 or bf16");
  if (!peer_buf) return fail(FNX_EINVAL, "null peer buffer");
  DenseCall c = {x, ldx, w, ldw, w_dtype, nullptr, 0, scale, scale_kind, y, ldy, nullptr, 0,
                 0, out_f32, argmax_out, nullptr, row_offset, M, N, K, 0, cfg, ws, pdl,
                 static_cast<cudaStream_t>(stream)};
  c.peerbuf = static_cast<unsigned char*>(peer_buf);
  return run_dense(c);
}

int fnx_w4a16_nvfp4_gemv(const void* x, int64_t ldx, const void* wq, int64_t ldwq,
                         const void* bs, int64_t ldbs, const float* gscale,
                         int gscale_per_row, void* y, int64_t ldy, void* y2, int64_t ldy2,
                         int64_t split_n, int out_f32, int64_t* argmax_out,
                         unsigned long long* argmax_key_out, int64_t row_offset, int M,
                         int N, int K, const fnx_gemv_cfg* cfg, const fnx_workspace* ws,
                         int pdl, fnx_stream_t stream) {
  if (!gscale) return fail(FNX_EINVAL, "null gscale");
  DenseCall c = {x, ldx, wq, ldwq, FNX_W_NVFP4, bs, ldbs, gscale,
                 gscale_per_row ? FNX_SCALE_F32_ROW : FNX_SCALE_F32_SCALAR, y, ldy, y2, ldy2,
                 split_n, out_f32, argmax_out, argmax_key_out, row_offset, M, N, K, 0, cfg, ws,
                 pdl, static_cast<cudaStream_t>(stream)};
  return run_dense(c);
}

int fnx_nvfp4_quantize(const void* w, int64_t ldw, int w_f32, int N, int K, void* wq,
                       int64_t ldwq, void* bs, int64_t ldbs, float* gscale,
                       unsigned int* scratch, fnx_stream_t stream) {
  g_err.clear();
  if (N < 1 || K < 16 || K % 16) return fail(FNX_EINVAL, "N=%d, K=%d: K must be a multiple of 16", N, K);
  if (!w || !wq || !bs || !gscale || !scratch) return fail(FNX_EINVAL, "null argument");
  if (ldw < K || ldwq < K / 2 || ldbs < K / 16 || ldwq % 8 || !aligned(wq, 8))
    return fail(FNX_EINVAL, "bad strides: need ldw >= K, ldwq >= K/2 (multiple of 8, wq 8-byte "
                "aligned), ldbs >= K/16");
  if (fnx::launch_nvfp4_quantize(w, ldw, w_f32, N, K, static_cast<uint8_t*>(wq), ldwq,
                                 static_cast<uint8_t*>(bs), ldbs, gscale, scratch,
                                 static_cast<cudaStream_t>(stream)))
    return cuda_fail("NVFP4 quantise launch");
  return FNX_OK;
}

int fnx_nvfp4_dequantize(const void* wq, int64_t ldwq, const void* bs, int64_t ldbs,
                         const float* gscale, int gscale_per_row, void* out, int64_t ldo,
                         int out_f32, int N, int K, fnx_stream_t stream) {
  g_err.clear();
  if (N < 0 || K < 16 || K % 16) return fail(FNX_EINVAL, "N=%d, K=%d: K must be a multiple of 16", N, K);
  if (N == 0) return FNX_OK;
  if (!wq || !bs || !gscale || !out) return fail(FNX_EINVAL, "null argument");
  if (ldwq < K / 2 || ldbs < K / 16 || ldo < K || ldwq % 8 || !aligned(wq, 8))
    return fail(FNX_EINVAL, "bad strides: need ldwq >= K/2 (multiple of 8, wq 8-byte aligned), "
                "ldbs >= K/16, ldo >= K");
  if (fnx::launch_nvfp4_dequantize(static_cast<const uint8_t*>(wq), ldwq,
                                   static_cast<const uint8_t*>(bs), ldbs, gscale, gscale_per_row,
                                   out, ldo, out_f32, N, K, static_cast<cudaStream_t>(stream)))
    return cuda_fail("NVFP4 dequantise launch");
  return FNX_OK;
}

int fnx_moe_workspace_bytes(int max_m, int max_routes, int num_experts, int H, int I,
                            fnx_moe_workspace_sizes* out) {
  g_err.clear();
  if (!out || max_m < 1 || max_routes < 1 || num_experts < 1 || H < 64 || I < 1)
    return fail(FNX_EINVAL, "bad MoE shape");
  MoeGeo geo;
  if (int rc = moe_geometry(max_m, max_routes, num_experts, H, I, geo)) return rc;
  const int64_t pairs = (int64_t)max_m * (max_routes + 1);
  const int64_t dcap = std::min<int64_t>(num_experts, (int64_t)max_m * max_routes) + 1;
  const int64_t vcap = fnx::fused_vcap(max_m, max_routes, num_experts);
  // the three-launch form: 16 slots per distinct expert; the fused form: 8 per virtual one
  out->act = std::max(dcap * 16, vcap * fnx::kFusedSlots) * (2LL * I + 64);
  out->partials = pairs * H * 4;
  out->counters = vcap + H / 64 + 1;
  return FNX_OK;
}

namespace {

// Launch geometry of the fused layer: the deepest weight ring that fits beside the staged
// activations, the act and result slots and the routing tables (at least 4 stages).
int fused_plan(int M, int R, int E, int H, int I, int vcap, int& NG, int& NS, size_t& smem) {
  const fnx::FusedLayout L0 = fnx::fused_layout(M, R, E, H, I, 0, vcap);
  int64_t ns = ((int64_t)kMaxSmem - L0.total - 256) / (L0.stage_bytes + 16);
  ns = std::min<int64_t>(ns, 12);
  ns -= ns % fnx::kFusedRing;  // every stage owned by one producer warp and one consumer group
  if (ns < 4)
    return fail(FNX_EUNSUPPORTED, "fused MoE: shared memory too small for M=%d, H=%d, I=%d", M, H, I);
  NG = fnx::kFusedMaxGroups;
  NS = (int)ns;
  smem = fnx::fused_layout(M, R, E, H, I, NS, vcap).total;
  return FNX_OK;
}

}  // namespace

int fnx_plan_moe(int M, int R, int E, int H, int I, int* fused, int* stages, int* groups,
                 int64_t* smem_bytes) {
  g_err.clear();
  if (!fused) return fail(FNX_EINVAL, "null fused");
  if (M < 1 || M > FNX_MAX_M || R < 1 || R > 32 || E < 1 || E > 4096)
    return fail(FNX_EINVAL, "M=%d, R=%d, E=%d out of range", M, R, E);
  int ng = 0, ns = 0;
  size_t smem = 0;
  if (g_moe_path.load(std::memory_order_relaxed) == FNX_MOE_PATH_AUTO &&
      fnx::moe_lean_plan(M, R, E, H, I, fnx::num_sms(), ns, smem)) {
    *fused = 2;
    if (stages) *stages = ns;
    if (groups) *groups = 2;
    if (smem_bytes) *smem_bytes = (int64_t)smem;
    return FNX_OK;
  }
  const bool f = fnx::moe_fused_has(H, I) &&
                 fused_plan(M, R, E, H, I, fnx::fused_vcap(M, R, E), ng, ns, smem) == FNX_OK;
  g_err.clear();
  *fused = f ? 1 : 0;
  if (stages) *stages = f ? ns : 0;
  if (groups) *groups = f ? ng : 0;
  if (smem_bytes) *smem_bytes = f ? (int64_t)smem : 0;
  return FNX_OK;
}

int fnx_moe_gemv(const void* x, int64_t ldx, const int32_t* topk_ids,
                 const float* topk_weights, int M, int R, const fnx_moe_weights* experts,
                 const fnx_moe_weights* shared, void* out, int64_t ldo, int out_f32,
                 const fnx_moe_workspace* ws, int pdl, fnx_stream_t stream) {
  g_err.clear();
  if (!experts || !ws || !out || !x) return fail(FNX_EINVAL, "null argument");
  if (M < 0 || M > FNX_MAX_M) return fail(FNX_EINVAL, "M=%d must be in [0, 16]", M);
  if (M == 0) return FNX_OK;
  if (R < 1 || R > 32) return fail(FNX_EINVAL, "top_k=%d must be in [1, 32]", R);
  if (!topk_ids || !topk_weights) return fail(FNX_EINVAL, "null topk_ids / topk_weights");
  const int H = experts->hidden, I = experts->inter, E = experts->num_experts;
  if (E < 1 || E > 4096) return fail(FNX_EINVAL, "num_experts=%d must be in [1, 4096]", E);
  if (!experts->w13 || !experts->w13_scale || !experts->w13_gscale || !experts->w2 ||
      !experts->w2_scale || !experts->w2_gscale)
    return fail(FNX_EINVAL, "null expert tensor");
  if (!aligned(experts->w13, 16) || !aligned(experts->w2, 16) || !aligned(experts->w13_scale, 2) ||
      !aligned(experts->w2_scale, 2))
    return fail(FNX_EINVAL, "expert weights must be 16-byte aligned, scales 2-byte aligned");
  if (!aligned(x, 16) || (ldx * 2) % 16 || ldx < H)
    return fail(FNX_EINVAL, "x rows must be 16-byte aligned with ldx >= H");
  if (ldo < H) return fail(FNX_EINVAL, "ldo < H");
  if (shared) {
    if (shared->hidden != H || shared->inter != I || !shared->w13 || !shared->w2 ||
        !shared->w13_scale || !shared->w2_scale || !shared->w13_gscale || !shared->w2_gscale)
      return fail(FNX_EINVAL, "shared expert must match H and I");
    if (shared->scales_swizzled != experts->scales_swizzled)
      return fail(FNX_EINVAL, "shared and routed experts must use one scale layout");
    if (!aligned(shared->w13, 16) || !aligned(shared->w2, 16))
      return fail(FNX_EINVAL, "shared expert weights must be 16-byte aligned");
  }
  if (!ws->act || !ws->partials || ws->max_m < M || ws->max_routes < R)
    return fail(FNX_EINVAL, "MoE workspace missing or sized for fewer tokens/routes");
  if (!aligned(ws->act, 16)) return fail(FNX_EINVAL, "MoE workspace act rows must be 16-byte aligned");
  // the one-launch layer when the workspace has its counters, the tiling is compiled and
  // its shared memory fits; otherwise the three-launch layer
  int fng = 0, fns = 0;
  size_t fsmem = 0;
  const bool fused = ws->counters && fnx::moe_fused_has(H, I) &&
                     fused_plan(M, R, E, H, I, fnx::fused_vcap(M, R, E), fng, fns, fsmem) == FNX_OK;
  g_err.clear();
  if (fused && (int64_t)ws->n_counters < (int64_t)fnx::fused_vcap(M, R, E) + H / 64 + 1)
    return fail(FNX_EINVAL, "MoE workspace counters too few for M=%d, R=%d, E=%d", M, R, E);
  const int NT = M > 8 ? 2 : 1;
  const int sms = fnx::num_sms();
  const int has_shared = shared ? 1 : 0;
  const int dmax = std::min(E, M * R) + has_shared;

  fnx::MoeArgs a = {};
  a.x = x;
  a.ldx = ldx;
  a.ids = topk_ids;
  a.wts = topk_weights;
  a.M = M;
  a.R = R;
  a.E = E;
  a.H = H;
  a.I = I;
  a.w13 = static_cast<const uint8_t*>(experts->w13);
  a.s13 = static_cast<const uint8_t*>(experts->w13_scale);
  a.g13 = experts->w13_gscale;
  a.g13_stride = experts->w13_gscale_stride;
  a.w2 = static_cast<const uint8_t*>(experts->w2);
  a.s2 = static_cast<const uint8_t*>(experts->w2_scale);
  a.g2 = experts->w2_gscale;
  a.g2_stride = experts->w2_gscale_stride;
  if (shared) {
    a.sh_w13 = static_cast<const uint8_t*>(shared->w13);
    a.sh_s13 = static_cast<const uint8_t*>(shared->w13_scale);
    a.sh_g13 = shared->w13_gscale;
    a.sh_w2 = static_cast<const uint8_t*>(shared->w2);
    a.sh_s2 = static_cast<const uint8_t*>(shared->w2_scale);
    a.sh_g2 = shared->w2_gscale;
  }
  a.has_shared = has_shared;
  a.swizzled = experts->scales_swizzled;
  a.e_lo = experts->expert_offset;
  a.act = static_cast<uint8_t*>(ws->act);
  a.part = ws->partials;
  a.err = ws->error_flag;
  a.out = out;
  a.ldo = ldo;
  a.out_f32 = out_f32;
  a.NT = NT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  // The decode-width layer (M <= 8, swizzled scales): every SM one CTA, all resident.
  if (ws->counters && experts->scales_swizzled &&
      g_moe_path.load(std::memory_order_relaxed) == FNX_MOE_PATH_AUTO &&
      aligned(experts->w13_scale, 16) && aligned(experts->w2_scale, 16) &&
      (!shared || (aligned(shared->w13_scale, 16) && aligned(shared->w2_scale, 16))) &&
      (int64_t)ws->n_counters >= fnx::moe_lean_counters(M, R, E)) {
    int lns = 0;
    size_t lsmem = 0;
    if (fnx::moe_lean_plan(M, R, E, H, I, sms, lns, lsmem)) {
      a.cnt = ws->counters;
      a.pdl = pdl;
      const int rc = fnx::launch_moe_lean(a, lns, sms, lsmem, st);
      if (rc == 0) return FNX_OK;
      if (rc != 3) return cuda_fail("decode-width MoE launch");
      // rc 3: the weights' tensor maps could not be encoded: the general layer below
    }
  }

  if (fused) {
    a.vcap = fnx::fused_vcap(M, R, E);
    a.cnt = ws->counters;
    a.NG = fng;
    a.NS = fns;
    const size_t smem = fsmem;
    a.pdl = pdl;
    // one CTA per SM at most (the CTAs wait for one another), never more than the items
    const int64_t max_items = (int64_t)a.vcap * (I / 8 + H / 64);
    const int grid = (int)std::min<int64_t>(max_items, sms);
    const int rc = fnx::launch_moe_fused(a, grid, smem, st);
    if (rc == 1) return fail(FNX_EUNSUPPORTED, "no fused MoE instance for H=%d, I=%d", H, I);
    if (rc) return cuda_fail("fused MoE launch");
    return FNX_OK;
  }

  MoeGeo geo;
  if (int rc = moe_geometry(M, R, E, H, I, geo)) return rc;
  const int w1 = geo.w1, cpw1 = geo.cpw1, ns1 = geo.ns1;
  const int cpw2 = geo.cpw2, ns2 = geo.ns2;
  a.EW = geo.EW;
  a.RS = geo.EW;

  a.W = w1;
  a.CPW = cpw1;
  a.NS = ns1;
  a.pdl = pdl;
  const size_t smem1 = geo.smem1;
  const int occ1 = fnx::moe_up_occupancy(NT, cpw1, (w1 + 1 + a.EW) * 32, smem1);
  if (occ1 <= 0) return fail(FNX_EUNSUPPORTED, "k1 does not fit on an SM");
  const int64_t units1 = (int64_t)dmax * (I / 8);
  const int grid1 = (int)std::min<int64_t>(units1, (int64_t)sms * occ1);
  int rc = fnx::launch_moe_up(a, NT, grid1, smem1, st);
  if (rc == 1) return fail(FNX_EUNSUPPORTED, "no k1 instance");
  if (rc) return cuda_fail("MoE k1 launch");

  a.W = 8;
  a.CPW = cpw2;
  a.NS = ns2;
  a.RS = 0;
  a.pdl = 1;  // k2 decodes the routes and streams W2 while k1 drains
  const size_t smem2 = geo.smem2;
  const int occ2 = fnx::moe_down_occupancy(NT, cpw2, 10 * 32, smem2);
  if (occ2 <= 0) return fail(FNX_EUNSUPPORTED, "k2 does not fit on an SM");
  const int64_t units2 = (int64_t)dmax * (H / 128);
  const int grid2 = (int)std::min<int64_t>(units2, (int64_t)sms * occ2);
  rc = fnx::launch_moe_down(a, NT, grid2, smem2, st);
  if (rc == 1) return fail(FNX_EUNSUPPORTED, "no k2 instance");
  if (rc) return cuda_fail("MoE k2 launch");
  if (fnx::launch_moe_sum(a, st)) return cuda_fail("MoE route-sum launch");
  return FNX_OK;
}

int fnx_argmax_decode(const unsigned long long* keys, int64_t* out, int M,
                      fnx_stream_t stream) {
  g_err.clear();
  if (!keys || !out || M < 1 || M > 32) return fail(FNX_EINVAL, "bad argmax_decode arguments");
  if (fnx::launch_argmax_decode(keys, out, M, static_cast<cudaStream_t>(stream)))
    return cuda_fail("argmax decode launch");
  return FNX_OK;
}

const char* fnx_last_error(void) { return g_err.c_str(); }

const char* fnx_version(void) { return "fnx-b200 0.1.0 (sm_100a)"; }

}  // extern "C"
