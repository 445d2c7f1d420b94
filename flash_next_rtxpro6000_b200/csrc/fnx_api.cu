// C ABI of the GEMV library (include/fnx_gemv.h): argument validation mirroring the
// reference's Python wrappers, the launch planner, and the kernel launches.
#include <cuda_runtime.h>

#include <algorithm>
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

size_t dense_smem(int M, int K, int W, int G, int NT) {
  return (size_t)M * fnx::stage_row_bytes(K) + 64 + (size_t)G * 2 * W * 32 * NT * 16 + 64;
}

constexpr size_t kMaxSmem = 227 * 1024;

// Planner for the dense GEMVs.  One 16-row tile (8 SiLU outputs) per unit; the warps of
// a group split the tile's k range; k is also split across groups (ksplit) when the tile
// count alone cannot keep every SM streaming.
int plan_dense(int M, int N, int K, int wt, int silu, fnx_gemv_cfg* out) {
  const int CH = chunk_k(wt);
  if (K <= 0 || K % CH)
    return fail(FNX_EUNSUPPORTED, "K=%d must be a positive multiple of %d for this weight type",
                K, CH);
  const int nch = K / CH;
  const int row_tiles = silu ? (N + 7) / 8 : (N + 15) / 16;
  const int sms = fnx::num_sms();
  const int min_w = std::max(1, (M + 1) / 2);  // one output thread per (token, tile row)
  int best_ks = -1, best_w = 0, best_cpw = 0;
  for (int ks = 1; ks <= nch; ++ks) {
    if (nch % ks) continue;
    const int cpu = nch / ks;
    int w = 0, cpw = 0;
    for (int c : {2, 1, 4}) {
      if (cpu % c) continue;
      const int ww = cpu / c;
      if (ww >= min_w && ww <= 16) {
        w = ww;
        cpw = c;
        break;
      }
    }
    if (!w) continue;
    if (best_ks < 0) {
      best_ks = ks;
      best_w = w;
      best_cpw = cpw;
    }
    if ((int64_t)row_tiles * best_ks >= 3 * sms) break;
    if (ks > best_ks) {
      best_ks = ks;
      best_w = w;
      best_cpw = cpw;
    }
  }
  if (best_ks < 0)
    return fail(FNX_EUNSUPPORTED, "no tiling of K=%d (%d chunks) for M=%d", K, nch, M);
  out->ksplit = best_ks;
  out->warps = best_w;
  out->chunks_per_warp = best_cpw;
  // groups share a CTA through named barriers 1..groups (ids 0..15 exist; keep <= 8)
  out->groups = std::max(1, std::min(std::min(16 / best_w, 8), row_tiles * best_ks));
  out->grid = 0;
  return FNX_OK;
}

int check_cfg(int M, int K, int wt, const fnx_gemv_cfg& c) {
  const int CH = chunk_k(wt);
  if (K % CH) return fail(FNX_EUNSUPPORTED, "K=%d not a multiple of %d", K, CH);
  const int nch = K / CH;
  if (c.chunks_per_warp != 1 && c.chunks_per_warp != 2 && c.chunks_per_warp != 4)
    return fail(FNX_EINVAL, "chunks_per_warp must be 1, 2 or 4");
  if (c.warps < 1 || c.groups < 1 || c.groups > 8 || c.warps * c.groups > 16)
    return fail(FNX_EINVAL, "need 1 <= groups <= 8 and warps * groups <= 16");
  if (c.warps * 32 < 16 * M)
    return fail(FNX_EINVAL, "warps=%d too few for M=%d (need warps >= M/2)", c.warps, M);
  if (c.ksplit < 1 || (int64_t)c.warps * c.chunks_per_warp * c.ksplit != nch)
    return fail(FNX_EINVAL, "warps * chunks_per_warp * ksplit must equal K/%d = %d", CH, nch);
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
    if (!c.bs || c.ldbs < c.K / 16 || c.ldbs % 2 || !aligned(c.bs, 2))
      return fail(FNX_EINVAL, "block scales must be [N, K/16] with an even row stride");
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

  fnx_gemv_cfg cfg;
  if (c.cfg) {
    cfg = *c.cfg;
  } else {
    const int rc = plan_dense(c.M, c.N, c.K, c.wt, c.silu, &cfg);
    if (rc) return rc;
  }
  int rc = check_cfg(c.M, c.K, c.wt, cfg);
  if (rc) return rc;

  const int NT = c.M > 8 ? 2 : 1;
  const int row_tiles = c.silu ? (c.N + 7) / 8 : (c.N + 15) / 16;
  const int64_t n_units = (int64_t)row_tiles * cfg.ksplit;
  if (n_units > 0x7FFFFFFF) return fail(FNX_EUNSUPPORTED, "too many tiles");
  const size_t smem = dense_smem(c.M, c.K, cfg.warps, cfg.groups, NT);
  if (smem > kMaxSmem)
    return fail(FNX_EUNSUPPORTED, "shared memory %zu > %zu (M=%d K=%d)", smem, kMaxSmem, c.M, c.K);

  const bool want_argmax = c.argmax_out || c.argmax_key_out;
  if (cfg.ksplit > 1) {
    if (!c.ws || !c.ws->partials || !c.ws->counters)
      return fail(FNX_EINVAL, "ksplit=%d needs a workspace", cfg.ksplit);
    if (c.ws->partial_floats < n_units * 256 || c.ws->n_counters < row_tiles)
      return fail(FNX_EINVAL, "workspace too small: need %lld floats and %d counters",
                  (long long)(n_units * 256), row_tiles);
  }
  if (want_argmax && (!c.ws || !c.ws->argmax_keys || !c.ws->argmax_count))
    return fail(FNX_EINVAL, "argmax needs the workspace's argmax_keys/argmax_count");

  const int threads = cfg.warps * cfg.groups * 32;
  int grid = cfg.grid;
  if (grid <= 0) {
    const int occ = fnx::dense_occupancy(c.wt, NT, cfg.chunks_per_warp, threads, smem);
    if (occ <= 0) return fail(FNX_EUNSUPPORTED, "kernel does not fit on an SM (smem %zu)", smem);
    const int64_t want = (n_units + cfg.groups - 1) / cfg.groups;
    grid = (int)std::min<int64_t>(want, (int64_t)fnx::num_sms() * occ);
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
  a.M = c.M;
  a.N = c.N;
  a.K = c.K;
  a.ksplit = cfg.ksplit;
  a.silu = c.silu;
  a.W = cfg.warps;
  a.G = cfg.groups;
  a.row_tiles = row_tiles;
  a.n_units = (int)n_units;
  a.pdl = c.pdl;
  rc = fnx::launch_dense(a, c.wt, NT, cfg.chunks_per_warp, grid, smem, c.stream);
  if (rc == 1) return fail(FNX_EUNSUPPORTED, "no kernel instance for this configuration");
  if (rc) return cuda_fail("dense GEMV launch");
  return FNX_OK;
}

}  // namespace

extern "C" {

int fnx_plan_gemv(int M, int N, int K, int w_dtype, int fused_silu, int argmax,
                  fnx_gemv_cfg* out) {
  (void)argmax;
  g_err.clear();
  if (!out) return fail(FNX_EINVAL, "null out");
  if (M < 1 || M > FNX_MAX_M) return fail(FNX_EINVAL, "M=%d must be in [1, 16]", M);
  if (w_dtype < FNX_W_INT8 || w_dtype > FNX_W_NVFP4) return fail(FNX_EINVAL, "bad w_dtype");
  return plan_dense(M, N, K, w_dtype, fused_silu, out);
}

int fnx_gemv_workspace_need(int M, int N, int K, int w_dtype, int fused_silu,
                            const fnx_gemv_cfg* cfg, int64_t* partial_floats,
                            int64_t* n_counters) {
  fnx_gemv_cfg c;
  if (cfg) {
    c = *cfg;
  } else {
    const int rc = fnx_plan_gemv(M, N, K, w_dtype, fused_silu, 0, &c);
    if (rc) return rc;
  }
  const int64_t row_tiles = fused_silu ? (N + 7) / 8 : (N + 15) / 16;
  if (partial_floats) *partial_floats = c.ksplit > 1 ? row_tiles * c.ksplit * 256 : 0;
  if (n_counters) *n_counters = c.ksplit > 1 ? row_tiles : 0;
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

int fnx_moe_workspace_bytes(int M, int R, int H, int I, int64_t* act_bytes,
                            int64_t* partial_bytes, int64_t* counter_bytes) {
  g_err.clear();
  if (M < 1 || R < 1 || H < 16 || I < 1) return fail(FNX_EINVAL, "bad MoE shape");
  const int64_t pairs = (int64_t)M * (R + 1);
  if (act_bytes) *act_bytes = pairs * I * 2;
  if (partial_bytes) *partial_bytes = pairs * H * 4;
  if (counter_bytes) *counter_bytes = (int64_t)(H / 16) * 4;
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
  if (H % 128 || I % 128 || H <= 0 || I <= 0)
    return fail(FNX_EUNSUPPORTED, "H=%d and I=%d must be multiples of 128", H, I);
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
  if (!ws->act || !ws->partials || !ws->counters || ws->max_m < M || ws->max_routes < R)
    return fail(FNX_EINVAL, "MoE workspace missing or sized for fewer tokens/routes");

  const int NT = M > 8 ? 2 : 1;
  const int sms = fnx::num_sms();
  const int has_shared = shared ? 1 : 0;
  const int dmax = std::min(E, M * R) + has_shared;

  // k1: the warps of a group split H into 128-wide chunks.
  const int ch1 = H / 128;
  int w1 = ch1, cpw1 = 1;
  if (w1 > 16 || w1 < 8) {
    if (ch1 % 2 == 0 && ch1 / 2 >= 8 && ch1 / 2 <= 16) {
      w1 = ch1 / 2;
      cpw1 = 2;
    } else {
      return fail(FNX_EUNSUPPORTED, "H=%d: no k1 tiling (needs 8..32 chunks of 128)", H);
    }
  }
  const int g1 = 1;
  // k2: I in 128-wide chunks, several tiles per CTA.
  const int ch2 = I / 128;
  int w2 = ch2, cpw2 = 1;
  if (w2 > 16) {
    if (ch2 % 2 == 0 && ch2 / 2 <= 16) {
      w2 = ch2 / 2;
      cpw2 = 2;
    } else {
      return fail(FNX_EUNSUPPORTED, "I=%d: no k2 tiling", I);
    }
  }
  const int g2 = std::max(1, std::min(16 / w2, 8));
  const size_t smem1 = fnx::moe_up_smem(M, R, E, H, w1, g1, NT);
  const size_t smem2 = fnx::moe_down_smem(M, R, E, I, w2, g2, NT);
  if (smem1 > kMaxSmem || smem2 > kMaxSmem)
    return fail(FNX_EUNSUPPORTED, "MoE shared memory %zu / %zu exceeds %zu", smem1, smem2,
                kMaxSmem);

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
  a.act = ws->act;
  a.part = ws->partials;
  a.cnt = ws->counters;
  a.out = out;
  a.ldo = ldo;
  a.out_f32 = out_f32;
  a.pdl = pdl;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  a.W = w1;
  a.G = g1;
  const int occ1 = fnx::moe_up_occupancy(NT, cpw1, w1 * g1 * 32, smem1);
  if (occ1 <= 0) return fail(FNX_EUNSUPPORTED, "k1 does not fit on an SM");
  const int64_t units1 = (int64_t)dmax * (I / 8);
  const int grid1 = (int)std::min<int64_t>((units1 + g1 - 1) / g1, (int64_t)sms * occ1);
  int rc = fnx::launch_moe_up(a, NT, grid1, smem1, st);
  if (rc == 1) return fail(FNX_EUNSUPPORTED, "no k1 instance");
  if (rc) return cuda_fail("MoE k1 launch");

  a.W = w2;
  a.G = g2;
  a.pdl = 1;  // k2 always overlaps its weight prefetch with k1's tail
  const int occ2 = fnx::moe_down_occupancy(NT, cpw2, w2 * g2 * 32, smem2);
  if (occ2 <= 0) return fail(FNX_EUNSUPPORTED, "k2 does not fit on an SM");
  const int64_t units2 = (int64_t)dmax * (H / 16);
  const int grid2 = (int)std::min<int64_t>((units2 + g2 - 1) / g2, (int64_t)sms * occ2);
  rc = fnx::launch_moe_down(a, NT, grid2, smem2, st);
  if (rc == 1) return fail(FNX_EUNSUPPORTED, "no k2 instance");
  if (rc) return cuda_fail("MoE k2 launch");
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
