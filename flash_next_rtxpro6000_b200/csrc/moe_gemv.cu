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
// Both kernels are persistent and warp-specialised like the dense GEMV: warp 0 bulk-
// copies the unit's weight rows (and, in k2, its B rows) into a shared-memory ring,
// warps 2.. dequantise + MMA, warp 1 runs the epilogue.
//
// k1 unit: (distinct expert, 8 columns of I): MMA rows 0..7 are up rows, 8..15 the
// matching gate rows, so one epilogue lane holds both and applies
// silu(gate * g) * (up * g) (0112-...patch:220-224), rounding act to bf16.  The last k1
// unit of an expert to finish converts that expert's act rows to fp16 scaled by a
// per-route power of two, in the B-fragment layout, for k2 to bulk-copy.
// k2 unit: (distinct expert, 16 * RT rows of H, RT <= 4): contribution = <W2 row, act> * (g2 * w_r)
// (0112-...patch:268-269) written as an fp32 partial per (token, route); the last unit
// to finish a 64-row group sums each token's routes in route order (then the shared
// expert) and rounds once to bf16: deterministic, no float atomics.
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
  return r;
}

// Build the routing table (CTA-wide; ends with __syncthreads).
__device__ void route_decode(const MoeArgs& a, const Routing& rt) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nthreads = blockDim.x, nwarps = nthreads >> 5;
  const int n = a.M * a.R;
  const int nw = (a.E + 31) / 32;
  for (int i = tid; i < nw; i += nthreads) rt.bitmap[i] = 0u;
  for (int i = tid; i < n; i += nthreads) {
    const int t = i / a.R, r = i - t * a.R;
    const int id = __ldcg(a.ids + (size_t)t * a.R + r);
    const int loc = id - a.e_lo;
    rt.ids[i] = (id >= 0 && loc >= 0 && loc < a.E) ? loc : -1;
  }
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
  __syncthreads();
  const int D = rt.misc[0];
  for (int d = warp; d < D; d += nwarps) {
    const int e = rt.exp_of[d];
    int cnt = 0;
    for (int base = 0; base < n; base += 32) {
      const int i = base + lane;
      const bool match = (i < n) && rt.ids[i] == e;
      const uint32_t bal = __ballot_sync(0xffffffffu, match);
      if (match) {
        const int k = cnt + __popc(bal & ((1u << lane) - 1u));
        if (k < kSlotCap) rt.ent[d * kSlotCap + k] = (short)i;
      }
      cnt += __popc(bal);
    }
    if (lane == 0) rt.cnt_of[d] = cnt < kSlotCap ? cnt : kSlotCap;
  }
  __syncthreads();
}

// Byte offset of the two e4m3 scales of (row, kb..kb+1) inside one expert's scale block.
__device__ __forceinline__ int64_t scale_offset(int swizzled, int row, int kb, int KP) {
  if (!swizzled) return (int64_t)row * KP + kb;
  // 128x4 layout: (m/128)*128*KP + (kb/4)*512 + (m%32)*16 + ((m%128)/32)*4 + kb%4
  return (int64_t)(row >> 7) * 128 * KP + (int64_t)(kb >> 2) * 512 + (row & 31) * 16 +
         ((row & 127) >> 5) * 4 + (kb & 3);
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

__device__ __forceinline__ int pair_of(int entry, int R) {
  if (entry < 0) {  // shared expert: token -1 - entry, route slot R
    const int t = -1 - entry;
    return t * (R + 1) + R;
  }
  return entry + entry / R;  // t * (R + 1) + r
}

__device__ __forceinline__ int token_of(int entry, int R) {
  return entry < 0 ? -1 - entry : entry / R;
}

}  // namespace

// ------------------------------------------------------------------------------------
// k1: act[t*(R+1)+r, j] = bf16(silu(g * <gate_j, x_t>) * g * <up_j, x_t>)
// ------------------------------------------------------------------------------------
template <int NT, int CPW>
__global__ void __launch_bounds__(kDenseThreadsMax, 1) moe_up_kernel(const MoeArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int Q = Geo<W_NVFP4>::Q;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int M = a.M, R = a.R, H = a.H, I = a.I, W = a.W, NS = a.NS, RS = a.RS;
  const MoeLayout L = moe_layout(1, M, R, a.E, H, I, W, NS, RS, NT, 1);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + NS;
  uint64_t* rfull = empty + NS;
  uint64_t* rfree = rfull + RS;
  uint8_t* stages = smem + L.stages;
  uint8_t* xs = smem + L.xs;
  float* unscale = reinterpret_cast<float*>(smem + L.unscale);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* sred = red + RS * W * 32 * NT * 4;
  const Routing rt = routing_view(smem, L);
  const int srow = stage_row_bytes(H);
  const int KP = H / 16;
  const int UB = H / 2;
  const int g = lane >> 2, c = lane & 3;
  const int pg = phys_lo(g), pg8 = phys_hi(g);
  const int bpitch = 2 * I + 64;

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], W);
    }
    for (int r = 0; r < RS; ++r) {
      mbar_init(&rfull[r], W);
      mbar_init(&rfree[r], 1);
    }
    mbar_fence_init();
  }
  // x and topk_ids come from earlier kernels.
  pdl_wait();
  route_decode(a, rt);  // ends with __syncthreads (also publishes the barrier inits)
  const int D = rt.misc[0];
  const int tiles = I / 8;
  const int n_units = (D + a.has_shared) * tiles;
  const int stride = gridDim.x, first = blockIdx.x;
  const int my_units = first < n_units ? (n_units - first + stride - 1) / stride : 0;

  auto unit_routes = [&](int u) {
    UnitRoutes ur;
    ur.d = u / tiles;
    ur.shared = ur.d >= D;
    const int n = ur.shared ? M : rt.cnt_of[ur.d];
    ur.n = n < 8 * NT ? n : 8 * NT;
    return ur;
  };
  auto expert_w = [&](int d) -> const uint8_t* {
    return d < D ? a.w13 + (size_t)rt.exp_of[d] * (2 * I) * UB : a.sh_w13;
  };
  auto expert_s = [&](int d) -> const uint8_t* {
    return d < D ? a.s13 + (size_t)rt.exp_of[d] * (2 * I) * KP : a.sh_s13;
  };
  // weight row of physical row r: 0..7 up rows, 8..15 the matching gate rows
  auto wrow = [&](int tile, int r) { return r < 8 ? tile * 8 + r : I + tile * 8 + (r - 8); };

  auto issue = [&](int i) {
    const uint64_t pol = policy_evict_first();
    const int u = first + i * stride;
    const int s = i % NS;
    const int d = u / tiles, tile = u - d * tiles;
    const uint8_t* wq = expert_w(d);
    if (lane == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)(16 * UB));
    __syncwarp();
    if (lane < 2)  // two contiguous 8-row blocks: up rows, gate rows
      bulk_g2s(stages + (size_t)s * L.stage_bytes + tile_row_offset(8 * lane, UB),
               wq + (size_t)wrow(tile, 8 * lane) * UB, (uint32_t)(8 * UB), &full[s], pol);
  };

  if (warp == 0) {
    const int pre = my_units < NS ? my_units : NS;
    for (int i = 0; i < pre; ++i) issue(i);
  }
  stage_rows<W_NVFP4>(xs, unscale, M, H, [&](int r) {
    return reinterpret_cast<const __nv_bfloat16*>(a.x) + (size_t)r * a.ldx;
  });
  __syncthreads();

  if (warp == 0) {
    int issued = my_units < NS ? my_units : NS;
    for (int i = NS; i < my_units; ++i) {
      if (!mbar_wait(&empty[i % NS], ((i / NS) & 1) ^ 1)) {
        record_error(a.err, ERR_WAIT_EMPTY);
        break;
      }
      issue(i);
      issued = i + 1;
    }
    for (int j = issued > NS ? issued - NS : 0; j < issued; ++j)
      if (!mbar_wait(&full[j % NS], (j / NS) & 1)) record_error(a.err, ERR_DRAIN);
  } else if (warp >= 2) {
    const int cw = warp - 2;  // k slice of the unit
    const uint64_t pol = policy_evict_first();
    uint32_t sa[CPW], sb[CPW], na[CPW], nb[CPW];
    float gsc = 0.f, ngsc = 0.f;
    auto prefetch = [&](int i, uint32_t(&xa)[CPW], uint32_t(&xb)[CPW], float& gs) {
      const int u = first + i * stride;
      const int d = u / tiles, tile = u - d * tiles;
      const uint8_t* sf = expert_s(d);
      const int ra = wrow(tile, pg), rb = wrow(tile, pg8);
#pragma unroll
      for (int cc = 0; cc < CPW; ++cc) {
        const int kb = (cw * CPW + cc) * 8 + c * 2;
        xa[cc] = ldg_u16_stream(sf + scale_offset(a.swizzled, ra, kb, KP), pol);
        xb[cc] = ldg_u16_stream(sf + scale_offset(a.swizzled, rb, kb, KP), pol);
      }
      if (cw == 0 && lane == 0)
        gs = d < D ? __ldg(a.g13 + (size_t)rt.exp_of[d] * a.g13_stride) : __ldg(a.sh_g13);
    };
    if (my_units > 0) prefetch(0, sa, sb, gsc);
    for (int i = 0; i < my_units; ++i) {
      const int u = first + i * stride;
      const UnitRoutes ur = unit_routes(u);
      if (i + 1 < my_units) prefetch(i + 1, na, nb, ngsc);
      int tok[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int sl = nt * 8 + g;
        tok[nt] = sl < ur.n ? token_of(slot_entry(rt, ur, sl), R) : -1;
      }
      const int s = i % NS;
      if (!mbar_wait(&full[s], (i / NS) & 1)) {
        record_error(a.err, ERR_WAIT_FULL);
        break;
      }
      const uint8_t* st = stages + (size_t)s * L.stage_bytes;
      const uint8_t* rowa = st + tile_row_offset(pg, UB) + c * 16;
      const uint8_t* rowb = st + tile_row_offset(pg8, UB) + c * 16;
      float acc[2][NT][4];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int r = 0; r < 4; ++r) acc[h][nt][r] = 0.f;
#pragma unroll
      for (int cc = 0; cc < CPW; ++cc) {
        const int ch = cw * CPW + cc;
        const uint4 va = lds128(rowa + ch * 64);
        const uint4 vb = lds128(rowb + ch * 64);
        uint4 xf[NT][Q];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int q = 0; q < Q; ++q)
            xf[nt][q] = tok[nt] >= 0
                            ? lds128(xs + (size_t)tok[nt] * srow + ((ch * Q + q) * 4 + c) * 16)
                            : make_uint4(0u, 0u, 0u, 0u);
        chunk_mma<W_NVFP4, NT>(acc[0], acc[1], va, vb, sa[cc], sb[cc], xf, ur.n > 8 ? 2 : 1);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      const int rs = i % RS;
      if (!mbar_wait(&rfree[rs], ((i / RS) & 1) ^ 1)) {
        record_error(a.err, ERR_WAIT_RFREE);
        break;
      }
      float* dst = red + ((size_t)(rs * W + cw) * 32 + lane) * NT * 4;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        *reinterpret_cast<float4*>(dst + nt * 4) =
            make_float4(acc[0][nt][0] + acc[1][nt][0], acc[0][nt][1] + acc[1][nt][1],
                        acc[0][nt][2] + acc[1][nt][2], acc[0][nt][3] + acc[1][nt][3]);
      if (cw == 0 && lane == 0) sred[rs * 64] = gsc;
      __syncwarp();
      if (lane == 0) mbar_arrive(&rfull[rs]);
#pragma unroll
      for (int cc = 0; cc < CPW; ++cc) {
        sa[cc] = na[cc];
        sb[cc] = nb[cc];
      }
      gsc = ngsc;
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    for (int i = 0; i < my_units; ++i) {
      const int u = first + i * stride;
      const UnitRoutes ur = unit_routes(u);
      const int tile = u - ur.d * tiles;
      const int rs = i % RS;
      if (!mbar_wait(&rfull[rs], (i / RS) & 1)) {
        record_error(a.err, ERR_WAIT_RED);
        break;
      }
      const float gs = sred[rs * 64];
      float v[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int w = 0; w < W; ++w) {
          const float4 p =
              *reinterpret_cast<const float4*>(red + ((size_t)(rs * W + w) * 32 + lane) * NT * 4 + nt * 4);
          sum.x += p.x;
          sum.y += p.y;
          sum.z += p.z;
          sum.w += p.w;
        }
        v[nt][0] = sum.x;
        v[nt][1] = sum.y;
        v[nt][2] = sum.z;
        v[nt][3] = sum.w;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&rfree[rs]);
      // MMA row g is physical row pg: the up row of column g for even g, the gate row
      // for odd g; MMA row g + 8 is the other one.
      const bool odd = g & 1;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const int sl = nt * 8 + 2 * c + p;
          if (sl >= ur.n) continue;
          const int entry = slot_entry(rt, ur, sl);
          const int t = token_of(entry, R);
          const float us = unscale[t];
          const float upv = (odd ? v[nt][2 + p] : v[nt][p]) * us * gs;
          const float gv = (odd ? v[nt][p] : v[nt][2 + p]) * us * gs;
          reinterpret_cast<__nv_bfloat16*>(a.act)[(size_t)pair_of(entry, R) * I + tile * 8 + g] =
              __float2bfloat16_rn(silu_f32(gv) * upv);
        }
      // The last unit of this expert converts its act rows into k2's B-operand rows
      // (expert-contiguous: row d * 16 + slot).
      __threadfence();
      __syncwarp();
      unsigned prev = 0;
      if (lane == 0) prev = atomicAdd(&a.ecnt[ur.d], 1u);
      prev = __shfl_sync(0xffffffffu, prev, 0);
      if (prev == (unsigned)(tiles - 1)) {
        __threadfence();
        for (int sl = 0; sl < ur.n; ++sl) {
          const int pair = pair_of(slot_entry(rt, ur, sl), R);
          const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(a.act) + (size_t)pair * I;
          float m = 0.f;
          for (int k8 = lane; k8 < I / 8; k8 += 32) m = fmaxf(m, bf16x8_absmax(ldg_cg_u4(src + 8 * k8)));
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          const int e = stage_exponent(m);
          uint8_t* dst = a.act_f16 + (size_t)(ur.d * kSlotCap + sl) * bpitch;
          for (int k8 = lane; k8 < I / 8; k8 += 32)
            *reinterpret_cast<uint4*>(dst + stage_unit_offset<W_NVFP4>(8 * k8)) =
                bf16x8_to_f16x8_scaled(ldg_cg_u4(src + 8 * k8), e);
          if (lane == 0) a.pair_unscale[ur.d * kSlotCap + sl] = pow2f(-e);
        }
        if (lane == 0) a.ecnt[ur.d] = 0u;
      }
    }
  }
  pdl_trigger();
}

// ------------------------------------------------------------------------------------
// k2: out[t, n] = sum_r w_{t,r} * g2_{e_r} * <W2[e_r, n], act_{t,r}>  (+ shared expert)
// ------------------------------------------------------------------------------------
template <int NT, int CPW>
__global__ void __launch_bounds__(kDenseThreadsMax, 1) moe_down_kernel(const MoeArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int Q = Geo<W_NVFP4>::Q;
  constexpr int kMaxRT = 4;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int M = a.M, R = a.R, H = a.H, I = a.I, W = a.W, NS = a.NS, RS = a.RS;
  const int RT = a.RT;  // 16-row tiles per unit (16 * RT rows of H)
  const int KSL = W / RT;
  const MoeLayout L = moe_layout(2, M, R, a.E, H, I, W, NS, RS, NT, RT);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + NS;
  uint64_t* rfull = empty + NS;
  uint64_t* rfree = rfull + RS;
  uint8_t* stages = smem + L.stages;
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* sred = red + RS * W * 32 * NT * 4;
  const Routing rt = routing_view(smem, L);
  const int KP = I / 16;
  const int UB = I / 2;
  const int g = lane >> 2, c = lane & 3;
  const int pg = phys_lo(g), pg8 = phys_hi(g);

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], W);
    }
    for (int r = 0; r < RS; ++r) {
      mbar_init(&rfull[r], W);
      mbar_init(&rfree[r], 1);
    }
    mbar_fence_init();
  }
  // topk_ids were written before k1 started, and k1 lets this grid launch only after
  // its own griddepcontrol.wait, so they are visible here; act_f16 is read after
  // this kernel's pdl_wait().
  route_decode(a, rt);
  const int D = rt.misc[0];
  const int Dtot = D + a.has_shared;
  const int groups = H / (16 * RT);
  const int n_units = Dtot * groups;
  const int stride = gridDim.x, first = blockIdx.x;
  const int my_units = first < n_units ? (n_units - first + stride - 1) / stride : 0;
  if (Dtot == 0) {  // every route skipped: the layer output is zero
    pdl_wait();
    for (int o = blockIdx.x * blockDim.x + tid; o < M * H; o += gridDim.x * blockDim.x) {
      const int t = o / H, n = o - t * H;
      if (a.out_f32)
        reinterpret_cast<float*>(a.out)[(size_t)t * a.ldo + n] = 0.f;
      else
        reinterpret_cast<__nv_bfloat16*>(a.out)[(size_t)t * a.ldo + n] = __float2bfloat16_rn(0.f);
    }
    pdl_trigger();
    return;
  }

  auto unit_routes = [&](int u) {
    UnitRoutes ur;
    ur.d = u / groups;
    ur.shared = ur.d >= D;
    const int n = ur.shared ? M : rt.cnt_of[ur.d];
    ur.n = n < 8 * NT ? n : 8 * NT;
    return ur;
  };
  auto expert_w = [&](int d) -> const uint8_t* {
    return d < D ? a.w2 + (size_t)rt.exp_of[d] * H * UB : a.sh_w2;
  };
  auto expert_s = [&](int d) -> const uint8_t* {
    return d < D ? a.s2 + (size_t)rt.exp_of[d] * H * KP : a.sh_s2;
  };

  // Weight blocks of stage i (valid before k1 completes) and its B rows (after pdl_wait).
  auto issue_weights = [&](int i, int brows) {
    const uint64_t pol = policy_evict_first();
    const int u = first + i * stride;
    const int s = i % NS;
    const int d = u / groups, grp = u - d * groups;
    const uint8_t* wq = expert_w(d) + (size_t)grp * RT * 16 * UB;
    if (lane == 0)
      mbar_arrive_expect_tx(&full[s], (uint32_t)(RT * 16 * UB + brows * L.bpitch));
    __syncwarp();
    if (lane < 2 * RT)  // tile lane/2, half lane%2: 8 contiguous rows
      bulk_g2s(stages + (size_t)s * L.stage_bytes + (lane >> 1) * L.wpitch +
                   tile_row_offset(8 * (lane & 1), UB),
               wq + (size_t)(lane * 8) * UB, (uint32_t)(8 * UB), &full[s], pol);
  };
  auto issue_brows = [&](int i) {
    const uint64_t pol = policy_evict_first();
    const int u = first + i * stride;
    const int s = i % NS;
    const UnitRoutes ur = unit_routes(u);
    if (lane == 0 && ur.n > 0)
      bulk_g2s(stages + (size_t)s * L.stage_bytes + L.brow0,
               a.act_f16 + (size_t)(ur.d * kSlotCap) * L.bpitch, (uint32_t)(ur.n * L.bpitch),
               &full[s], pol);
  };

  const int pre = my_units < NS ? my_units : NS;
  if (warp == 0)
    for (int i = 0; i < pre; ++i) issue_weights(i, unit_routes(first + i * stride).n);
  pdl_wait();
  __syncthreads();

  if (warp == 0) {
    for (int i = 0; i < pre; ++i) issue_brows(i);
    int issued = pre;
    for (int i = NS; i < my_units; ++i) {
      if (!mbar_wait(&empty[i % NS], ((i / NS) & 1) ^ 1)) {
        record_error(a.err, ERR_WAIT_EMPTY);
        break;
      }
      issue_weights(i, unit_routes(first + i * stride).n);
      issue_brows(i);
      issued = i + 1;
    }
    for (int j = issued > NS ? issued - NS : 0; j < issued; ++j)
      if (!mbar_wait(&full[j % NS], (j / NS) & 1)) record_error(a.err, ERR_DRAIN);
  } else if (warp >= 2) {
    const int cw = warp - 2;
    const int rtile = cw / KSL, kq = cw - rtile * KSL;
    const bool factor_warp = cw == 0;  // hands the unit's per-route factors over
    const uint64_t pol = policy_evict_first();
    uint32_t sa[CPW], sb[CPW], na[CPW], nb[CPW];
    float fac = 0.f, nfac = 0.f;
    auto prefetch = [&](int i, uint32_t(&xa)[CPW], uint32_t(&xb)[CPW], float& f) {
      const int u = first + i * stride;
      const int d = u / groups, grp = u - d * groups;
      const uint8_t* sf = expert_s(d);
      const int base = (grp * RT + rtile) * 16;
      const int ra = base + pg, rb = base + pg8;
#pragma unroll
      for (int cc = 0; cc < CPW; ++cc) {
        const int kb = (kq * CPW + cc) * 8 + c * 2;
        xa[cc] = ldg_u16_stream(sf + scale_offset(a.swizzled, ra, kb, KP), pol);
        xb[cc] = ldg_u16_stream(sf + scale_offset(a.swizzled, rb, kb, KP), pol);
      }
      if (factor_warp) {  // lane s: factor of route slot s = act unscale * g2 * weight
        const UnitRoutes ur = unit_routes(u);
        if (lane < ur.n) {
          const int entry = slot_entry(rt, ur, lane);
          const float g2 = d < D ? __ldg(a.g2 + (size_t)rt.exp_of[d] * a.g2_stride) : __ldg(a.sh_g2);
          const float wr = entry < 0 ? 1.f : __ldg(a.wts + entry);
          f = __ldcg(a.pair_unscale + d * kSlotCap + lane) * (g2 * wr);
        }
      }
    };
    if (my_units > 0) prefetch(0, sa, sb, fac);
    for (int i = 0; i < my_units; ++i) {
      const int u = first + i * stride;
      const UnitRoutes ur = unit_routes(u);
      if (i + 1 < my_units) prefetch(i + 1, na, nb, nfac);
      const int s = i % NS;
      if (!mbar_wait(&full[s], (i / NS) & 1)) {
        record_error(a.err, ERR_WAIT_FULL);
        break;
      }
      const uint8_t* st = stages + (size_t)s * L.stage_bytes;
      const uint8_t* wst = st + (size_t)rtile * L.wpitch;
      const uint8_t* rowa = wst + tile_row_offset(pg, UB) + c * 16;
      const uint8_t* rowb = wst + tile_row_offset(pg8, UB) + c * 16;
      const uint8_t* bst = st + L.brow0;
      float acc[2][NT][4];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int r = 0; r < 4; ++r) acc[h][nt][r] = 0.f;
#pragma unroll
      for (int cc = 0; cc < CPW; ++cc) {
        const int ch = kq * CPW + cc;
        const uint4 va = lds128(rowa + ch * 64);
        const uint4 vb = lds128(rowb + ch * 64);
        uint4 xf[NT][Q];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int sl = nt * 8 + g;
#pragma unroll
          for (int q = 0; q < Q; ++q)
            xf[nt][q] = sl < ur.n ? lds128(bst + (size_t)sl * L.bpitch + ((ch * Q + q) * 4 + c) * 16)
                                  : make_uint4(0u, 0u, 0u, 0u);
        }
        chunk_mma<W_NVFP4, NT>(acc[0], acc[1], va, vb, sa[cc], sb[cc], xf, ur.n > 8 ? 2 : 1);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      const int rs = i % RS;
      if (!mbar_wait(&rfree[rs], ((i / RS) & 1) ^ 1)) {
        record_error(a.err, ERR_WAIT_RFREE);
        break;
      }
      float* dst = red + ((size_t)(rs * W + cw) * 32 + lane) * NT * 4;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        *reinterpret_cast<float4*>(dst + nt * 4) =
            make_float4(acc[0][nt][0] + acc[1][nt][0], acc[0][nt][1] + acc[1][nt][1],
                        acc[0][nt][2] + acc[1][nt][2], acc[0][nt][3] + acc[1][nt][3]);
      if (factor_warp && lane < ur.n) sred[rs * 64 + lane] = fac;
      __syncwarp();
      if (lane == 0) mbar_arrive(&rfull[rs]);
#pragma unroll
      for (int cc = 0; cc < CPW; ++cc) {
        sa[cc] = na[cc];
        sb[cc] = nb[cc];
      }
      fac = nfac;
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    for (int i = 0; i < my_units; ++i) {
      const int u = first + i * stride;
      const UnitRoutes ur = unit_routes(u);
      const int grp = u - ur.d * groups;
      const int rs = i % RS;
      if (!mbar_wait(&rfull[rs], (i / RS) & 1)) {
        record_error(a.err, ERR_WAIT_RED);
        break;
      }
      float sc[NT][2];
      int pr[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const int sl = nt * 8 + 2 * c + p;
          const bool live = sl < ur.n;
          pr[nt][p] = live ? pair_of(slot_entry(rt, ur, sl), R) : -1;
          sc[nt][p] = live ? sred[rs * 64 + sl] : 0.f;
        }
      float v[kMaxRT][NT][4];
#pragma unroll
      for (int r4 = 0; r4 < kMaxRT; ++r4) {
        if (r4 >= RT) break;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int kq = 0; kq < KSL; ++kq) {
            const float4 p = *reinterpret_cast<const float4*>(
                red + ((size_t)(rs * W + r4 * KSL + kq) * 32 + lane) * NT * 4 + nt * 4);
            sum.x += p.x;
            sum.y += p.y;
            sum.z += p.z;
            sum.w += p.w;
          }
          v[r4][nt][0] = sum.x;
          v[r4][nt][1] = sum.y;
          v[r4][nt][2] = sum.z;
          v[r4][nt][3] = sum.w;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&rfree[rs]);
#pragma unroll
      for (int r4 = 0; r4 < kMaxRT; ++r4) {
        if (r4 >= RT) break;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int p = 0; p < 2; ++p) {
            if (pr[nt][p] < 0) continue;
            float* dst = a.part + (size_t)pr[nt][p] * H + (grp * RT + r4) * 16;
            st_cg_f32(dst + pg, v[r4][nt][p] * sc[nt][p]);
            st_cg_f32(dst + pg8, v[r4][nt][2 + p] * sc[nt][p]);
          }
      }
      __threadfence();
      __syncwarp();
      unsigned prev = 0;
      if (lane == 0) prev = atomicAdd(&a.cnt[grp], 1u);
      prev = __shfl_sync(0xffffffffu, prev, 0);
      if (prev == (unsigned)(Dtot - 1)) {
        // every expert of this 64-row group is in: sum each token's routes in route
        // order, then the shared expert, round once
        __threadfence();
        for (int o = lane; o < M * RT * 16; o += 32) {
          const int t = o / (RT * 16), n = grp * RT * 16 + (o - t * RT * 16);
          float sum = 0.f;
          for (int r = 0; r < R; ++r)
            if (rt.ids[t * R + r] >= 0) sum += ld_cg_f32(a.part + (size_t)(t * (R + 1) + r) * H + n);
          if (a.has_shared) sum += ld_cg_f32(a.part + (size_t)(t * (R + 1) + R) * H + n);
          if (a.out_f32)
            reinterpret_cast<float*>(a.out)[(size_t)t * a.ldo + n] = sum;
          else
            reinterpret_cast<__nv_bfloat16*>(a.out)[(size_t)t * a.ldo + n] = __float2bfloat16_rn(sum);
        }
        if (lane == 0) a.cnt[grp] = 0u;
      }
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
  if (nt == 1) return cpw == 1 ? moe_down_kernel<1, 1> : cpw == 2 ? moe_down_kernel<1, 2> : cpw == 4 ? moe_down_kernel<1, 4> : nullptr;
  if (nt == 2) return cpw == 1 ? moe_down_kernel<2, 1> : cpw == 2 ? moe_down_kernel<2, 2> : cpw == 4 ? moe_down_kernel<2, 4> : nullptr;
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
  return launch_with_pdl((const void*)k, a, grid, (a.W + 2) * 32, smem, a.pdl, stream);
}

int launch_moe_down(const MoeArgs& a, int nt, int grid, size_t smem, cudaStream_t stream) {
  MoeKernel k = moe_down_ptr(nt, a.CPW);
  if (!k) return 1;
  if (!prepare_kernel((const void*)k)) return 2;
  return launch_with_pdl((const void*)k, a, grid, (a.W + 2) * 32, smem, a.pdl, stream);
}

}  // namespace fnx
