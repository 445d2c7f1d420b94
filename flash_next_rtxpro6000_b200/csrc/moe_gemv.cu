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
// Routing table.  Every CTA decodes topk_ids itself (a 512-bit expert bitmap, a prefix
// count, and per distinct expert the list of routes that chose it, in route order),
// which costs a few hundred cycles and no extra launch.  Each distinct expert's rows are
// then streamed ONCE for all tokens routed to it: the tokens are the B operand of the
// tensor-core MMA, so verify widths cost D distinct experts, not M * top_k routes.
// Route ids < 0 (and ids outside this launch's expert slice) are skipped
// (0112-...patch:205, :259).
//
// k1 unit: (distinct expert, 8 columns of I): MMA rows 0..7 are up rows, 8..15 the
// matching gate rows, so one lane holds both and applies silu(gate * g) * (up * g)
// (0112-...patch:220-224) before rounding act to bf16.
// k2 unit: (distinct expert, 16 rows of H): contribution = <W2 row, act> * (g2 * w_r)
// (0112-...patch:268-269) written as an fp32 partial per (token, route); the last unit
// to finish a row tile sums each token's routes in route order (then the shared expert)
// and rounds once to bf16: deterministic, no float atomics.
#include "fnx_common.cuh"
#include "fnx_kernels.h"

namespace fnx {

namespace {

constexpr int kSlotCap = 16;  // routes per distinct expert handled by one unit (M <= 16)

struct MoeSmem {
  int xs, unscale, red, flags, ids, bitmap, wbase, exp_of, cnt_of, ent, misc, total;
};

__host__ __device__ inline int align_up(int v, int a) { return (v + a - 1) / a * a; }

// Shared-memory layout of both MoE kernels.  `rows` staged rows of `K` elements.
__host__ __device__ inline MoeSmem moe_smem_layout(int rows, int K, int M, int R, int E, int W,
                                                   int G, int NT) {
  MoeSmem s;
  const int nw = (E + 31) / 32;
  const int dcap = (E < M * R ? E : M * R) + 1;
  int off = 0;
  s.xs = off;
  off += rows * stage_row_bytes(K);
  s.unscale = off;
  off += align_up(rows, 4) * 4;
  s.red = off;
  off += G * 2 * W * 32 * NT * 16;
  s.flags = off;
  off += align_up(G, 4) * 4;
  s.ids = off;
  off += align_up(M * R, 4) * 4;
  s.bitmap = off;
  off += align_up(nw, 4) * 4;
  s.wbase = off;
  off += align_up(nw, 4) * 4;
  s.exp_of = off;
  off += align_up(dcap, 4) * 4;
  s.cnt_of = off;
  off += align_up(dcap, 4) * 4;
  s.ent = off;
  off += align_up(dcap * kSlotCap * 2, 16);
  s.misc = off;
  off += 16;
  s.total = off;
  return s;
}

struct Routing {
  int* ids;          // [M*R] local expert id or -1
  uint32_t* bitmap;  // [nw]
  int* wbase;        // [nw]
  int* exp_of;       // [dcap] local expert id of distinct slot d (ascending)
  int* cnt_of;       // [dcap] routes of slot d
  short* ent;        // [dcap][16] route entries (t * R + r), ascending
  int* misc;         // misc[0] = D (distinct routed experts)
};

__device__ inline Routing routing_view(uint8_t* smem, const MoeSmem& L) {
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
  // Distinct experts in ascending id order.
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
  // Route list of every distinct expert, in route order (one warp per expert).
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

}  // namespace

// ------------------------------------------------------------------------------------
// k1: act[t*(R+1)+r, j] = bf16(silu(g * <gate_j, x_t>) * g * <up_j, x_t>)
// ------------------------------------------------------------------------------------
template <int NT, int CPW, int S>
__global__ void __launch_bounds__(512, 1) moe_up_kernel(const MoeArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int W = a.W;
  const int grp = warp / W, wig = warp - grp * W;
  const int gthreads = W * 32, gtid = tid - grp * gthreads;
  const int g = lane >> 2, c = lane & 3;
  const int M = a.M, R = a.R, H = a.H, I = a.I;
  const MoeSmem L = moe_smem_layout(M, H, M, R, a.E, W, a.G, NT);
  uint8_t* xs = smem + L.xs;
  float* unscale = reinterpret_cast<float*>(smem + L.unscale);
  float* red = reinterpret_cast<float*>(smem + L.red);
  const Routing rt = routing_view(smem, L);
  const int srow = stage_row_bytes(H);
  const int KP = H / 16;
  const uint64_t pol = policy_evict_first();

  // x and topk_ids come from earlier kernels.
  pdl_wait();
  route_decode(a, rt);
  const int D = rt.misc[0];
  const int tiles = I / 8;
  const int n_units = (D + a.has_shared) * tiles;
  const int stride = gridDim.x * a.G;
  const int first = blockIdx.x * a.G + grp;

  auto expert_ptrs = [&](int d, const uint8_t*& wq, const uint8_t*& sf) {
    if (d < D) {
      const int e = rt.exp_of[d];
      wq = a.w13 + (size_t)e * (2 * I) * (H / 2);
      sf = a.s13 + (size_t)e * (2 * I) * KP;
    } else {
      wq = a.sh_w13;
      sf = a.sh_s13;
    }
  };

  WeightRing<CPW, S> ring;
  auto load = [&](int u, uint4(&va)[CPW], uint4(&vb)[CPW], uint32_t(&sa)[CPW],
                  uint32_t(&sb)[CPW]) {
    const int d = u / tiles, tile = u - d * tiles;
    const uint8_t *wq, *sf;
    expert_ptrs(d, wq, sf);
    const int ra = tile * 8 + g;      // up row
    const int rb = I + tile * 8 + g;  // gate row
#pragma unroll
    for (int cc = 0; cc < CPW; ++cc) {
      const int chunk = wig * CPW + cc;
      const int off = chunk * 64 + c * 16;
      va[cc] = ldg_stream(wq + (size_t)ra * (H / 2) + off, pol);
      vb[cc] = ldg_stream(wq + (size_t)rb * (H / 2) + off, pol);
      const int kb = chunk * 8 + c * 2;
      sa[cc] = ldg_u16_stream(sf + scale_offset(a.swizzled, ra, kb, KP), pol);
      sb[cc] = ldg_u16_stream(sf + scale_offset(a.swizzled, rb, kb, KP), pol);
    }
  };

  auto process = [&](int u, const uint4(&va)[CPW], const uint4(&vb)[CPW],
                     const uint32_t(&sa)[CPW], const uint32_t(&sb)[CPW], int it) {
    const int d = u / tiles, tile = u - d * tiles;
    const bool shared = d >= D;
    const int n_e = shared ? M : rt.cnt_of[d];
    // Token of B column slot (nt * 8 + g).
    int tok[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int s = nt * 8 + g;
      tok[nt] = (s < n_e) ? (shared ? s : rt.ent[d * kSlotCap + s] / R) : -1;
    }
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[nt][r] = 0.f;
#pragma unroll
    for (int cc = 0; cc < CPW; ++cc) {
      const int chunk = wig * CPW + cc;
      uint4 xf[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int q = 0; q < 4; ++q)
          xf[nt][q] = (tok[nt] >= 0)
                          ? *reinterpret_cast<const uint4*>(xs + (size_t)tok[nt] * srow +
                                                            ((chunk * 4 + q) * 4 + c) * 16)
                          : make_uint4(0u, 0u, 0u, 0u);
      chunk_mma<W_NVFP4, NT>(acc, va[cc], vb[cc], sa[cc], sb[cc], xf, n_e > 8 ? 2 : 1);
    }
    float* rbuf = red + (size_t)((grp * 2 + (it & 1)) * W) * 32 * NT * 4;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
      *reinterpret_cast<float4*>(rbuf + ((size_t)(wig * 32 + lane) * NT + nt) * 4) =
          make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]);
    group_sync(1 + grp, gthreads);

    // gtid = slot * 16 + i; rows 0..7 up, 8..15 gate (gthreads >= 256).
    const int slot = gtid >> 4, i = gtid & 15;
    const bool live = slot < n_e;
    float rowsum = 0.f;
    if (live) {
      const int nt = slot >> 3, col = slot & 7;
      const int src = (i & 7) * 4 + (col >> 1);
      const int reg = ((i >> 3) << 1) | (col & 1);
      for (int w = 0; w < W; ++w) rowsum += rbuf[((size_t)(w * 32 + src) * NT + nt) * 4 + reg];
    }
    const float gate = __shfl_down_sync(0xffffffffu, rowsum, 8);
    if (live && i < 8) {
      int t, pair;
      if (shared) {
        t = slot;
        pair = t * (R + 1) + R;
      } else {
        const int entry = rt.ent[d * kSlotCap + slot];
        t = entry / R;
        pair = entry + t;
      }
      const float gs = shared ? __ldg(a.sh_g13) : __ldg(a.g13 + (size_t)rt.exp_of[d] * a.g13_stride);
      const float us = unscale[t];
      const float upv = rowsum * us * gs;
      const float gv = gate * us * gs;
      reinterpret_cast<__nv_bfloat16*>(a.act)[(size_t)pair * I + tile * 8 + i] =
          __float2bfloat16_rn(silu_f32(gv) * upv);
    }
  };

#pragma unroll
  for (int s = 0; s < S - 1; ++s) {
    const int u = first + s * stride;
    if (u < n_units) load(u, ring.va[s], ring.vb[s], ring.sa[s], ring.sb[s]);
  }
  stage_rows<W_NVFP4>(xs, unscale, M, H, [&](int r) {
    return reinterpret_cast<const __nv_bfloat16*>(a.x) + (size_t)r * a.ldx;
  });
  __syncthreads();

  int it = 0;
  for (int base = first; base < n_units; base += S * stride) {
#pragma unroll
    for (int s = 0; s < S; ++s) {
      const int u = base + s * stride;
      if (u >= n_units) break;
      const int un = u + (S - 1) * stride;
      const int nxt = (s + S - 1) % S;
      if (un < n_units) load(un, ring.va[nxt], ring.vb[nxt], ring.sa[nxt], ring.sb[nxt]);
      process(u, ring.va[s], ring.vb[s], ring.sa[s], ring.sb[s], it);
      ++it;
    }
  }
  pdl_trigger();
}

// ------------------------------------------------------------------------------------
// k2: out[t, n] = sum_r w_{t,r} * g2_{e_r} * <W2[e_r, n], act_{t,r}>  (+ shared expert)
// ------------------------------------------------------------------------------------
template <int NT, int CPW, int S>
__global__ void __launch_bounds__(512, 1) moe_down_kernel(const MoeArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int W = a.W;
  const int grp = warp / W, wig = warp - grp * W;
  const int gthreads = W * 32, gtid = tid - grp * gthreads;
  const int g = lane >> 2, c = lane & 3;
  const int M = a.M, R = a.R, H = a.H, I = a.I;
  const int P = M * (R + 1);
  const MoeSmem L = moe_smem_layout(P, I, M, R, a.E, W, a.G, NT);
  uint8_t* xs = smem + L.xs;
  float* unscale = reinterpret_cast<float*>(smem + L.unscale);
  float* red = reinterpret_cast<float*>(smem + L.red);
  int* flags = reinterpret_cast<int*>(smem + L.flags);
  const Routing rt = routing_view(smem, L);
  const int srow = stage_row_bytes(I);
  const int KP = I / 16;
  const uint64_t pol = policy_evict_first();

  // topk_ids were written before k1 started and k1 triggers this launch only after its
  // own wait, so they are visible here; act (k1's output) is read after pdl_wait().
  route_decode(a, rt);
  const int D = rt.misc[0];
  const int Dtot = D + a.has_shared;
  const int tiles = H / 16;
  const int n_units = Dtot * tiles;
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
  const int stride = gridDim.x * a.G;
  const int first = blockIdx.x * a.G + grp;

  auto expert_ptrs = [&](int d, const uint8_t*& wq, const uint8_t*& sf) {
    if (d < D) {
      const int e = rt.exp_of[d];
      wq = a.w2 + (size_t)e * H * (I / 2);
      sf = a.s2 + (size_t)e * H * KP;
    } else {
      wq = a.sh_w2;
      sf = a.sh_s2;
    }
  };

  WeightRing<CPW, S> ring;
  auto load = [&](int u, uint4(&va)[CPW], uint4(&vb)[CPW], uint32_t(&sa)[CPW],
                  uint32_t(&sb)[CPW]) {
    const int d = u / tiles, tile = u - d * tiles;
    const uint8_t *wq, *sf;
    expert_ptrs(d, wq, sf);
    const int ra = tile * 16 + g, rb = ra + 8;
#pragma unroll
    for (int cc = 0; cc < CPW; ++cc) {
      const int chunk = wig * CPW + cc;
      const int off = chunk * 64 + c * 16;
      va[cc] = ldg_stream(wq + (size_t)ra * (I / 2) + off, pol);
      vb[cc] = ldg_stream(wq + (size_t)rb * (I / 2) + off, pol);
      const int kb = chunk * 8 + c * 2;
      sa[cc] = ldg_u16_stream(sf + scale_offset(a.swizzled, ra, kb, KP), pol);
      sb[cc] = ldg_u16_stream(sf + scale_offset(a.swizzled, rb, kb, KP), pol);
    }
  };

  auto process = [&](int u, const uint4(&va)[CPW], const uint4(&vb)[CPW],
                     const uint32_t(&sa)[CPW], const uint32_t(&sb)[CPW], int it) {
    const int d = u / tiles, tile = u - d * tiles;
    const bool shared = d >= D;
    const int n_e = shared ? M : rt.cnt_of[d];
    int prow[NT];  // staged act row (pair id) of B column slot nt*8+g
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int s = nt * 8 + g;
      if (s >= n_e) {
        prow[nt] = -1;
      } else if (shared) {
        prow[nt] = s * (R + 1) + R;
      } else {
        const int entry = rt.ent[d * kSlotCap + s];
        prow[nt] = entry + entry / R;
      }
    }
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[nt][r] = 0.f;
#pragma unroll
    for (int cc = 0; cc < CPW; ++cc) {
      const int chunk = wig * CPW + cc;
      uint4 xf[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int q = 0; q < 4; ++q)
          xf[nt][q] = (prow[nt] >= 0)
                          ? *reinterpret_cast<const uint4*>(xs + (size_t)prow[nt] * srow +
                                                            ((chunk * 4 + q) * 4 + c) * 16)
                          : make_uint4(0u, 0u, 0u, 0u);
      chunk_mma<W_NVFP4, NT>(acc, va[cc], vb[cc], sa[cc], sb[cc], xf, n_e > 8 ? 2 : 1);
    }
    float* rbuf = red + (size_t)((grp * 2 + (it & 1)) * W) * 32 * NT * 4;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
      *reinterpret_cast<float4*>(rbuf + ((size_t)(wig * 32 + lane) * NT + nt) * 4) =
          make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]);
    group_sync(1 + grp, gthreads);

    const float g2 = shared ? __ldg(a.sh_g2) : __ldg(a.g2 + (size_t)rt.exp_of[d] * a.g2_stride);
    for (int o = gtid; o < 16 * n_e; o += gthreads) {
      const int slot = o >> 4, i = o & 15;
      const int nt = slot >> 3, col = slot & 7;
      const int src = (i & 7) * 4 + (col >> 1);
      const int reg = ((i >> 3) << 1) | (col & 1);
      float rowsum = 0.f;
      for (int w = 0; w < W; ++w) rowsum += rbuf[((size_t)(w * 32 + src) * NT + nt) * 4 + reg];
      int pair;
      float wr;
      if (shared) {
        pair = slot * (R + 1) + R;
        wr = 1.f;
      } else {
        const int entry = rt.ent[d * kSlotCap + slot];
        pair = entry + entry / R;
        wr = __ldg(a.wts + entry);
      }
      st_cg_f32(a.part + (size_t)pair * H + tile * 16 + i, rowsum * unscale[pair] * (g2 * wr));
    }
    __threadfence();
    group_sync(1 + grp, gthreads);
    if (gtid == 0) {
      const unsigned prev = atomicAdd(&a.cnt[tile], 1u);
      flags[grp] = (prev == (unsigned)(Dtot - 1));
    }
    group_sync(1 + grp, gthreads);
    if (!flags[grp]) return;
    __threadfence();
    for (int o = gtid; o < 16 * M; o += gthreads) {
      const int t = o >> 4, i = o & 15;
      const int n = tile * 16 + i;
      float s = 0.f;
      for (int r = 0; r < R; ++r)
        if (rt.ids[t * R + r] >= 0) s += ld_cg_f32(a.part + (size_t)(t * (R + 1) + r) * H + n);
      if (a.has_shared) s += ld_cg_f32(a.part + (size_t)(t * (R + 1) + R) * H + n);
      if (a.out_f32)
        reinterpret_cast<float*>(a.out)[(size_t)t * a.ldo + n] = s;
      else
        reinterpret_cast<__nv_bfloat16*>(a.out)[(size_t)t * a.ldo + n] = __float2bfloat16_rn(s);
    }
    if (gtid == 0) a.cnt[tile] = 0u;  // all Dtot arrivals for this tile have happened
  };

  // W2 does not depend on k1: start streaming it before waiting for act.
#pragma unroll
  for (int s = 0; s < S - 1; ++s) {
    const int u = first + s * stride;
    if (u < n_units) load(u, ring.va[s], ring.vb[s], ring.sa[s], ring.sb[s]);
  }
  pdl_wait();
  stage_rows<W_NVFP4>(xs, unscale, P, I, [&](int p) -> const __nv_bfloat16* {
    const int t = p / (R + 1), r = p - t * (R + 1);
    const bool used = (r == R) ? (a.has_shared != 0) : (rt.ids[t * R + r] >= 0);
    return used ? reinterpret_cast<const __nv_bfloat16*>(a.act) + (size_t)p * I : nullptr;
  });
  __syncthreads();

  int it = 0;
  for (int base = first; base < n_units; base += S * stride) {
#pragma unroll
    for (int s = 0; s < S; ++s) {
      const int u = base + s * stride;
      if (u >= n_units) break;
      const int un = u + (S - 1) * stride;
      const int nxt = (s + S - 1) % S;
      if (un < n_units) load(un, ring.va[nxt], ring.vb[nxt], ring.sa[nxt], ring.sb[nxt]);
      process(u, ring.va[s], ring.vb[s], ring.sa[s], ring.sb[s], it);
      ++it;
    }
  }
  pdl_trigger();
}

using MoeKernel = void (*)(const MoeArgs);

MoeKernel moe_up_ptr(int nt, int cpw) {
  if (nt == 1) return cpw == 1 ? moe_up_kernel<1, 1, 4> : (cpw == 2 ? moe_up_kernel<1, 2, 3> : nullptr);
  if (nt == 2) return cpw == 1 ? moe_up_kernel<2, 1, 4> : (cpw == 2 ? moe_up_kernel<2, 2, 3> : nullptr);
  return nullptr;
}

MoeKernel moe_down_ptr(int nt, int cpw) {
  if (nt == 1)
    return cpw == 1 ? moe_down_kernel<1, 1, 4> : (cpw == 2 ? moe_down_kernel<1, 2, 3> : nullptr);
  if (nt == 2)
    return cpw == 1 ? moe_down_kernel<2, 1, 4> : (cpw == 2 ? moe_down_kernel<2, 2, 3> : nullptr);
  return nullptr;
}

int occupancy_of(MoeKernel k, int threads, size_t smem) {
  if (!k || !prepare_kernel((const void*)k)) return 0;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, threads, smem) != cudaSuccess) return 0;
  return n;
}

size_t moe_up_smem(int M, int R, int E, int H, int W, int G, int NT) {
  return (size_t)moe_smem_layout(M, H, M, R, E, W, G, NT).total;
}
size_t moe_down_smem(int M, int R, int E, int I, int W, int G, int NT) {
  return (size_t)moe_smem_layout(M * (R + 1), I, M, R, E, W, G, NT).total;
}

int moe_up_occupancy(int nt, int cpw, int threads, size_t smem) {
  return occupancy_of(moe_up_ptr(nt, cpw), threads, smem);
}
int moe_down_occupancy(int nt, int cpw, int threads, size_t smem) {
  return occupancy_of(moe_down_ptr(nt, cpw), threads, smem);
}

// CPW is fixed by the shapes: k1 streams H / 128 chunks over W warps, k2 I / 128.
int launch_moe_up(const MoeArgs& a, int nt, int grid, size_t smem, cudaStream_t stream) {
  const int chunks = a.H / 128;
  const int cpw = chunks / a.W;
  if (cpw * a.W != chunks) return 1;
  MoeKernel k = moe_up_ptr(nt, cpw);
  if (!k) return 1;
  if (!prepare_kernel((const void*)k)) return 2;
  return launch_with_pdl((const void*)k, a, grid, a.W * a.G * 32, smem, a.pdl, stream);
}

int launch_moe_down(const MoeArgs& a, int nt, int grid, size_t smem, cudaStream_t stream) {
  const int chunks = a.I / 128;
  const int cpw = chunks / a.W;
  if (cpw * a.W != chunks) return 1;
  MoeKernel k = moe_down_ptr(nt, cpw);
  if (!k) return 1;
  if (!prepare_kernel((const void*)k)) return 2;
  return launch_with_pdl((const void*)k, a, grid, a.W * a.G * 32, smem, a.pdl, stream);
}

}  // namespace fnx
