// Dense weight-only GEMV for M <= 16 tokens: y[m, n] = (sum_k W[n, k] x[m, k]) * s[n].
//
// Replaces the reference's Triton kernels
//   _w8a16_gemv_kernel        kernels/sglang/srt/layers/quantization/w8a16_gemv.py:132-322
//   _w8a16_gemv_silu_kernel   w8a16_gemv.py:865-961
//   _w4a16_nvfp4_gemv_kernel  kernels/sglang/srt/layers/quantization/w4a16_nvfp4_gemv.py:122-216
// with one persistent sm_100a kernel family.
//
// Work decomposition.  A work unit is RT 16-row weight tiles (a SiLU tile is 8 gate rows
// plus the matching 8 up rows) over the k range of one split.  Each persistent CTA runs
// three roles:
//   * warp 0, producer: bulk copies (cp.async.bulk, mbarrier completion) of the unit's
//     weight rows (two 8-row blocks per contiguous tile) and cp.async copies of its row
//     scales and NVFP4 block scales into an NS-stage shared-memory ring, all completing
//     on the stage's one mbarrier;
//   * warps E+1 .., consumers: each takes one k slice of one row tile, reads its 64-byte
//     chunks from the stage with conflict-free 128-bit loads, dequantises in registers
//     and runs mma.sync on independent accumulator chains; it then hands the partial
//     tile to an epilogue warp through a reduction slot;
//   * warps 1 .. E, epilogue (units alternate between them): sum the k slices in a fixed
//     order, apply the per-token and per-row scales, round to bf16 (w8a16_gemv.py:92-95)
//     and store; with ksplit > 1 the split's tile sums are published and the last split
//     to arrive sums them in split order and resets the tile counter
//     (w8a16_gemv.py:289-321).
// Roles synchronise only through mbarriers (no CTA-wide barrier in the steady state),
// every wait is bounded (an expired wait records an error code and ends the role), and
// unit positions advance without integer division.
//
// Greedy argmax (fused).  The epilogue builds a 64-bit key of each bf16-rounded logit
// and its global row; the key maximum is the largest logit with the lowest row on ties
// (torch.argmax).  Each lane keeps its running maximum per token in registers; at the
// end the eight lanes of a token combine theirs with shuffles, each CTA does one
// atomicMax per token, and the last CTA decodes and clears the keys.
//
// The kernel is compiled in three modes (DenseMode), each in its own translation unit:
// plain (whole activation rows staged), slice (the grid is a multiple of ksplit and each
// CTA stages only its k split) and norm (the gated RMSNorm of w8a16_gemv_norm_gated on
// the activation load).
#pragma once

#include "fnx_common.cuh"
#include "fnx_kernels.h"

namespace fnx {

template <int WT, int NT, int CPW, int MODE>
__global__ void __launch_bounds__(kDenseThreadsMax, 1) dense_gemv_kernel(const DenseArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int Q = Geo<WT>::Q;
  constexpr int kMaxRT = 4;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int M = a.M, N = a.N, K = a.K;
  const int W = a.W, RT = a.RT, NS = a.NS, E = a.E, UB = a.UB, TILE = a.TILE;
  const int RS = E;        // one reduction slot per epilogue warp
  const int KSL = W / RT;  // consumer warps sharing one row tile (k slices)
  const DenseStage SG = dense_stage(WT == W_NVFP4, RT, TILE, a.nch_u);
  // slice / norm modes: the epilogue unscales each CTA's sums before the split-K fix-up
  // (CTAs that staged different k ranges have their own powers of two)
  constexpr bool kPreUnscale = MODE != DENSE_PLAIN;
  const bool xslice = MODE == DENSE_SLICE || (MODE == DENSE_NORM && a.xslice);
  constexpr int kPerChunk = WT == W_BF16 ? 32 : (WT == W_NVFP4 ? 128 : 64);
  const int kpu = a.nch_u * kPerChunk;  // k extent of one unit
  const int kx = xslice ? kpu : K;      // k extent of the staged activations
  const DenseLayout L = dense_layout(M, kx, W, NS, RS, NT, SG.bytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + NS;
  uint64_t* rfull = empty + NS;
  uint64_t* rfree = rfull + RS;
  uint64_t* xbar = rfree + RS;  // bulk copy of the activation rows
  uint8_t* stages = smem + L.stages;
  uint8_t* xs = smem + L.xs;
  float* unscale = reinterpret_cast<float*>(smem + L.unscale);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* sred = reinterpret_cast<float*>(smem + L.sred);
  const int srow = stage_row_bytes(kx);
  const int ksplit = a.ksplit;
  const int n_units = a.n_units;
  const int stride = gridDim.x;
  const int first = blockIdx.x;
  const int my_units = first < n_units ? (n_units - first + stride - 1) / stride : 0;
  const bool silu = a.silu != 0;
  const bool per_row = a.scale_kind == SCALE_F32_ROW || a.scale_kind == SCALE_BF16_ROW;
  const int esz = a.scale_kind == SCALE_BF16_ROW ? 2 : 4;
  const int g = lane >> 2, c = lane & 3;
  const int pg = phys_lo(g), pg8 = phys_hi(g);  // physical rows of MMA rows g, g + 8

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
  __syncthreads();

  // Weight row of physical row r (0..15) of row tile t; rows past the end read row 0.
  auto row_of = [&](int t, int r, bool& ok) -> int {
    if (silu) {  // rows 0..7 gate, 8..15 up
      const int col = t * 8 + (r & 7);
      ok = col < N;
      return ok ? ((r < 8) ? col : N + col) : 0;
    }
    const int n = t * 16 + r;
    ok = n < N;
    return ok ? n : 0;
  };
  auto whole_tile = [&](int t) { return silu ? (t * 8 + 7 < N) : (t * 16 + 15 < N); };
  const bool contiguous = a.ldw == UB;  // a half tile is one block of 8 rows
  // Row scales are staged when a full tile's 16 (or 2 x 8, SiLU) values are 16-byte
  // aligned blocks; otherwise the consumer reads them from global memory.
  auto staged_scales = [&](int t) {
    if (!per_row || !whole_tile(t)) return false;
    const uintptr_t base = reinterpret_cast<uintptr_t>(a.scale);
    if (silu) return ((base + (size_t)t * 8 * esz) % 16 == 0) && ((base + ((size_t)N + t * 8) * esz) % 16 == 0);
    return (base + (size_t)t * 16 * esz) % 16 == 0;
  };

  // Producer: weights by bulk copy (two 8-row blocks per full contiguous tile, else a
  // copy per row), the unit's scales by cp.async; all complete on full[s].
  auto issue = [&](const UnitCursor& cu) {
    const uint64_t pol = policy_evict_first();
    const int s = cu.s;
    const int tg = cu.q, ks = cu.r;
    uint8_t* st = stages + (size_t)s * SG.bytes;
    if (lane == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)(RT * 16 * UB));
    __syncwarp();
    for (int rt = 0; rt < RT; ++rt) {
      const int t = tg * RT + rt;
      if (contiguous && whole_tile(t)) {
        if (lane < 2) {
          bool ok;
          const int row = row_of(t, lane * 8, ok);
          bulk_g2s(st + rt * TILE + tile_row_offset(lane * 8, UB), a.w + (size_t)row * a.ldw,
                   (uint32_t)(8 * UB), &full[s], pol);
        }
      } else if (lane < 16) {
        bool ok;
        const int row = row_of(t, lane, ok);
        bulk_g2s(st + rt * TILE + tile_row_offset(lane, UB),
                 a.w + (size_t)row * a.ldw + (size_t)ks * UB, (uint32_t)UB, &full[s], pol);
      }
      if (staged_scales(t)) {
        // 16 raw scales: 16 * esz bytes = esz chunks of 16 B (SiLU: 8 gate + 8 up values)
        const uint8_t* sbase = reinterpret_cast<const uint8_t*>(a.scale);
        if (lane < esz) {
          // 16-B chunks per 8 values: one (bf16) or two (fp32)
          const int h = esz == 2 ? lane : lane >> 1, j = esz == 2 ? 0 : lane & 1;
          const size_t first_val = silu ? (size_t)(h ? N + t * 8 : t * 8) : (size_t)t * 16 + 8 * h;
          cp_async16(st + SG.rsoff + rt * 64 + h * 8 * esz + j * 16, sbase + first_val * esz + j * 16);
        }
      }
      if constexpr (WT == W_NVFP4) {
        // e4m3 block scales of this unit's k range: nch_u * 8 bytes per row, 8 at a time
        for (int r = 0; r < 16; ++r) {
          bool ok;
          const int row = row_of(t, r, ok);
          for (int j = lane; j < a.nch_u; j += 32)
            cp_async8(st + SG.bsoff + (rt * 16 + r) * SG.sbr + j * 8,
                      a.bs + (size_t)row * a.ldbs + (size_t)ks * a.nch_u * 8 + j * 8);
        }
      }
    }
    cp_async_arrive(&full[s]);
  };

  // xslice: the grid is a multiple of ksplit, so every unit of this CTA has the k split
  // first % ksplit and only that k range of the activations is staged (and sized).
  const int kb = xslice ? (first % ksplit) * kpu : 0;
  const int ke = xslice ? kb + kpu : K;
  const __nv_bfloat16* xrows = reinterpret_cast<const __nv_bfloat16*>(a.x);
  const bool x_direct = M <= 2;  // rows loaded by the staging warps, no bulk copy
  UnitCursor pc;  // producer position
  pc.init(first, stride, ksplit, NS);
  if (warp == 0) {
    // The weights and scales do not depend on the previous kernel; the activations may.
    // Without programmatic dependent launch the activation rows go first, so that they do
    // not queue behind the weight stages in the copy engine.
    if (lane == 0 && !a.pdl && !x_direct) issue_x_rows(xs, M, kb, ke, xrows, a.ldx, xbar);
    const int pre = my_units < NS ? my_units : NS;
    for (int i = 0; i < pre; ++i, pc.next()) issue(pc);
  }
  pdl_wait();
  if (tid == 0 && a.pdl && !x_direct) issue_x_rows(xs, M, kb, ke, xrows, a.ldx, xbar);
  // The other warps stage the activations meanwhile; the producer never waits for them.
  if (warp > 0) {
    constexpr bool kNorm = MODE == DENSE_NORM && WT != W_NVFP4;
    stage_rows_bulk<WT, kNorm>(xs, unscale, M, kb, ke, xrows, a.ldx, a.norm, xbar, a.err,
                               x_direct, 32, blockDim.x - 32, 1);
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
    // No copy may still be landing when the CTA exits.
    for (int j = issued > NS ? issued - NS : 0; j < issued; ++j)
      if (!mbar_wait(&full[j % NS], (j / NS) & 1)) record_error(a.err, ERR_DRAIN);
  } else if (warp > E) {
    // ---------------------------------------------------------------- consumers
    const int cw = warp - 1 - E;
    const int rt = cw / KSL, kq = cw - rt * KSL;
    const bool scale_lane = per_row && (kq == 0) && (c == 0);  // hands the row scales over
    const int offa = rt * TILE + tile_row_offset(pg, UB) + c * 16;
    const int offb = rt * TILE + tile_row_offset(pg8, UB) + c * 16;
    const int soffa = SG.bsoff + (rt * 16 + pg) * SG.sbr + c * 2;
    const int soffb = SG.bsoff + (rt * 16 + pg8) * SG.sbr + c * 2;
    UnitCursor cu;
    cu.init(first, stride, ksplit, NS);
    int rs = 0, rph = 0;  // reduction slot of this unit and its phase parity
    for (int i = 0; i < my_units; ++i, cu.next()) {
      const int tg = cu.q, ks = cu.r;
      const int t = tg * RT + rt;
      const int s = cu.s;
      if (!mbar_wait(&full[s], cu.ph)) {
        record_error(a.err, ERR_WAIT_FULL);
        break;
      }
      const uint8_t* st = stages + (size_t)s * SG.bytes;
      float r0 = 0.f, r1 = 0.f;
      if (scale_lane) {
        if (staged_scales(t)) {
          const uint8_t* rsb = st + SG.rsoff + rt * 64;
          if (esz == 2) {
            r0 = bf16_bits_to_f32(*reinterpret_cast<const unsigned short*>(rsb + pg * 2));
            r1 = bf16_bits_to_f32(*reinterpret_cast<const unsigned short*>(rsb + pg8 * 2));
          } else {
            r0 = *reinterpret_cast<const float*>(rsb + pg * 4);
            r1 = *reinterpret_cast<const float*>(rsb + pg8 * 4);
          }
        } else {  // ragged last tile or unaligned scales
          bool oka, okb;
          r0 = load_row_scale(a.scale, a.scale_kind, row_of(t, pg, oka));
          r1 = load_row_scale(a.scale, a.scale_kind, row_of(t, pg8, okb));
        }
      }
      const uint8_t* rowa = st + offa;
      const uint8_t* rowb = st + offb;
      const uint8_t* sca = st + soffa;
      const uint8_t* scb = st + soffb;
      constexpr int NC = NT == 1 ? 4 : 2;  // independent accumulator chains
      float acc[NC][NT][4];
#pragma unroll
      for (int h = 0; h < NC; ++h)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int r = 0; r < 4; ++r) acc[h][nt][r] = 0.f;
#pragma unroll
      for (int cc = 0; cc < CPW; ++cc) {
        const int cl = kq * CPW + cc;
        const int ch = xslice ? cl : ks * a.nch_u + cl;  // chunk within the staged x
        const uint4 va = lds128(rowa + cl * 64);
        const uint4 vb = lds128(rowb + cl * 64);
        uint32_t sa = 0, sb = 0;
        if constexpr (WT == W_NVFP4) {
          sa = *reinterpret_cast<const unsigned short*>(sca + cl * 8);
          sb = *reinterpret_cast<const unsigned short*>(scb + cl * 8);
        }
        uint4 xf[NT][Q];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int tk = nt * 8 + g;
#pragma unroll
          for (int q = 0; q < Q; ++q)
            xf[nt][q] = (tk < M) ? lds128(xs + (size_t)tk * srow + ((ch * Q + q) * 4 + c) * 16)
                                 : make_uint4(0u, 0u, 0u, 0u);
        }
        chunk_mma<WT, NT>(acc[(2 * cc) % NC], acc[(2 * cc + 1) % NC], va, vb, sa, sb, xf);
      }
      __syncwarp();  // every lane's reads of the stage are complete
      if (lane == 0) mbar_arrive(&empty[s]);
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
      if (scale_lane) {
        sred[rs * 64 + rt * 16 + pg] = r0;
        sred[rs * 64 + rt * 16 + pg8] = r1;
      }
      __syncwarp();  // orders the lanes' stores before the release
      if (lane == 0) mbar_arrive(&rfull[rs]);
      if (++rs == RS) {
        rs = 0;
        rph ^= 1;
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue warps
    // Epilogue warp e takes units i = e, e + E, ...  Lane L owns the outputs of MMA
    // lane L: physical rows (pg, pg8) x tokens (nt*8 + 2c + {0,1}) of every row tile.
    const int e = warp - 1;
    const float scalar_scale = per_row ? 0.f : load_row_scale(a.scale, a.scale_kind, 0);
    unsigned long long best[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) best[nt][0] = best[nt][1] = 0ull;
    const bool do_argmax = a.am_keys != nullptr;
    UnitCursor cu;  // units e, e + E, ... of this CTA; slot e, parity flipping per unit
    cu.init(first + e * stride, E * stride, ksplit, 1);
    for (int i = e; i < my_units; i += E, cu.next()) {
      const int tg = cu.q, ks = cu.r;
      const int rs = e;
      if (!mbar_wait(&rfull[rs], cu.ph)) {
        record_error(a.err, ERR_WAIT_RED);
        break;
      }
      float v[kMaxRT][NT][4];
      float scl[kMaxRT][2];
#pragma unroll
      for (int rt = 0; rt < kMaxRT; ++rt) {
        if (rt >= RT) break;
        scl[rt][0] = per_row ? sred[rs * 64 + rt * 16 + pg] : scalar_scale;
        scl[rt][1] = per_row ? sred[rs * 64 + rt * 16 + pg8] : scalar_scale;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          // k slices in batches of four independent loads, summed in slice order on two
          // chains (even / odd slices)
          float4 s0 = make_float4(0.f, 0.f, 0.f, 0.f), s1 = s0;
          const float* rbase = red + ((size_t)(rs * W + rt * KSL) * 32 + lane) * NT * 4 + nt * 4;
          for (int k0 = 0; k0 < KSL; k0 += 4) {
            float4 pv[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
              pv[j] = k0 + j < KSL ? *reinterpret_cast<const float4*>(rbase + (size_t)(k0 + j) * 32 * NT * 4)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int j = 0; j < 4; j += 2) {
              s0.x += pv[j].x; s0.y += pv[j].y; s0.z += pv[j].z; s0.w += pv[j].w;
              s1.x += pv[j + 1].x; s1.y += pv[j + 1].y; s1.z += pv[j + 1].z; s1.w += pv[j + 1].w;
            }
          }
          v[rt][nt][0] = s0.x + s1.x;
          v[rt][nt][1] = s0.y + s1.y;
          v[rt][nt][2] = s0.z + s1.z;
          v[rt][nt][3] = s0.w + s1.w;
          if constexpr (kPreUnscale) {
            // times this CTA's power-of-two unscale of each token (exact), so the split
            // sums are published unscaled; 0 for the padding tokens
            const int tok = nt * 8 + 2 * c;
            const float u0 = tok < M ? unscale[tok] : 0.f;
            const float u1 = tok + 1 < M ? unscale[tok + 1] : 0.f;
            v[rt][nt][0] *= u0;
            v[rt][nt][1] *= u1;
            v[rt][nt][2] *= u0;
            v[rt][nt][3] *= u1;
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&rfree[rs]);

      bool finish = true;
      if (ksplit > 1) {
        // Split-K fix-up: publish this split's tile sums; the last split sums them in
        // split order and resets the counter.
        float* wsp = a.ws + ((size_t)tg * ksplit + ks) * RT * 256;
#pragma unroll
        for (int rt = 0; rt < kMaxRT; ++rt) {
          if (rt >= RT) break;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int r = 0; r < 4; ++r) st_cg_f32(wsp + rt * 256 + (nt * 4 + r) * 32 + lane, v[rt][nt][r]);
        }
        __threadfence();
        __syncwarp();
        unsigned prev = 0;
        if (lane == 0) prev = atomicAdd(&a.ws_cnt[tg], 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        finish = prev == (unsigned)(ksplit - 1);
        if (finish) {
          __threadfence();
#pragma unroll
          for (int rt = 0; rt < kMaxRT; ++rt) {
            if (rt >= RT) break;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int r = 0; r < 4; ++r) {
                float acc = 0.f;
                const float* base = a.ws + (size_t)tg * ksplit * RT * 256 + rt * 256 + (nt * 4 + r) * 32 + lane;
                for (int k2 = 0; k2 < ksplit; ++k2) acc += ld_cg_f32(base + (size_t)k2 * RT * 256);
                v[rt][nt][r] = acc;
              }
          }
          if (lane == 0) a.ws_cnt[tg] = 0u;
        }
      }

      if (finish) {
#pragma unroll
        for (int rt = 0; rt < kMaxRT; ++rt) {
          if (rt >= RT) break;
          const int t = tg * RT + rt;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
            for (int p = 0; p < 2; ++p) {
              const int tok = nt * 8 + 2 * c + p;
              const bool tok_ok = tok < M;
              const float us = !tok_ok ? 0.f : (kPreUnscale ? 1.f : unscale[tok]);
              if (silu) {
                // physical rows < 8 are gate, >= 8 up; both hold column t*8 + g
                const int n = t * 8 + g;
                if (tok_ok && n < N) {
                  const bool odd = g & 1;  // MMA row g is the up row for odd g
                  const float gsum = odd ? v[rt][nt][2 + p] : v[rt][nt][p];
                  const float usum = odd ? v[rt][nt][p] : v[rt][nt][2 + p];
                  const float gsc = odd ? scl[rt][1] : scl[rt][0];
                  const float usc = odd ? scl[rt][0] : scl[rt][1];
                  reinterpret_cast<__nv_bfloat16*>(a.y)[(size_t)tok * a.ldy + n] =
                      __float2bfloat16_rn(silu_f32(gsum * us * gsc) * (usum * us * usc));
                }
                continue;
              }
              unsigned long long key = 0ull;
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int n = t * 16 + (h ? pg8 : pg);
                if (!(tok_ok && n < N)) continue;
                const __nv_bfloat16 o = __float2bfloat16_rn(v[rt][nt][2 * h + p] * us * scl[rt][h]);
                void* dst = a.y;
                int64_t ld = a.ldy, col = n;
                if (a.split_n > 0 && n >= a.split_n) {
                  dst = a.y2;
                  ld = a.ldy2;
                  col = n - a.split_n;
                }
                if (a.out_f32)
                  reinterpret_cast<float*>(dst)[(size_t)tok * ld + col] = __bfloat162float(o);
                else
                  reinterpret_cast<__nv_bfloat16*>(dst)[(size_t)tok * ld + col] = o;
                const unsigned long long k =
                    argmax_key((uint32_t)__bfloat16_as_ushort(o), (uint32_t)(a.row_offset + n));
                key = k > key ? k : key;
              }
              if (key > best[nt][p]) best[nt][p] = key;  // lanes of one token: reduced at the end
            }
          }
        }
      }
    }

    if (do_argmax) {
      // the eight lanes (g = 0..7) that share a token column hold its per-lane maxima
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int p = 0; p < 2; ++p)
#pragma unroll
          for (int o = 4; o < 32; o <<= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best[nt][p], o);
            best[nt][p] = other > best[nt][p] ? other : best[nt][p];
          }
      if (g == 0) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int p = 0; p < 2; ++p) {
            const int tok = nt * 8 + 2 * c + p;
            if (tok < M && best[nt][p] != 0ull) atomicMax(&a.am_keys[tok], best[nt][p]);
          }
      }
      __threadfence();
      __syncwarp();
      unsigned prev = 0;
      if (lane == 0) prev = atomicAdd(a.am_count, 1u);
      prev = __shfl_sync(0xffffffffu, prev, 0);
      if (prev == gridDim.x * (unsigned)E - 1) {
        __threadfence();
        unsigned long long key = lane < M ? atomicExch(&a.am_keys[lane], 0ull) : 0ull;
        if (a.peerbuf) key = peer_key_max(a.peerbuf, key, M, a.err);  // whole warp
        if (lane < M) {
          const int64_t row = (int64_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
          if (a.am_out) a.am_out[lane] = row;
          if (a.am_key_out) a.am_key_out[lane] = key;
          if (a.chain.topk_index || a.chain.topk_p || a.chain.draft_tokens || a.chain.positions)
            draft_chain_store(a.chain, lane, row);
        }
        if (lane == 0) *a.am_count = 0u;
      }
    }
  }
  pdl_trigger();
}

// Decode argmax keys (after a cross-rank MAX reduction of the keys) into row ids.
using DenseKernel = void (*)(const DenseArgs);

template <int WT, int NT, int MODE>
DenseKernel pick_cpw(int cpw) {
  switch (cpw) {
    case 1: return dense_gemv_kernel<WT, NT, 1, MODE>;
    case 2: return dense_gemv_kernel<WT, NT, 2, MODE>;
    case 4: return dense_gemv_kernel<WT, NT, 4, MODE>;
    case 8: return dense_gemv_kernel<WT, NT, 8, MODE>;
    default: return nullptr;
  }
}

template <int WT, int MODE>
DenseKernel pick_nt(int nt, int cpw) {
  return nt == 1 ? pick_cpw<WT, 1, MODE>(cpw) : (nt == 2 ? pick_cpw<WT, 2, MODE>(cpw) : nullptr);
}

template <int MODE>
DenseKernel dense_kernel_mode(int wtype, int nt, int cpw) {
  switch (wtype) {
    case W_INT8: return pick_nt<W_INT8, MODE>(nt, cpw);
    case W_FP8: return pick_nt<W_FP8, MODE>(nt, cpw);
    case W_BF16: return pick_nt<W_BF16, MODE>(nt, cpw);
    case W_NVFP4:
      if constexpr (MODE == DENSE_NORM) return nullptr;  // the fused norm is a W8A16 form
      else return pick_nt<W_NVFP4, MODE>(nt, cpw);
    default: return nullptr;
  }
}

// The instances of the slice and norm modes (dense_gemv_slice.cu, dense_gemv_norm.cu).
DenseKernel dense_kernel_slice(int wtype, int nt, int cpw);
DenseKernel dense_kernel_norm(int wtype, int nt, int cpw);

}  // namespace fnx
