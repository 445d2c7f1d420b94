// Dense weight-only GEMV for M <= 16 tokens: y[m, n] = (sum_k W[n, k] x[m, k]) * s[n].
//
// Replaces the reference's Triton kernels
//   _w8a16_gemv_kernel        kernels/sglang/srt/layers/quantization/w8a16_gemv.py:132-322
//   _w8a16_gemv_silu_kernel   w8a16_gemv.py:865-961
//   _w4a16_nvfp4_gemv_kernel  kernels/sglang/srt/layers/quantization/w4a16_nvfp4_gemv.py:122-216
// with one persistent sm_100a kernel family.
//
// Work decomposition.  A work unit is one 16-row weight tile (8 output columns of gate
// plus the matching 8 of up for the fused SiLU form) over a k range; a group of W warps
// shares the unit, each warp streaming CPW 64-byte chunks of every row with 128-bit
// loads into a ring of S register stages, so S-1 units of loads are in flight while the
// current one is multiplied.  The group's partial tiles are summed in shared memory in a
// fixed order (deterministic), then scaled, rounded to bf16 (w8a16_gemv.py:92-95) and
// stored.  With ksplit > 1 the k range is split across groups and the last group to
// finish a tile sums the partials in split order and resets the tile counter
// (w8a16_gemv.py:289-321), so no memset is needed between calls or graph replays.
//
// Greedy argmax (fused).  Each output thread builds a 64-bit key of its bf16-rounded
// logit and global row; the key maximum is the largest logit with the lowest row on
// ties (torch.argmax).  Keys are reduced per tile with shuffles, per CTA in registers,
// across CTAs with one atomicMax per token, and the last CTA decodes and clears them.
#include "fnx_common.cuh"
#include "fnx_kernels.h"

namespace fnx {

template <int WT, int NT, int CPW, int S>
__global__ void __launch_bounds__(512, 1) dense_gemv_kernel(const DenseArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int Q = Geo<WT>::Q;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int W = a.W;
  const int grp = warp / W, wig = warp - grp * W;
  const int gthreads = W * 32, gtid = tid - grp * gthreads;
  const int g = lane >> 2, c = lane & 3;
  const int M = a.M, N = a.N, K = a.K;
  const int srow = stage_row_bytes(K);

  uint8_t* xs = smem;
  float* unscale = reinterpret_cast<float*>(smem + (size_t)M * srow);
  float* red = unscale + 16;  // [G][2][W][32][NT][4]
  int* flags = reinterpret_cast<int*>(red + (size_t)a.G * 2 * W * 32 * NT * 4);

  const uint64_t pol = policy_evict_first();
  const int stride = gridDim.x * a.G;
  const int first = blockIdx.x * a.G + grp;
  const int n_units = a.n_units;
  const int ksplit = a.ksplit;
  const int cpu = W * CPW;  // chunks per unit
  const bool silu = a.silu != 0;

  // Weight row of MMA row i (0..15) of a tile; `ok` false for rows past the end (their
  // loads are redirected to row 0 and their outputs dropped).
  auto row_of = [&](int tile, int i, bool& ok) -> int {
    if (silu) {
      const int col = tile * 8 + (i & 7);
      ok = col < N;
      return ok ? ((i < 8) ? col : N + col) : 0;
    }
    const int r = tile * 16 + i;
    ok = r < N;
    return ok ? r : 0;
  };

  WeightRing<CPW, S> ring;

  auto load = [&](int u, uint4(&va)[CPW], uint4(&vb)[CPW], uint32_t(&sa)[CPW],
                  uint32_t(&sb)[CPW]) {
    const int tile = u / ksplit, ks = u - tile * ksplit;
    bool oka, okb;
    const int ra = row_of(tile, g, oka), rb = row_of(tile, g + 8, okb);
    const uint8_t* pa = a.w + (size_t)ra * a.ldw;
    const uint8_t* pb = a.w + (size_t)rb * a.ldw;
#pragma unroll
    for (int cc = 0; cc < CPW; ++cc) {
      const int chunk = ks * cpu + wig * CPW + cc;
      const int off = chunk * 64 + c * 16;
      va[cc] = ldg_stream(pa + off, pol);
      vb[cc] = ldg_stream(pb + off, pol);
      if constexpr (WT == W_NVFP4) {
        const int kb = chunk * 8 + c * 2;
        sa[cc] = ldg_u16_stream(a.bs + (size_t)ra * a.ldbs + kb, pol);
        sb[cc] = ldg_u16_stream(a.bs + (size_t)rb * a.ldbs + kb, pol);
      } else {
        sa[cc] = 0;
        sb[cc] = 0;
      }
    }
  };

  // Running argmax key of this thread's token (threads with i == 0 of a token).
  unsigned long long best = 0ull;
  const bool do_argmax = a.am_keys != nullptr;

  auto process = [&](int u, const uint4(&va)[CPW], const uint4(&vb)[CPW],
                     const uint32_t(&sa)[CPW], const uint32_t(&sb)[CPW], int it) {
    const int tile = u / ksplit, ks = u - tile * ksplit;
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[nt][r] = 0.f;
#pragma unroll
    for (int cc = 0; cc < CPW; ++cc) {
      const int chunk = ks * cpu + wig * CPW + cc;
      uint4 xf[NT][Q];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int t = nt * 8 + g;
#pragma unroll
        for (int q = 0; q < Q; ++q) {
          xf[nt][q] = (t < M) ? *reinterpret_cast<const uint4*>(
                                    xs + (size_t)t * srow + ((chunk * Q + q) * 4 + c) * 16)
                              : make_uint4(0u, 0u, 0u, 0u);
        }
      }
      chunk_mma<WT, NT>(acc, va[cc], vb[cc], sa[cc], sb[cc], xf);
    }
    // Cross-warp reduction of the group's partial tiles (double-buffered by `it`).
    float* rbuf = red + (size_t)((grp * 2 + (it & 1)) * W) * 32 * NT * 4;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
      *reinterpret_cast<float4*>(rbuf + ((size_t)(wig * 32 + lane) * NT + nt) * 4) =
          make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]);
    group_sync(1 + grp, gthreads);

    // One thread per (token, tile row): gtid = tok * 16 + i (gthreads >= 16 * M).
    const int tok = gtid >> 4, i = gtid & 15;
    const bool live = tok < M;
    float rowsum = 0.f;
    if (live) {
      const int nt = tok >> 3, col = tok & 7;
      const int src = (i & 7) * 4 + (col >> 1);
      const int reg = ((i >> 3) << 1) | (col & 1);
      for (int w = 0; w < W; ++w) rowsum += rbuf[((size_t)(w * 32 + src) * NT + nt) * 4 + reg];
    }
    if (ksplit > 1) {
      float* wsp = a.ws + ((size_t)tile * ksplit + ks) * 256;
      if (live) st_cg_f32(wsp + i * 16 + tok, rowsum);
      __threadfence();
      group_sync(1 + grp, gthreads);
      if (gtid == 0) {
        const unsigned prev = atomicAdd(&a.ws_cnt[tile], 1u);
        flags[grp] = (prev == (unsigned)(ksplit - 1));
      }
      group_sync(1 + grp, gthreads);
      if (!flags[grp]) return;
      __threadfence();
      rowsum = 0.f;
      if (live) {
        const float* base = a.ws + (size_t)tile * ksplit * 256 + i * 16 + tok;
        for (int s = 0; s < ksplit; ++s) rowsum += ld_cg_f32(base + (size_t)s * 256);
      }
      if (gtid == 0) a.ws_cnt[tile] = 0u;  // every arrival for this tile has happened
    }

    if (silu) {
      // Rows 0..7 are gate, 8..15 up; lane i + 8 of the same token holds up's sum.
      const float up = __shfl_down_sync(0xffffffffu, rowsum, 8);
      const int n = tile * 8 + i;
      if (live && i < 8 && n < N) {
        const float us = unscale[tok];
        const float gv = rowsum * us * load_row_scale(a.scale, a.scale_kind, n);
        const float uv = up * us * load_row_scale(a.scale, a.scale_kind, (int64_t)N + n);
        const __nv_bfloat16 o = __float2bfloat16_rn(silu_f32(gv) * uv);
        reinterpret_cast<__nv_bfloat16*>(a.y)[(size_t)tok * a.ldy + n] = o;
      }
      return;
    }

    const int n = tile * 16 + i;
    const bool valid = live && n < N;
    uint32_t bits = 0;
    if (valid) {
      const float v = rowsum * unscale[tok] * load_row_scale(a.scale, a.scale_kind, n);
      const __nv_bfloat16 o = __float2bfloat16_rn(v);
      bits = (uint32_t)__bfloat16_as_ushort(o);
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
    }
    if (do_argmax) {
      unsigned long long key = valid ? argmax_key(bits, (uint32_t)(a.row_offset + n)) : 0ull;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
      }
      if (i == 0 && key > best) best = key;
    }
  };

  // Prologue: weight loads of the first S-1 units go out before waiting on the
  // previous kernel (the weights do not depend on it).
#pragma unroll
  for (int s = 0; s < S - 1; ++s) {
    const int u = first + s * stride;
    if (u < n_units) load(u, ring.va[s], ring.vb[s], ring.sa[s], ring.sb[s]);
  }
  pdl_wait();
  stage_rows<WT>(xs, unscale, M, K, [&](int r) {
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

  if (do_argmax) {
    const int tok = gtid >> 4, i = gtid & 15;
    if (i == 0 && tok < M && best != 0ull) atomicMax(&a.am_keys[tok], best);
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const unsigned prev = atomicAdd(a.am_count, 1u);
      flags[0] = (prev == gridDim.x - 1);
    }
    __syncthreads();
    if (flags[0]) {
      __threadfence();
      if (tid < M) {
        const unsigned long long key = atomicExch(&a.am_keys[tid], 0ull);
        if (a.am_out) a.am_out[tid] = (int64_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
        if (a.am_key_out) a.am_key_out[tid] = key;
      }
      if (tid == 0) *a.am_count = 0u;
    }
  }
}

// Decode argmax keys (after a cross-rank MAX reduction of the keys) into row ids.
__global__ void argmax_decode_kernel(const unsigned long long* keys, int64_t* out, int M) {
  const int t = threadIdx.x;
  if (t < M) out[t] = (int64_t)(0xFFFFFFFFu - (uint32_t)(keys[t] & 0xFFFFFFFFull));
}

int launch_argmax_decode(const unsigned long long* keys, int64_t* out, int M,
                         cudaStream_t stream) {
  argmax_decode_kernel<<<1, 32, 0, stream>>>(keys, out, M);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

using DenseKernel = void (*)(const DenseArgs);

template <int WT, int NT>
DenseKernel pick_cpw(int cpw) {
  switch (cpw) {
    case 1: return dense_gemv_kernel<WT, NT, 1, 4>;
    case 2: return dense_gemv_kernel<WT, NT, 2, 3>;
    case 4: return dense_gemv_kernel<WT, NT, 4, 2>;
    default: return nullptr;
  }
}

template <int WT>
DenseKernel pick_nt(int nt, int cpw) {
  return nt == 1 ? pick_cpw<WT, 1>(cpw) : (nt == 2 ? pick_cpw<WT, 2>(cpw) : nullptr);
}

DenseKernel dense_kernel(int wtype, int nt, int cpw) {
  switch (wtype) {
    case W_INT8: return pick_nt<W_INT8>(nt, cpw);
    case W_FP8: return pick_nt<W_FP8>(nt, cpw);
    case W_BF16: return pick_nt<W_BF16>(nt, cpw);
    case W_NVFP4: return pick_nt<W_NVFP4>(nt, cpw);
    default: return nullptr;
  }
}

int dense_occupancy(int wtype, int nt, int cpw, int threads, size_t smem) {
  DenseKernel k = dense_kernel(wtype, nt, cpw);
  if (!k || !prepare_kernel((const void*)k)) return 0;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, threads, smem) != cudaSuccess) return 0;
  return n;
}

int launch_dense(const DenseArgs& a, int wtype, int nt, int cpw, int grid, size_t smem,
                 cudaStream_t stream) {
  DenseKernel k = dense_kernel(wtype, nt, cpw);
  if (!k) return 1;
  if (!prepare_kernel((const void*)k)) return 2;
  return launch_with_pdl((const void*)k, a, grid, a.W * a.G * 32, smem, a.pdl, stream);
}

}  // namespace fnx
