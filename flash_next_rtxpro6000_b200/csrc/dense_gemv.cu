// Dense weight-only GEMV: the plain-mode instances of the kernel in dense_gemv.cuh, the
// argmax decode kernel and the launch entry points of all three modes.
#include "dense_gemv.cuh"

namespace fnx {

__global__ void argmax_decode_kernel(const unsigned long long* keys, int64_t* out, int M) {
  const int t = threadIdx.x;
  if (t < M) out[t] = (int64_t)(0xFFFFFFFFu - (uint32_t)(keys[t] & 0xFFFFFFFFull));
}

int launch_argmax_decode(const unsigned long long* keys, int64_t* out, int M,
                         cudaStream_t stream) {
  argmax_decode_kernel<<<1, 32, 0, stream>>>(keys, out, M);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

DenseKernel dense_kernel(int wtype, int nt, int cpw, int mode) {
  switch (mode) {
    case DENSE_PLAIN: return dense_kernel_mode<DENSE_PLAIN>(wtype, nt, cpw);
    case DENSE_SLICE: return dense_kernel_slice(wtype, nt, cpw);
    case DENSE_NORM: return dense_kernel_norm(wtype, nt, cpw);
    default: return nullptr;
  }
}

int dense_occupancy(int wtype, int nt, int cpw, int mode, int threads, size_t smem) {
  DenseKernel k = dense_kernel(wtype, nt, cpw, mode);
  if (!k || !prepare_kernel((const void*)k)) return 0;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, threads, smem) != cudaSuccess) return 0;
  return n;
}

int launch_dense(const DenseArgs& a, int wtype, int nt, int cpw, int grid, size_t smem,
                 cudaStream_t stream) {
  DenseKernel k = dense_kernel(wtype, nt, cpw, dense_mode(a));
  if (!k) return 1;
  if (!prepare_kernel((const void*)k)) return 2;
  return launch_with_pdl((const void*)k, a, grid, (a.W + 1 + a.E) * 32, smem, a.pdl, stream);
}

}  // namespace fnx
