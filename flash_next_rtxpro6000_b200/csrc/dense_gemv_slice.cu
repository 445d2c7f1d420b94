// The slice-mode instances of the dense GEMV kernel (dense_gemv.cuh), compiled apart
// so that the three modes build in parallel.
#include "dense_gemv.cuh"

namespace fnx {

DenseKernel dense_kernel_slice(int wtype, int nt, int cpw) {
  return dense_kernel_mode<DENSE_SLICE>(wtype, nt, cpw);
}

}  // namespace fnx
