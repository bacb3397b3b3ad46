// FP32 issue-rate probe: the measured CUDA-core peak that the roofline of the
// CUDA-core kernels (conv, symmetric contraction, edge) is compared with.
//
// Every thread runs eight independent fused multiply-add chains, so each SM
// sub-partition always has an independent FMA to issue; the compiler cannot
// fold the chains (their coefficients come from the arguments) and the result
// is stored so they are not dead.  FLOPs = blocks x 256 x 8 x 16 x iters x 2.
#include "common.cuh"

namespace {

__global__ void __launch_bounds__(256) k_fma_probe(float* out, float a, float b, int iters) {
  float x[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) x[k] = (float)(threadIdx.x + k) * 1e-3f;
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int r = 0; r < 16; ++r) {
#pragma unroll
      for (int k = 0; k < 8; ++k) x[k] = fmaf(x[k], a, b);
    }
  }
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) s += x[k];
  out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

}  // namespace

extern "C" int mace_fma_probe(float* out, int32_t blocks, int32_t iters, void* stream) {
  if (!out || blocks <= 0 || iters <= 0) return mace::fail(MACE_ERR_BAD_ARG, "mace_fma_probe: bad arguments");
  k_fma_probe<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(out, 0.999f, 1e-4f, iters);
  MACE_CUDA_TRY(cudaGetLastError());
  return MACE_OK;
}
