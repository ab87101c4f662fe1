// Test harness (not part of libnvattn.so): evaluates the kernels' FMA-pipe exponentials exp2_poly and exp2_poly2
// (nano-vllm-spec-decode_b200/csrc/nva_ptx.cuh) and CUDA's exp2f on the same inputs, so that a test can measure
// their error against float64 2^x.  Built by tests/test_gpu_exp2_poly.py (or __graft_entry__.build()) with nvcc.
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include "nva_ptx.cuh"

namespace {

__global__ void exp2_check_kernel(const float* __restrict__ x, int n, float* __restrict__ poly,
                                  float* __restrict__ poly2, float* __restrict__ ref) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (2 * i >= n) return;
  const float a = x[2 * i];
  const float b = 2 * i + 1 < n ? x[2 * i + 1] : 0.0f;
  const float2 p2 = nva::exp2_poly2(make_float2(a, b));
  poly[2 * i] = nva::exp2_poly(a);
  poly2[2 * i] = p2.x;
  ref[2 * i] = exp2f(a);
  if (2 * i + 1 < n) {
    poly[2 * i + 1] = nva::exp2_poly(b);
    poly2[2 * i + 1] = p2.y;
    ref[2 * i + 1] = exp2f(b);
  }
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int exp2_check(const float* x, int n, float* poly, float* poly2,
                                                                 float* ref, void* stream) {
  if (n <= 0) return 0;
  const int pairs = (n + 1) / 2;
  exp2_check_kernel<<<(pairs + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, n, poly, poly2, ref);
  return static_cast<int>(cudaGetLastError());
}
