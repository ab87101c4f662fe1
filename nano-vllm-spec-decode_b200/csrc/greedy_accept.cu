// (c) Greedy accept length (replaces the greedy core of verify_drafts, nanovllm/layers/sampler.py:66-82):
//   accepted[s, j] = target[s, j] == draft[s, j] && j < num_drafts[s];  num_accepted[s] = unbroken run from j = 0;
//   next_token[s] = target[s, num_accepted[s]].
// Integer-exact; one thread per sequence (S <= a few hundred, K <= 32: latency, not bandwidth, matters here).
#include "nva_kernels.h"

namespace nva {

namespace {

template <typename T>
__global__ void __launch_bounds__(128)
greedy_accept_kernel(const T* __restrict__ target, int64_t tstride, const T* __restrict__ drafts, int64_t dstride,
                     const T* __restrict__ num_drafts, int32_t S, int32_t K, T* __restrict__ num_accepted,
                     T* __restrict__ next_tokens) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= S) return;
  const T* trow = target + s * tstride;
  const T* drow = drafts + s * dstride;
  const int64_t nd = static_cast<int64_t>(num_drafts[s]);
  int a = 0;
  while (a < K && a < nd && trow[a] == drow[a]) ++a;
  num_accepted[s] = static_cast<T>(a);
  next_tokens[s] = trow[a];
}

}  // namespace

cudaError_t launch_greedy_accept(const void* target, int64_t target_row_stride, const void* drafts,
                                 int64_t draft_row_stride, const void* num_drafts, int32_t num_seqs, int32_t k,
                                 int32_t id_bytes, void* num_accepted, void* next_tokens, cudaStream_t stream) {
  if (num_seqs == 0) return cudaSuccess;
  const unsigned blocks = static_cast<unsigned>((num_seqs + 127) / 128);
  if (id_bytes == 4) {
    greedy_accept_kernel<int32_t><<<blocks, 128, 0, stream>>>(
        static_cast<const int32_t*>(target), target_row_stride, static_cast<const int32_t*>(drafts),
        draft_row_stride, static_cast<const int32_t*>(num_drafts), num_seqs, k, static_cast<int32_t*>(num_accepted),
        static_cast<int32_t*>(next_tokens));
  } else {
    greedy_accept_kernel<int64_t><<<blocks, 128, 0, stream>>>(
        static_cast<const int64_t*>(target), target_row_stride, static_cast<const int64_t*>(drafts),
        draft_row_stride, static_cast<const int64_t*>(num_drafts), num_seqs, k, static_cast<int64_t*>(num_accepted),
        static_cast<int64_t*>(next_tokens));
  }
  return cudaGetLastError();
}

}  // namespace nva
