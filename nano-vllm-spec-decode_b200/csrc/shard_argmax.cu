// Greedy verify from vocabulary shards (the argmax of verify_drafts, nanovllm/layers/sampler.py:66, over the logits
// that ParallelLMHead gathers to rank 0, nanovllm/layers/embed_head.py:56-68).
//
// shard_argmax: each rank reduces its logits shard [rows, V_shard] to one 64-bit key per row,
//     key = orderable(max value) << 32 | (0xFFFFFFFF - global index of its first occurrence),
// so that the largest key over all shards names the row's argmax with torch's tie rule (the lowest index of the
// maximum; NaN counts as the largest value, -0 equals +0).  HBM-bound: one pass over the logits, 16-byte loads.
// The row is split into chunks so that small calls still spread over every SM; chunk maxima meet in the output
// key with a 64-bit atomicMax (the output is cleared in stream order first).
//
// shard_accept: merges the keys of all shards into the target ids and applies the greedy accept rule
// (sampler.py:79-82) in the same thread: one thread per sequence.
#include <algorithm>
#include <type_traits>

#include "nva_kernels.h"

namespace nva {

namespace {

constexpr int kArgmaxThreads = 256;

__device__ __forceinline__ float widen(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float widen(float v) { return v; }

// Total order on floats as unsigned integers (NaN above +inf, -0 folded into +0).
__device__ __forceinline__ uint32_t orderable(float v) {
  uint32_t u = __float_as_uint(v);
  if (v != v) u = 0x7FC00000u;
  if (u == 0x80000000u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// "a beats b" for a later element a against the current best b: strictly greater, or NaN over a number.
__device__ __forceinline__ bool beats(float a, float b) { return a > b || (a != a && b == b); }

template <typename T, int VEC>
__global__ void __launch_bounds__(kArgmaxThreads)
shard_argmax_kernel(const T* __restrict__ logits, int64_t row_stride, int32_t vocab, int32_t chunk,
                    uint32_t vocab_offset, unsigned long long* __restrict__ keys) {
  const int row = blockIdx.y;
  const int c0 = blockIdx.x * chunk;
  const int c1 = min(vocab, c0 + chunk);
  const T* p = logits + static_cast<int64_t>(row) * row_stride;
  float best = -__int_as_float(0x7F800000);    // -inf
  int best_i = -1;
  int best_v = -1;   // bf16: the vector holding the first occurrence of `best`
  if constexpr (VEC > 1) {
    // chunk and row starts are multiples of VEC elements (16 bytes): whole vectors, four loads in flight per
    // thread (its elements stay in increasing index order), then the row's ragged end
    constexpr int kUnroll = 8;
    const int nvec = (c1 - c0) / VEC;
    for (int v0 = threadIdx.x; v0 < nvec; v0 += kUnroll * kArgmaxThreads) {
      uint4 raw[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int v = v0 + u * kArgmaxThreads;
        if (v < nvec) raw[u] = __ldg(reinterpret_cast<const uint4*>(p + c0 + v * VEC));
      }
      if constexpr (std::is_same_v<T, __nv_bfloat16>) {
        // bf16: per 16-byte vector, its maximum with packed NaN-propagating max instructions, and the vector that
        // first reached the running maximum; the element's position inside that vector is found once at the end
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int v = v0 + u * kArgmaxThreads;
          if (v < nvec) {
            const __nv_bfloat162* e2 = reinterpret_cast<const __nv_bfloat162*>(&raw[u]);
            const __nv_bfloat162 m2 = __hmax2_nan(__hmax2_nan(e2[0], e2[1]), __hmax2_nan(e2[2], e2[3]));
            const float vm = __bfloat162float(__hmax_nan(__low2bfloat16(m2), __high2bfloat16(m2)));
            const bool take = best_v < 0 || beats(vm, best);
            best = take ? vm : best;
            best_v = take ? v : best_v;
          }
        }
      } else {
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int v = v0 + u * kArgmaxThreads;
          if (v >= nvec) break;
          const T* e = reinterpret_cast<const T*>(&raw[u]);
#pragma unroll
          for (int j = 0; j < VEC; ++j) {
            const float x = widen(e[j]);
            if (best_i < 0 || beats(x, best)) { best = x; best_i = c0 + v * VEC + j; }
          }
        }
      }
    }
    if (best_v >= 0) {   // bf16: the first element of the best vector equal to its maximum (a NaN when it is NaN)
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p + c0 + best_v * VEC));
      const T* e = reinterpret_cast<const T*>(&raw);
      const bool want_nan = best != best;
      int j = VEC - 1;
#pragma unroll
      for (int q = VEC - 1; q >= 0; --q) {
        const float x = widen(e[q]);
        j = (want_nan ? x != x : x == best) ? q : j;
      }
      best_i = c0 + best_v * VEC + j;
    }
    for (int i = c0 + nvec * VEC + threadIdx.x; i < c1; i += kArgmaxThreads) {
      const float x = widen(p[i]);
      if (best_i < 0 || beats(x, best)) { best = x; best_i = i; }
    }
  } else {
    for (int i = c0 + threadIdx.x; i < c1; i += kArgmaxThreads) {
      const float x = widen(p[i]);
      if (best_i < 0 || beats(x, best)) { best = x; best_i = i; }
    }
  }
  unsigned long long key = 0ull;
  if (best_i >= 0)
    key = (static_cast<unsigned long long>(orderable(best)) << 32) |
          (0xFFFFFFFFu - (vocab_offset + static_cast<uint32_t>(best_i)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, key, o);
    key = other > key ? other : key;
  }
  __shared__ unsigned long long warp_best[kArgmaxThreads / 32];
  if ((threadIdx.x & 31) == 0) warp_best[threadIdx.x >> 5] = key;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kArgmaxThreads / 32; ++w) key = warp_best[w] > key ? warp_best[w] : key;
    atomicMax(keys + row, key);
  }
}

template <typename T>
__global__ void __launch_bounds__(128)
shard_accept_kernel(const unsigned long long* __restrict__ keys, int32_t num_shards, int32_t num_seqs, int32_t k,
                    const T* __restrict__ drafts, int64_t dstride, const T* __restrict__ num_drafts,
                    T* __restrict__ num_accepted, T* __restrict__ next_tokens) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= num_seqs) return;
  const int64_t rows = static_cast<int64_t>(num_seqs) * (k + 1);
  const int64_t nd = static_cast<int64_t>(num_drafts[s]);
  int a = 0;
  T target = 0;
  for (int j = 0; j <= k; ++j) {
    unsigned long long best = 0ull;
    for (int r = 0; r < num_shards; ++r) {
      const unsigned long long v = keys[r * rows + static_cast<int64_t>(s) * (k + 1) + j];
      best = v > best ? v : best;
    }
    target = static_cast<T>(0xFFFFFFFFu - static_cast<uint32_t>(best & 0xFFFFFFFFull));
    if (j == k || j >= nd || drafts[s * dstride + j] != target) break;
    ++a;
  }
  num_accepted[s] = static_cast<T>(a);
  next_tokens[s] = target;
}

}  // namespace

cudaError_t launch_shard_argmax(const void* logits, int64_t row_stride, int32_t rows, int32_t vocab,
                                uint32_t vocab_offset, int32_t elem_bytes, void* keys, int sms, cudaStream_t stream) {
  cudaError_t e = cudaMemsetAsync(keys, 0, static_cast<size_t>(rows) * sizeof(unsigned long long), stream);
  if (e != cudaSuccess) return e;
  const int vec = 16 / elem_bytes;
  const bool vector = (reinterpret_cast<uintptr_t>(logits) & 15u) == 0 && (row_stride * elem_bytes) % 16 == 0;
  // about four blocks per SM over the whole call, each at least 2048 elements, chunks whole vectors
  const int64_t want = std::max<int64_t>(1, (4LL * sms + rows - 1) / rows);
  int chunks = static_cast<int>(std::min<int64_t>(want, std::max<int64_t>(1, vocab / 2048)));
  int chunk = (vocab + chunks - 1) / chunks;
  chunk = (chunk + vec - 1) / vec * vec;
  chunks = (vocab + chunk - 1) / chunk;
  const dim3 grid(static_cast<unsigned>(chunks), static_cast<unsigned>(rows));
  auto* out = static_cast<unsigned long long*>(keys);
  if (elem_bytes == 2) {
    auto* x = static_cast<const __nv_bfloat16*>(logits);
    if (vector)
      shard_argmax_kernel<__nv_bfloat16, 8><<<grid, kArgmaxThreads, 0, stream>>>(x, row_stride, vocab, chunk,
                                                                                vocab_offset, out);
    else
      shard_argmax_kernel<__nv_bfloat16, 1><<<grid, kArgmaxThreads, 0, stream>>>(x, row_stride, vocab, chunk,
                                                                                vocab_offset, out);
  } else {
    auto* x = static_cast<const float*>(logits);
    if (vector)
      shard_argmax_kernel<float, 4><<<grid, kArgmaxThreads, 0, stream>>>(x, row_stride, vocab, chunk, vocab_offset,
                                                                         out);
    else
      shard_argmax_kernel<float, 1><<<grid, kArgmaxThreads, 0, stream>>>(x, row_stride, vocab, chunk, vocab_offset,
                                                                         out);
  }
  return cudaGetLastError();
}

cudaError_t launch_shard_accept(const void* keys, int32_t num_shards, int32_t num_seqs, int32_t k, const void* drafts,
                                int64_t draft_row_stride, const void* num_drafts, int32_t id_bytes,
                                void* num_accepted, void* next_tokens, cudaStream_t stream) {
  if (num_seqs == 0) return cudaSuccess;
  const unsigned blocks = static_cast<unsigned>((num_seqs + 127) / 128);
  auto* kp = static_cast<const unsigned long long*>(keys);
  if (id_bytes == 4) {
    shard_accept_kernel<int32_t><<<blocks, 128, 0, stream>>>(
        kp, num_shards, num_seqs, k, static_cast<const int32_t*>(drafts), draft_row_stride,
        static_cast<const int32_t*>(num_drafts), static_cast<int32_t*>(num_accepted),
        static_cast<int32_t*>(next_tokens));
  } else {
    shard_accept_kernel<int64_t><<<blocks, 128, 0, stream>>>(
        kp, num_shards, num_seqs, k, static_cast<const int64_t*>(drafts), draft_row_stride,
        static_cast<const int64_t*>(num_drafts), static_cast<int64_t*>(num_accepted),
        static_cast<int64_t*>(next_tokens));
  }
  return cudaGetLastError();
}

}  // namespace nva
