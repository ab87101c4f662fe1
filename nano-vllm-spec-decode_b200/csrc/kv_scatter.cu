// (a) Slot-mapped KV scatter into the paged cache (replaces store_kvcache_kernel, nanovllm/layers/attention.py:10-30).
// Token i with slot = slot_mapping[i] != -1 copies its key row and value row (row_elems contiguous elements each,
// any row stride) to cache row `slot`.  The copy is bit-exact: 16-byte vectors when every row start is 16-byte
// aligned, 4- or 2-byte words otherwise.  One thread moves one vector of the key row and the same vector of the
// value row, so a warp streams 512 contiguous bytes of each.
#include "nva_ptx.cuh"
#include "nva_kernels.h"

namespace nva {

namespace {

template <typename V>
__global__ void __launch_bounds__(256)
store_kvcache_kernel(const uint8_t* __restrict__ key, int64_t key_row_bytes, const uint8_t* __restrict__ value,
                     int64_t value_row_bytes, uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache,
                     int64_t num_slots, const int32_t* __restrict__ slots, int32_t num_tokens, int32_t vecs_per_row) {
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = static_cast<int64_t>(num_tokens) * vecs_per_row;
  if (gid >= total) return;
  const int32_t i = static_cast<int32_t>(gid / vecs_per_row);
  const int32_t v = static_cast<int32_t>(gid - static_cast<int64_t>(i) * vecs_per_row);
  const int64_t slot = __ldg(slots + i);
  if (slot == -1) return;                    // attention.py:23
  if (slot < 0 || slot >= num_slots) {       // never write outside the pool
    if (v == 0) atomicOr(&g_error_word, kErrSlotRange);
    return;
  }
  const int64_t row_bytes = static_cast<int64_t>(vecs_per_row) * sizeof(V);
  const V kx = __ldg(reinterpret_cast<const V*>(key + i * key_row_bytes) + v);
  const V vx = __ldg(reinterpret_cast<const V*>(value + i * value_row_bytes) + v);
  reinterpret_cast<V*>(k_cache + slot * row_bytes)[v] = kx;
  reinterpret_cast<V*>(v_cache + slot * row_bytes)[v] = vx;
}

template <typename V>
cudaError_t launch(const void* key, int64_t krb, const void* value, int64_t vrb, void* kc, void* vc,
                   int64_t num_slots, const int32_t* slots, int32_t n, int32_t vecs, cudaStream_t stream) {
  const int64_t total = static_cast<int64_t>(n) * vecs;
  const int64_t blocks = (total + 255) / 256;
  store_kvcache_kernel<V><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
      static_cast<const uint8_t*>(key), krb, static_cast<const uint8_t*>(value), vrb, static_cast<uint8_t*>(kc),
      static_cast<uint8_t*>(vc), num_slots, slots, n, vecs);
  return cudaGetLastError();
}

bool aligned(const void* p, int64_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace

cudaError_t launch_store_kvcache(const void* key, int64_t key_row_stride, const void* value,
                                 int64_t value_row_stride, void* k_cache, void* v_cache, int64_t num_slots,
                                 const int32_t* slots, int32_t num_tokens, int32_t row_elems, int32_t elem_bytes,
                                 cudaStream_t stream) {
  if (num_tokens == 0) return cudaSuccess;
  const int64_t row_bytes = static_cast<int64_t>(row_elems) * elem_bytes;
  const int64_t krb = key_row_stride * elem_bytes, vrb = value_row_stride * elem_bytes;
  auto fits = [&](int64_t a) {
    return row_bytes % a == 0 && krb % a == 0 && vrb % a == 0 && aligned(key, a) && aligned(value, a) &&
           aligned(k_cache, a) && aligned(v_cache, a);
  };
  if (fits(16))
    return launch<uint4>(key, krb, value, vrb, k_cache, v_cache, num_slots, slots, num_tokens,
                         static_cast<int32_t>(row_bytes / 16), stream);
  if (fits(4))
    return launch<uint32_t>(key, krb, value, vrb, k_cache, v_cache, num_slots, slots, num_tokens,
                            static_cast<int32_t>(row_bytes / 4), stream);
  return launch<uint16_t>(key, krb, value, vrb, k_cache, v_cache, num_slots, slots, num_tokens,
                          static_cast<int32_t>(row_bytes / 2), stream);
}

}  // namespace nva
