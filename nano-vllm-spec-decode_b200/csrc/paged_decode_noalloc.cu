// nva_paged_decode_noalloc: the paged decode / verify attention of nva_paged_decode for callers that cannot
// allocate device memory.
//
// nva_paged_decode needs a caller workspace for the split-KV partials.  Some callers have no way to provide one:
// code that runs inside an allocator hook or a host callback (where a cudaMalloc would recurse or deadlock),
// runtimes that carve every byte out of an arena reserved at start-up and only hand out the tensors they own, and
// embedders whose memory manager exposes no device allocation at all.  For them the partials live here, in a
// fixed array compiled into the library (NVA_NOALLOC_SCRATCH_BYTES on every GPU that loads it, held until the
// process exits).  The kernels are the same ones nva_paged_decode launches; only the scratch pointer differs.
//
// Rules of use (also stated in include/nvattn.h):
//  - the first call on each device looks up the array's device address with cudaGetSymbolAddress, with that device
//    current, and caches it; make that first call before any stream capture;
//  - every call on a device shares the one array and leaves its contents behind; the only part that must start at
//    zero (the merge tickets) is cleared by each call itself with a memset in stream order before its kernel, and
//    every partial a merge reads is written earlier in the same call; calls that overlap on the GPU (two streams,
//    say) race on the array and must be serialised by the caller;
//  - a call that needs more than NVA_NOALLOC_SCRATCH_BYTES is rejected with NVA_ERR_WORKSPACE before any launch;
//  - nothing here allocates: no cudaMalloc, no cudaFree, no allocating library routine.
#include <mutex>

#include "../../include/nvattn.h"
#include "nva_kernels.h"

namespace {

// The scratch.  Host code must not pass this symbol to a kernel: in host code it is only a stand-in, its device
// address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[NVA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};

// Device address of the scratch and the SM count of the current device, looked up once per device.
int current_device_scratch(void** addr, int* sms) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return nva::cuda_fail(e);
  if (dev < 0 || dev >= kMaxDevices) return NVA_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if ((e = cudaGetSymbolAddress(&p, g_noalloc_scratch)) != cudaSuccess) return nva::cuda_fail(e);
    if (p == nullptr) return nva::cuda_fail(cudaErrorInvalidSymbol);
    int n = 0;
    if ((e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return nva::cuda_fail(e);
    if (n <= 0) return nva::cuda_fail(cudaErrorInvalidDevice);
    g_sm_count[dev] = n;
    g_scratch_addr[dev] = p;
  }
  *addr = g_scratch_addr[dev];
  *sms = g_sm_count[dev];
  return NVA_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" NVA_API int nva_paged_decode_noalloc(const void* q, int64_t q_row_stride, const void* k_cache,
                                                const void* v_cache, int32_t num_blocks, int32_t block_size,
                                                const int32_t* context_lens, const int32_t* block_tables,
                                                int32_t bt_row_stride, int32_t num_seqs, int32_t q_per_seq,
                                                int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                                                float softmax_scale, void* out, int64_t out_row_stride,
                                                void* stream) {
  // the same argument checks as nva_paged_decode
  if (num_seqs < 0 || q_per_seq < 1 || num_heads <= 0 || num_kv_heads <= 0) return NVA_ERR_INVALID_ARGUMENT;
  if (num_heads % num_kv_heads != 0) return NVA_ERR_INVALID_ARGUMENT;
  if (!(softmax_scale > 0.f && softmax_scale < 3.0e38f)) return NVA_ERR_INVALID_ARGUMENT;   // positive, finite
  if (head_dim != nva::kHeadDim) return NVA_ERR_UNSUPPORTED;
  if (num_seqs == 0) return NVA_OK;
  if (num_seqs > nva::kMaxDecodeSeqs) return NVA_ERR_UNSUPPORTED;
  if (k_cache == nullptr || v_cache == nullptr || num_blocks <= 0 || block_size <= 0) return NVA_ERR_INVALID_ARGUMENT;
  if (block_size % nva::kTileTokens != 0) return NVA_ERR_UNSUPPORTED;
  if (static_cast<int64_t>(num_blocks) * block_size >= (int64_t(1) << 31)) return NVA_ERR_UNSUPPORTED;
  if (q == nullptr || out == nullptr || context_lens == nullptr || block_tables == nullptr || bt_row_stride < 1)
    return NVA_ERR_INVALID_ARGUMENT;
  if (q_row_stride < static_cast<int64_t>(num_heads) * head_dim ||
      out_row_stride < static_cast<int64_t>(num_heads) * head_dim)
    return NVA_ERR_INVALID_ARGUMENT;
  if (!aligned16(k_cache) || !aligned16(v_cache) || !aligned16(q) || (q_row_stride % 8) != 0 || !aligned16(out) ||
      (out_row_stride % 8) != 0)
    return NVA_ERR_ALIGNMENT;
  const int group = num_heads / num_kv_heads;
  const int np = nva::decode_rows_padded(q_per_seq * group);
  if (np == 0) return NVA_ERR_UNSUPPORTED;

  void* scratch = nullptr;
  int grid = 0;
  int rc = current_device_scratch(&scratch, &grid);
  if (rc != NVA_OK) return rc;
  // the partials of one call: 2 pieces per CTA x np rows x (128 dims + log-sum-exp) floats
  if (nva::decode_workspace_bytes(grid, np) > NVA_NOALLOC_SCRATCH_BYTES) return NVA_ERR_WORKSPACE;

  CUtensorMap tm_k, tm_v;
  const int64_t rows = static_cast<int64_t>(num_blocks) * block_size;
  const int64_t row_bytes = static_cast<int64_t>(num_kv_heads) * head_dim * 2;
  if ((rc = nva::encode_rows(&tm_k, k_cache, num_kv_heads, rows, row_bytes)) != NVA_OK) return rc;
  if ((rc = nva::encode_rows(&tm_v, v_cache, num_kv_heads, rows, row_bytes)) != NVA_OK) return rc;

  nva::DecodeParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_row_stride = q_row_stride;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_row_stride = out_row_stride;
  p.cu_q = nullptr;
  p.cu_k = nullptr;
  p.ctx_lens = context_lens;
  p.block_tables = block_tables;
  p.bt_stride = bt_row_stride;
  p.num_seqs = num_seqs;
  p.n_fixed = q_per_seq;
  p.num_heads = num_heads;
  p.num_kv_heads = num_kv_heads;
  p.group = group;
  p.max_n = np / group;
  p.block_size = block_size;
  p.num_blocks = num_blocks;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  nva::decode_workspace_layout(scratch, grid, np, &p);
  // The merge tickets at the start of the array must be zero when the kernel starts.  A normal call leaves them
  // zero, but one that gave up part-way may not have, so every call clears them first, in stream order (a memset
  // of the existing array: nothing is allocated).
  const size_t ticket_bytes =
      static_cast<size_t>(reinterpret_cast<unsigned char*>(p.part_o) - reinterpret_cast<unsigned char*>(p.counters));
  cudaError_t e = cudaMemsetAsync(p.counters, 0, ticket_bytes, static_cast<cudaStream_t>(stream));
  // (a plain launch: the operation before the kernel is the memset, not a kernel)
  if (e == cudaSuccess)
    e = nva::launch_paged_decode(tm_k, tm_v, p, np, grid, static_cast<cudaStream_t>(stream), false);
  return e == cudaSuccess ? NVA_OK : nva::cuda_fail(e);
}
