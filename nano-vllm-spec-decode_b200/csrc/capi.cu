// extern "C" entry points of libnvattn.so (declared in include/nvattn.h).  Argument checks mirror the asserts of
// the reference (nanovllm/layers/attention.py:36-39) but return status codes instead of raising; tensor maps for
// TMA are encoded on the host per call (a few hundred ns) from the caller's pointers, so nothing is cached
// across calls and a captured graph keeps the maps it was recorded with.
#include <cudaTypedefs.h>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <mutex>

#include "../../include/nvattn.h"
#include "nva_kernels.h"
#include "nva_ptx.cuh"

namespace nva {
// The device error word (bits in include/nvattn.h); defined here so the host accessors below own its symbol.
__device__ uint32_t g_error_word = 0;

thread_local char g_last_cuda_error[256] = "";

// Host helpers shared with paged_decode_noalloc.cu (declared in nva_kernels.h).
int cuda_fail(cudaError_t e) {
  snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
  return NVA_ERR_CUDA;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Rank-3 bf16 view {128 dims, heads, rows} with the given row stride (bytes), 64 x 1 x 128 boxes, 128B swizzle.
int encode_rows(CUtensorMap* tm, const void* base, int64_t heads, int64_t rows, int64_t row_stride_bytes) {
  auto fn = encode_fn();
  if (fn == nullptr) return NVA_ERR_CUDA;
  cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[2] = {128 * 2, static_cast<cuuint64_t>(row_stride_bytes)};
  cuuint32_t box[3] = {64, 1, 128};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return NVA_ERR_CUDA;
  }
  return NVA_OK;
}

}  // namespace nva

namespace {

using nva::cuda_fail;
using nva::encode_rows;
using nva::g_last_cuda_error;

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  static int cached[64] = {0};
  if (dev < 64 && cached[dev] > 0) return cached[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  if (dev < 64) cached[dev] = n;
  return n;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
// The attention kernels take row maxima of unscaled scores and scale them afterwards: the scale must be positive
// (and finite); NaN fails the comparison.
bool valid_scale(float s) { return s > 0.f && s < 3.0e38f; }

int check_cache(const void* k_cache, const void* v_cache, int32_t num_blocks, int32_t block_size, int32_t kvh) {
  if (k_cache == nullptr || v_cache == nullptr || num_blocks <= 0 || block_size <= 0 || kvh <= 0)
    return NVA_ERR_INVALID_ARGUMENT;
  if (block_size % nva::kTileTokens != 0) return NVA_ERR_UNSUPPORTED;
  if (static_cast<int64_t>(num_blocks) * block_size >= (int64_t(1) << 31)) return NVA_ERR_UNSUPPORTED;
  if (!aligned16(k_cache) || !aligned16(v_cache)) return NVA_ERR_ALIGNMENT;
  return NVA_OK;
}

}  // namespace

extern "C" {

NVA_API int nva_version(void) { return (0 << 16) | 1; }

NVA_API const char* nva_status_string(int status) {
  switch (status) {
    case NVA_OK: return "ok";
    case NVA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case NVA_ERR_UNSUPPORTED: return "unsupported shape or dtype";
    case NVA_ERR_ALIGNMENT: return "pointer or stride not 16-byte aligned";
    case NVA_ERR_WORKSPACE: return "workspace missing or too small";
    case NVA_ERR_CUDA: return "CUDA error";
    default: return "unknown status";
  }
}

NVA_API const char* nva_last_cuda_error(void) { return g_last_cuda_error; }

NVA_API int nva_store_kvcache(const void* key, int64_t key_row_stride, const void* value, int64_t value_row_stride,
                              void* k_cache, void* v_cache, int64_t num_slots, const int32_t* slot_mapping,
                              int32_t num_tokens, int32_t num_kv_heads, int32_t head_dim, int32_t elem_bytes,
                              void* stream) {
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || num_slots < 0) return NVA_ERR_INVALID_ARGUMENT;
  if (elem_bytes != 2 && elem_bytes != 4) return NVA_ERR_UNSUPPORTED;
  if (num_tokens == 0) return NVA_OK;
  if (key == nullptr || value == nullptr || k_cache == nullptr || v_cache == nullptr || slot_mapping == nullptr)
    return NVA_ERR_INVALID_ARGUMENT;
  const int32_t row_elems = num_kv_heads * head_dim;
  if (key_row_stride < row_elems || value_row_stride < row_elems) return NVA_ERR_INVALID_ARGUMENT;
  cudaError_t e = nva::launch_store_kvcache(key, key_row_stride, value, value_row_stride, k_cache, v_cache,
                                            num_slots, slot_mapping, num_tokens, row_elems, elem_bytes,
                                            static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? NVA_OK : cuda_fail(e);
}

NVA_API size_t nva_paged_decode_workspace_bytes(int32_t num_seqs, int32_t q_per_seq, int32_t num_heads,
                                                int32_t num_kv_heads, int32_t head_dim) {
  (void)num_seqs;
  (void)head_dim;
  if (num_kv_heads <= 0 || num_heads % num_kv_heads != 0) return 0;
  const int np = nva::decode_rows_padded(q_per_seq * (num_heads / num_kv_heads));
  const int sms = sm_count();
  if (np == 0 || sms == 0) return 0;
  return nva::decode_workspace_bytes(sms, np);
}

NVA_API int nva_paged_decode(const void* q, int64_t q_row_stride, const void* k_cache, const void* v_cache,
                             int32_t num_blocks, int32_t block_size, const int32_t* context_lens,
                             const int32_t* block_tables, int32_t bt_row_stride, int32_t num_seqs, int32_t q_per_seq,
                             int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, float softmax_scale,
                             void* out, int64_t out_row_stride, void* workspace, size_t workspace_bytes,
                             void* stream) {
  if (num_seqs < 0 || q_per_seq < 1 || num_heads <= 0 || num_kv_heads <= 0) return NVA_ERR_INVALID_ARGUMENT;
  if (num_heads % num_kv_heads != 0) return NVA_ERR_INVALID_ARGUMENT;
  if (!valid_scale(softmax_scale)) return NVA_ERR_INVALID_ARGUMENT;
  if (head_dim != nva::kHeadDim) return NVA_ERR_UNSUPPORTED;
  if (num_seqs == 0) return NVA_OK;
  if (num_seqs > nva::kMaxDecodeSeqs) return NVA_ERR_UNSUPPORTED;
  int rc = check_cache(k_cache, v_cache, num_blocks, block_size, num_kv_heads);
  if (rc != NVA_OK) return rc;
  if (q == nullptr || out == nullptr || context_lens == nullptr || block_tables == nullptr || bt_row_stride < 1)
    return NVA_ERR_INVALID_ARGUMENT;
  if (q_row_stride < static_cast<int64_t>(num_heads) * head_dim || out_row_stride < static_cast<int64_t>(num_heads) * head_dim)
    return NVA_ERR_INVALID_ARGUMENT;
  if (!aligned16(q) || (q_row_stride % 8) != 0 || !aligned16(out) || (out_row_stride % 8) != 0)
    return NVA_ERR_ALIGNMENT;
  const int group = num_heads / num_kv_heads;
  const int np = nva::decode_rows_padded(q_per_seq * group);
  if (np == 0) return NVA_ERR_UNSUPPORTED;
  const int grid = sm_count();
  if (grid == 0) return cuda_fail(cudaGetLastError());
  const size_t need = nva::decode_workspace_bytes(grid, np);
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace)) return NVA_ERR_WORKSPACE;

  CUtensorMap tm_k, tm_v;
  const int64_t rows = static_cast<int64_t>(num_blocks) * block_size;
  const int64_t rs = static_cast<int64_t>(num_kv_heads) * head_dim * 2;
  if ((rc = encode_rows(&tm_k, k_cache, num_kv_heads, rows, rs)) != NVA_OK) return rc;
  if ((rc = encode_rows(&tm_v, v_cache, num_kv_heads, rows, rs)) != NVA_OK) return rc;

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
  nva::decode_workspace_layout(workspace, grid, np, &p);
  // a plain launch: a programmatic dependency on the KV scatter measured no faster on the decode step
  cudaError_t e = nva::launch_paged_decode(tm_k, tm_v, p, np, grid, static_cast<cudaStream_t>(stream), false);
  return e == cudaSuccess ? NVA_OK : cuda_fail(e);
}

}  // extern "C"

namespace {

// Varlen workspace: the decode kernel's split partials (48-row tiles) followed by the prefill work plan
// (count, capacity entries, work counter).
size_t varlen_decode_part(int sms) { return (nva::decode_workspace_bytes(sms, 48) + 255) & ~size_t(255); }
int varlen_plan_capacity(int32_t num_seqs, int32_t total_q) { return total_q / 128 + num_seqs + 1; }

}  // namespace

extern "C" {

NVA_API size_t nva_varlen_workspace_bytes(int32_t num_seqs, int32_t total_q, int32_t num_heads,
                                          int32_t num_kv_heads, int32_t head_dim) {
  (void)head_dim;
  if (num_kv_heads <= 0 || num_heads % num_kv_heads != 0 || num_seqs < 0 || total_q < 0) return 0;
  const int sms = sm_count();
  if (sms == 0) return 0;
  return varlen_decode_part(sms) + sizeof(int32_t) * (2 + static_cast<size_t>(varlen_plan_capacity(num_seqs, total_q)));
}

NVA_API int nva_varlen_attention(const void* q, int64_t q_row_stride, const void* key, int64_t key_row_stride,
                                 const void* value, int64_t value_row_stride, const void* k_cache,
                                 const void* v_cache, int32_t num_blocks, int32_t block_size,
                                 const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int32_t num_seqs,
                                 int32_t total_q, int32_t total_k, int32_t max_seqlen_q, int32_t max_seqlen_k,
                                 const int32_t* block_tables, int32_t bt_row_stride, int32_t num_heads,
                                 int32_t num_kv_heads, int32_t head_dim, float softmax_scale, void* out,
                                 int64_t out_row_stride, void* workspace, size_t workspace_bytes, void* stream) {
  if (num_seqs < 0 || total_q < 0 || num_heads <= 0 || num_kv_heads <= 0 || max_seqlen_q < 0 || max_seqlen_k < 0)
    return NVA_ERR_INVALID_ARGUMENT;
  if (num_heads % num_kv_heads != 0) return NVA_ERR_INVALID_ARGUMENT;
  if (!valid_scale(softmax_scale)) return NVA_ERR_INVALID_ARGUMENT;
  if (head_dim != nva::kHeadDim) return NVA_ERR_UNSUPPORTED;
  if (num_seqs == 0 || total_q == 0) return NVA_OK;
  if (num_seqs > nva::kMaxDecodeSeqs) return NVA_ERR_UNSUPPORTED;
  if (q == nullptr || out == nullptr || cu_seqlens_q == nullptr || cu_seqlens_k == nullptr)
    return NVA_ERR_INVALID_ARGUMENT;
  if (!aligned16(q) || (q_row_stride % 8) != 0 || !aligned16(out) || (out_row_stride % 8) != 0)
    return NVA_ERR_ALIGNMENT;
  const int group = num_heads / num_kv_heads;
  const bool paged = block_tables != nullptr;
  int rc;
  CUtensorMap tm_k, tm_v;
  if (paged) {
    if ((rc = check_cache(k_cache, v_cache, num_blocks, block_size, num_kv_heads)) != NVA_OK) return rc;
    if (bt_row_stride < 1) return NVA_ERR_INVALID_ARGUMENT;
    const int64_t rows = static_cast<int64_t>(num_blocks) * block_size;
    const int64_t rs = static_cast<int64_t>(num_kv_heads) * head_dim * 2;
    if ((rc = encode_rows(&tm_k, k_cache, num_kv_heads, rows, rs)) != NVA_OK) return rc;
    if ((rc = encode_rows(&tm_v, v_cache, num_kv_heads, rows, rs)) != NVA_OK) return rc;
  } else {
    if (key == nullptr || value == nullptr || total_k <= 0) return NVA_ERR_INVALID_ARGUMENT;
    if (!aligned16(key) || !aligned16(value) || (key_row_stride % 8) != 0 || (value_row_stride % 8) != 0)
      return NVA_ERR_ALIGNMENT;
    if ((rc = encode_rows(&tm_k, key, num_kv_heads, total_k, key_row_stride * 2)) != NVA_OK) return rc;
    if ((rc = encode_rows(&tm_v, value, num_kv_heads, total_k, value_row_stride * 2)) != NVA_OK) return rc;
  }
  const int grid = sm_count();
  if (grid == 0) return cuda_fail(cudaGetLastError());
  const int np = 48;
  const int max_n = np / group;                // query runs up to this length use the decode kernel
  const int cap = varlen_plan_capacity(num_seqs, total_q);
  if (cap > nva::kMaxPrefillTiles) return NVA_ERR_UNSUPPORTED;
  const size_t need = varlen_decode_part(grid) + sizeof(int32_t) * (2 + static_cast<size_t>(cap));
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace)) return NVA_ERR_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Launch order: prefill plan, decode kernel (short runs), prefill kernel (long runs), each with a programmatic
  // dependency on the one before.  The decode kernel waits for the plan kernel before it lets the prefill kernel
  // start, and the prefill kernel does not depend on the decode kernel, so its blocks fill the SMs that the decode
  // kernel's blocks leave.
  const bool long_runs = !paged || max_seqlen_q > max_n;
  nva::PrefillParams pp{};
  CUtensorMap tm_q, tm_o;
  bool o_tma = false;
  // Work items of two query tiles (prefill_pair_kernel) share each K / V tile between two softmax groups, faster per
  // tile, but halve the number of items: chosen when the call's rows x heads give at least four such items per SM
  // and some query run can fill two tiles (max_seqlen_q > 128: with shorter runs every item would have one tile and
  // half of the pair kernel's softmax warps would idle).
  const bool pair = max_seqlen_q > 128 && static_cast<int64_t>(total_q) * num_heads >= 4LL * grid * 256;
  if (long_runs) {
    if ((rc = encode_rows(&tm_q, q, num_heads, total_q, q_row_stride * 2)) != NVA_OK) return rc;
    // single-tile kernel: full 128-row output tiles leave through TMA stores when the output rows allow a tensor map
    o_tma = !pair && aligned16(out) && (out_row_stride * 2) % 16 == 0;
    if (o_tma && (rc = encode_rows(&tm_o, out, num_heads, total_q, out_row_stride * 2)) != NVA_OK) return rc;
    pp.q = static_cast<const __nv_bfloat16*>(q);
    pp.q_row_stride = q_row_stride;
    pp.out = static_cast<__nv_bfloat16*>(out);
    pp.out_row_stride = out_row_stride;
    pp.cu_q = cu_seqlens_q;
    pp.cu_k = cu_seqlens_k;
    pp.block_tables = block_tables;
    pp.bt_stride = bt_row_stride;
    pp.num_seqs = num_seqs;
    pp.num_heads = num_heads;
    pp.num_kv_heads = num_kv_heads;
    pp.group = group;
    pp.min_q = paged ? max_n + 1 : 1;
    pp.block_size = block_size;
    pp.num_blocks = num_blocks;
    pp.q_tiles_bound = cap;
    pp.tiles_per_item = pair ? 2 : 1;
    pp.o_tma = o_tma ? 1 : 0;
    pp.wait_primary = paged ? 0 : 1;   // after the decode kernel / directly after the plan kernel
    pp.scale_log2 = softmax_scale * 1.4426950408889634f;
    pp.plan = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(workspace) + varlen_decode_part(grid));
    cudaError_t e = nva::launch_prefill_plan(pp, s);
    if (e != cudaSuccess) return cuda_fail(e);
  }
  if (paged) {
    nva::DecodeParams p{};
    p.q = static_cast<const __nv_bfloat16*>(q);
    p.q_row_stride = q_row_stride;
    p.out = static_cast<__nv_bfloat16*>(out);
    p.out_row_stride = out_row_stride;
    p.cu_q = cu_seqlens_q;
    p.cu_k = cu_seqlens_k;
    p.ctx_lens = nullptr;
    p.block_tables = block_tables;
    p.bt_stride = bt_row_stride;
    p.num_seqs = num_seqs;
    p.n_fixed = 0;
    p.num_heads = num_heads;
    p.num_kv_heads = num_kv_heads;
    p.group = group;
    p.max_n = max_n;
    p.block_size = block_size;
    p.num_blocks = num_blocks;
    p.scale_log2 = softmax_scale * 1.4426950408889634f;
    nva::decode_workspace_layout(workspace, grid, np, &p);
    cudaError_t e = nva::launch_paged_decode(tm_k, tm_v, p, np, grid, s, true);
    if (e != cudaSuccess) return cuda_fail(e);
  }
  if (long_runs) {
    const int pgrid = static_cast<int>(std::min<int64_t>(grid, static_cast<int64_t>(cap) * num_heads));
    cudaError_t e = pair ? nva::launch_prefill_pair(tm_q, tm_k, tm_v, pp, pgrid, s)
                         : nva::launch_prefill(tm_q, tm_k, tm_v, o_tma ? tm_o : tm_q, pp, pgrid, s);
    if (e != cudaSuccess) return cuda_fail(e);
  }
  return NVA_OK;
}

NVA_API int nva_greedy_accept(const void* target_ids, int64_t target_row_stride, const void* draft_ids,
                              int64_t draft_row_stride, const void* num_drafts, int32_t num_seqs, int32_t k,
                              int32_t id_bytes, void* num_accepted, void* next_tokens, void* stream) {
  if (num_seqs < 0 || k < 0) return NVA_ERR_INVALID_ARGUMENT;
  if (id_bytes != 4 && id_bytes != 8) return NVA_ERR_UNSUPPORTED;
  if (num_seqs == 0) return NVA_OK;
  if (target_ids == nullptr || num_drafts == nullptr || num_accepted == nullptr || next_tokens == nullptr)
    return NVA_ERR_INVALID_ARGUMENT;
  if (k > 0 && draft_ids == nullptr) return NVA_ERR_INVALID_ARGUMENT;
  if (target_row_stride < k + 1 || (k > 0 && draft_row_stride < k)) return NVA_ERR_INVALID_ARGUMENT;
  cudaError_t e = nva::launch_greedy_accept(target_ids, target_row_stride, draft_ids, draft_row_stride, num_drafts,
                                            num_seqs, k, id_bytes, num_accepted, next_tokens,
                                            static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? NVA_OK : cuda_fail(e);
}

NVA_API int nva_qk_norm_rope_store(const void* qkv, int64_t qkv_row_stride, int32_t num_tokens, int32_t num_heads,
                                   int32_t num_kv_heads, int32_t head_dim, const int64_t* positions,
                                   const float* cos_sin, int32_t max_position, const void* q_norm_weight,
                                   const void* k_norm_weight, float eps, void* q_out, int64_t q_out_row_stride,
                                   void* k_out, int64_t k_out_row_stride, void* k_cache, void* v_cache,
                                   int64_t num_slots, const int32_t* slot_mapping, void* stream) {
  if (num_tokens < 0 || num_heads <= 0 || num_kv_heads <= 0 || max_position <= 0 || num_slots < 0)
    return NVA_ERR_INVALID_ARGUMENT;
  if (head_dim != nva::kHeadDim) return NVA_ERR_UNSUPPORTED;
  if (num_heads + 2 * num_kv_heads > 64) return NVA_ERR_UNSUPPORTED;   // one block of 8 warps x 8 heads per token
  if (num_tokens == 0) return NVA_OK;
  if (qkv == nullptr || positions == nullptr || cos_sin == nullptr || q_norm_weight == nullptr ||
      k_norm_weight == nullptr || q_out == nullptr)
    return NVA_ERR_INVALID_ARGUMENT;
  if (slot_mapping != nullptr && (k_cache == nullptr || v_cache == nullptr)) return NVA_ERR_INVALID_ARGUMENT;
  const int64_t width = static_cast<int64_t>(num_heads + 2 * num_kv_heads) * head_dim;
  if (qkv_row_stride < width || q_out_row_stride < static_cast<int64_t>(num_heads) * head_dim ||
      (k_out != nullptr && k_out_row_stride < static_cast<int64_t>(num_kv_heads) * head_dim))
    return NVA_ERR_INVALID_ARGUMENT;
  // 8-byte vectors (4 bf16) everywhere, 16-byte float4 reads of the cos / sin table
  auto al8 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; };
  if (!al8(qkv) || qkv_row_stride % 4 != 0 || !al8(q_out) || q_out_row_stride % 4 != 0 || !aligned16(cos_sin) ||
      (k_out != nullptr && (!al8(k_out) || k_out_row_stride % 4 != 0)) ||
      (k_cache != nullptr && (!al8(k_cache) || !al8(v_cache))) || !al8(q_norm_weight) || !al8(k_norm_weight))
    return NVA_ERR_ALIGNMENT;
  cudaError_t e = nva::launch_qk_prologue(qkv, qkv_row_stride, num_tokens, num_heads, num_kv_heads, positions, cos_sin,
                                          max_position, q_norm_weight, k_norm_weight, eps, q_out, q_out_row_stride,
                                          k_out, k_out_row_stride, k_cache, v_cache, num_slots, slot_mapping,
                                          static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? NVA_OK : cuda_fail(e);
}

NVA_API int nva_shard_argmax(const void* logits, int64_t row_stride, int32_t rows, int32_t vocab_shard,
                             int64_t vocab_offset, int32_t elem_bytes, uint64_t* keys, void* stream) {
  if (rows < 0 || vocab_shard < 0 || vocab_offset < 0) return NVA_ERR_INVALID_ARGUMENT;
  if (elem_bytes != 2 && elem_bytes != 4) return NVA_ERR_UNSUPPORTED;
  if (rows == 0) return NVA_OK;
  if (logits == nullptr || keys == nullptr || vocab_shard == 0 || row_stride < vocab_shard)
    return NVA_ERR_INVALID_ARGUMENT;
  if (rows > 65535 || vocab_offset + vocab_shard > int64_t(0xFFFFFFFF)) return NVA_ERR_UNSUPPORTED;
  const int sms = sm_count();
  if (sms <= 0) return cuda_fail(cudaGetLastError());
  cudaError_t e = nva::launch_shard_argmax(logits, row_stride, rows, vocab_shard, static_cast<uint32_t>(vocab_offset),
                                           elem_bytes, keys, sms, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? NVA_OK : cuda_fail(e);
}

NVA_API int nva_shard_accept(const uint64_t* keys, int32_t num_shards, int32_t num_seqs, int32_t k,
                             const void* draft_ids, int64_t draft_row_stride, const void* num_drafts, int32_t id_bytes,
                             void* num_accepted, void* next_tokens, void* stream) {
  if (num_seqs < 0 || k < 0 || num_shards <= 0) return NVA_ERR_INVALID_ARGUMENT;
  if (id_bytes != 4 && id_bytes != 8) return NVA_ERR_UNSUPPORTED;
  if (num_seqs == 0) return NVA_OK;
  if (keys == nullptr || num_drafts == nullptr || num_accepted == nullptr || next_tokens == nullptr)
    return NVA_ERR_INVALID_ARGUMENT;
  if (k > 0 && (draft_ids == nullptr || draft_row_stride < k)) return NVA_ERR_INVALID_ARGUMENT;
  cudaError_t e = nva::launch_shard_accept(keys, num_shards, num_seqs, k, draft_ids, draft_row_stride, num_drafts,
                                           id_bytes, num_accepted, next_tokens, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? NVA_OK : cuda_fail(e);
}

NVA_API int nva_get_device_error(uint32_t* out_bits) {
  if (out_bits == nullptr) return NVA_ERR_INVALID_ARGUMENT;
  cudaError_t e = cudaMemcpyFromSymbol(out_bits, nva::g_error_word, sizeof(uint32_t));
  return e == cudaSuccess ? NVA_OK : cuda_fail(e);
}

NVA_API int nva_clear_device_error(void) {
  const uint32_t zero = 0;
  cudaError_t e = cudaMemcpyToSymbol(nva::g_error_word, &zero, sizeof(uint32_t));
  return e == cudaSuccess ? NVA_OK : cuda_fail(e);
}

}  // extern "C"
