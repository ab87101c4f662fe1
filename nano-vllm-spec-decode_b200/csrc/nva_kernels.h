// Internal launch interface between the C ABI (capi.cu) and the kernels.  Not part of the public header.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <utility>

namespace nva {

constexpr int kHeadDim = 128;
constexpr int kTileTokens = 128;      // KV tokens per pipeline stage (= UMMA M)
constexpr int kMaxDecodeSeqs = 1024;  // sequences the decode kernel's on-chip schedule holds
constexpr int kMaxDecodeRows = 48;    // q_per_seq * group rows per kv head (UMMA N)

// One attention step over paged KV, seen from the decode / verify kernel.  Two modes:
//   decode  (cu_q == nullptr): sequence b owns q rows [b*n_fixed, (b+1)*n_fixed), keys [0, ctx_lens[b]);
//   varlen  (cu_q != nullptr): rows [cu_q[b], cu_q[b+1]), keys [0, cu_k[b+1]-cu_k[b]); only sequences with
//           1 <= q_len <= max_n are handled here (longer ones go to the prefill kernel).
struct DecodeParams {
  const __nv_bfloat16* q;
  int64_t q_row_stride;
  __nv_bfloat16* out;
  int64_t out_row_stride;
  const int32_t* cu_q;
  const int32_t* cu_k;
  const int32_t* ctx_lens;
  const int32_t* block_tables;
  int32_t bt_stride;
  int32_t num_seqs;
  int32_t n_fixed;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t group;
  int32_t max_n;
  int32_t block_size;
  int32_t num_blocks;
  float scale_log2;
  float* part_o;     // [2 * grid, NP, 128] split partial outputs (normalised)
  float* part_lse;   // [2 * grid, NP] their log2-sum-exp
  int32_t* counters; // [grid][4] merge tickets per cut segment (CTA of its first piece) and softmax group: zero on
                     // entry and on exit
  int32_t pdl;       // 1: launched with a programmatic dependency on the preceding kernel (launch_paged_decode sets it)
};

size_t decode_workspace_bytes(int grid, int np);
// Carve the workspace (decode_workspace_bytes(grid, np) bytes) into the partials and the merge counters.
void decode_workspace_layout(void* ws, int grid, int np, DecodeParams* p);
int decode_rows_padded(int rows);  // 16, 32 or 48 (0 if too many)
// pdl: launch with a programmatic dependency on the preceding kernel in the stream (the kernel's blocks may start
// while it finishes; they wait for it before their first global read, and only then let the next such grid start).
// Only for a preceding kernel, not a memset or copy.
cudaError_t launch_paged_decode(const CUtensorMap& tm_k, const CUtensorMap& tm_v, const DecodeParams& p, int np,
                                int grid, cudaStream_t stream, bool pdl);

// Launch helper: `kernel` with a programmatic dependency on the preceding kernel when `pdl`, else a plain launch.
template <class... KArgs, class... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Varlen prefill kernel (long query runs) — q rows tiled by 128 per (sequence, q head).
struct PrefillParams {
  const __nv_bfloat16* q;
  int64_t q_row_stride;
  __nv_bfloat16* out;
  int64_t out_row_stride;
  const int32_t* cu_q;
  const int32_t* cu_k;
  const int32_t* block_tables;  // nullptr: contiguous K/V rows cu_k[b] + pos
  int32_t bt_stride;
  int32_t num_seqs;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t group;
  int32_t min_q;                // sequences with q_len >= min_q are handled here
  int32_t block_size;
  int32_t num_blocks;
  int32_t q_tiles_bound;        // capacity of the work plan: an upper bound on the number of 128-row q tiles
  int32_t tiles_per_item;       // 128-row q tiles per work item: 1 (prefill_kernel) or 2 (prefill_pair_kernel)
  int32_t o_tma;                // 1: full output tiles are written by TMA stores through the output tensor map
  int32_t wait_primary;         // 1: the preceding kernel (the plan kernel) produced data this grid reads
  float scale_log2;
  int32_t* plan;                // workspace: [0] = number of items, [1..] = (seq << 12 | item of the sequence),
                                // heaviest first, [1 + q_tiles_bound] = work counter (items taken after the first
                                // wave)
};
constexpr int kMaxPrefillTiles = 4096;

// Key tiles visible to 128-row query tile qt of a sequence with n queries and L keys, causal bottom-right: at least
// one (a fully masked tile keeps the pipeline uniform; those rows get a zero output), 0 past the last query tile.
__host__ __device__ __forceinline__ int prefill_tile_nkv(int n, int L, int qt) {
  const int rows = n - qt * 128 < 128 ? n - qt * 128 : 128;
  if (rows <= 0) return 0;
  const int t = (L - n + qt * 128 + rows - 1) / 128 + 1;
  return t > 1 ? t : 1;
}
// The prefill work plan (one block), launched with a programmatic dependency on the preceding kernel.
cudaError_t launch_prefill_plan(const PrefillParams& p, cudaStream_t stream);
// The prefill kernel, launched with a programmatic dependency on the preceding kernel: the plan kernel
// (p.wait_primary = 1: it waits for the plan before reading it) or the decode kernel of the same call, which comes
// after the plan kernel and has waited for it (p.wait_primary = 0: its blocks may run beside the decode kernel's
// last blocks).  Either way the grid completes only after the preceding one has.
cudaError_t launch_prefill(const CUtensorMap& tm_q, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                           const CUtensorMap& tm_o, const PrefillParams& p, int grid, cudaStream_t stream);
// The same step with work items of two consecutive query tiles (p.tiles_per_item = 2 in the plan): one softmax
// warpgroup per tile, sharing each K / V tile.  Same launch contract as launch_prefill.
cudaError_t launch_prefill_pair(const CUtensorMap& tm_q, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                                const PrefillParams& p, int grid, cudaStream_t stream);

cudaError_t launch_store_kvcache(const void* key, int64_t key_row_stride, const void* value,
                                 int64_t value_row_stride, void* k_cache, void* v_cache, int64_t num_slots,
                                 const int32_t* slots, int32_t num_tokens, int32_t row_elems, int32_t elem_bytes,
                                 cudaStream_t stream);

cudaError_t launch_greedy_accept(const void* target, int64_t target_row_stride, const void* drafts,
                                 int64_t draft_row_stride, const void* num_drafts, int32_t num_seqs, int32_t k,
                                 int32_t id_bytes, void* num_accepted, void* next_tokens, cudaStream_t stream);

// Host helpers of the C ABI (capi.cu): record a CUDA error's text for nva_last_cuda_error() and return NVA_ERR_CUDA;
// encode a rank-3 bf16 tensor map {128 dims, heads, rows} (row stride in bytes) with 64 x 1 x 128 boxes and 128-byte
// swizzle, the layout every TMA load of the kernels uses (an encoder failure is recorded the same way).
int cuda_fail(cudaError_t e);
int encode_rows(CUtensorMap* tm, const void* base, int64_t heads, int64_t rows, int64_t row_stride_bytes);

// Qwen3's attention prologue in one pass (q/k RMSNorm, rotary, KV scatter); see qk_prologue.cu.
cudaError_t launch_qk_prologue(const void* qkv, int64_t qkv_stride, int32_t T, int32_t H, int32_t KVH,
                               const int64_t* positions, const float* cos_sin, int32_t max_pos, const void* q_w,
                               const void* k_w, float eps, void* q_out, int64_t q_out_stride, void* k_out,
                               int64_t k_out_stride, void* k_cache, void* v_cache, int64_t num_slots,
                               const int32_t* slots, cudaStream_t stream);

// Per-row (max, index) keys of a vocabulary shard of logits (bf16 when elem_bytes == 2, float when 4), and the merge
// of several shards' keys into greedy accept lengths; see shard_argmax.cu.
cudaError_t launch_shard_argmax(const void* logits, int64_t row_stride, int32_t rows, int32_t vocab,
                                uint32_t vocab_offset, int32_t elem_bytes, void* keys, int sms, cudaStream_t stream);
cudaError_t launch_shard_accept(const void* keys, int32_t num_shards, int32_t num_seqs, int32_t k, const void* drafts,
                                int64_t draft_row_stride, const void* num_drafts, int32_t id_bytes,
                                void* num_accepted, void* next_tokens, cudaStream_t stream);

}  // namespace nva
