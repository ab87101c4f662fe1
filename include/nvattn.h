/*
 * nvattn.h — C ABI of the B200 (sm_100a) attention hot path for nano-vllm-spec-decode.
 *
 * Every entry point:
 *   - takes plain device pointers, element strides and sizes (no framework types);
 *   - is asynchronous on the `stream` argument (a cudaStream_t passed as void*), makes no host
 *     synchronisation and performs no device allocation, so it can be captured in a CUDA graph;
 *   - returns an nva_status (0 = success). Invalid arguments are rejected before any launch.
 *
 * Tensor layouts follow nano-vllm (nanovllm/layers/attention.py):
 *   q        [T_q, H, D]        bf16, head stride D, row stride q_row_stride (elements)
 *   key/value[T, KVH, D]        bf16, head stride D, row stride *_row_stride (elements)
 *   k_cache  [NB, BS, KVH, D]   bf16, contiguous (one layer's slice of the [2, L, NB, BS, KVH, D] pool)
 *   block_tables [B, W]         int32, row stride bt_row_stride, -1 = unused
 *   out      [T_q, H, D]        bf16, row stride out_row_stride (elements)
 * Query head h reads kv head h / (H / KVH) (grouped-query attention).
 */
#ifndef NVATTN_H
#define NVATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NVA_API __attribute__((visibility("default")))

typedef enum {
  NVA_OK = 0,
  NVA_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, shape mismatch */
  NVA_ERR_UNSUPPORTED = 2,      /* a shape or dtype the kernels do not implement (e.g. head_dim != 128) */
  NVA_ERR_ALIGNMENT = 3,        /* pointer or stride not 16-byte aligned where the kernel needs it */
  NVA_ERR_WORKSPACE = 4,        /* workspace pointer null or smaller than *_workspace_bytes() */
  NVA_ERR_CUDA = 5,             /* a CUDA runtime/driver call failed (launch error, no device) */
} nva_status;

/* Library version, (major << 16) | minor. */
NVA_API int nva_version(void);

/* Static description of an nva_status value. */
NVA_API const char* nva_status_string(int status);

/* Text of the last CUDA error seen by this thread inside the library ("" if none). */
NVA_API const char* nva_last_cuda_error(void);

/*
 * (a) KV scatter.  Replaces store_kvcache / store_kvcache_kernel (nanovllm/layers/attention.py:10-40).
 * For every token i with slot = slot_mapping[i] != -1:
 *     k_cache.flat[slot * row_elems + j] = key[i * key_row_stride + j]   for j < row_elems
 * and the same for value/v_cache, where row_elems = num_kv_heads * head_dim.  Bit copy: any 2- or 4-byte
 * element type.  Slots outside [0, num_slots) are skipped and recorded in the device error word.
 */
NVA_API int nva_store_kvcache(const void* key, int64_t key_row_stride, const void* value, int64_t value_row_stride,
                              void* k_cache, void* v_cache, int64_t num_slots, const int32_t* slot_mapping,
                              int32_t num_tokens, int32_t num_kv_heads, int32_t head_dim, int32_t elem_bytes,
                              void* stream);

/*
 * (b)+(c) Paged decode / speculative-verify attention.  Replaces flash_attn_with_kvcache as called from
 * Attention.forward's decode branch (nanovllm/layers/attention.py:71-78):
 *     q [num_seqs, q_per_seq, H, D] -> out [num_seqs, q_per_seq, H, D], causal, bottom-right aligned:
 *     query i of sequence b attends to cache positions [0, context_lens[b] - q_per_seq + i].
 * context_lens include the q_per_seq new tokens (already stored by nva_store_kvcache).  A sequence with
 * context length 0 (batch padding) reads nothing and gets a zero output.  q_per_seq * (H / KVH) <= 48.
 * Requires head_dim 128, bf16, block_size a multiple of 128, softmax_scale positive and finite (else
 * NVA_ERR_INVALID_ARGUMENT; also for nva_varlen_attention and nva_paged_decode_noalloc).
 * workspace >= nva_paged_decode_workspace_bytes().
 * Workspace contract: zero-fill it once before its first use (cudaMemset); every call leaves its first 256-byte
 * aligned block of merge tickets at zero again, so the same workspace serves every later call in stream order (also
 * nva_varlen_attention calls, and captured CUDA graphs).  Calls that may overlap on one device (different streams)
 * need separate workspaces.
 */
NVA_API int nva_paged_decode(const void* q, int64_t q_row_stride, const void* k_cache, const void* v_cache,
                             int32_t num_blocks, int32_t block_size, const int32_t* context_lens,
                             const int32_t* block_tables, int32_t bt_row_stride, int32_t num_seqs, int32_t q_per_seq,
                             int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, float softmax_scale,
                             void* out, int64_t out_row_stride, void* workspace, size_t workspace_bytes,
                             void* stream);

NVA_API size_t nva_paged_decode_workspace_bytes(int32_t num_seqs, int32_t q_per_seq, int32_t num_heads,
                                                int32_t num_kv_heads, int32_t head_dim);

/*
 * (d) Varlen causal attention for prefill and mixed prefill+decode batches.  Replaces flash_attn_varlen_func
 * as called from Attention.forward's prefill branch (nanovllm/layers/attention.py:64-70).
 * Sequence b owns query rows [cu_seqlens_q[b], cu_seqlens_q[b+1]) and keys [0, Lk_b) with
 * Lk_b = cu_seqlens_k[b+1] - cu_seqlens_k[b]; query row i of the sequence attends to keys [0, Lk_b - Lq_b + i].
 * Keys/values come from the paged cache through block_tables when block_tables != NULL (prefix cache,
 * chunked prefill, mixed batches), else from the contiguous key/value tensors at rows cu_seqlens_k[b] + pos.
 * max_seqlen_q / max_seqlen_k are upper bounds only (they size nothing on the device).
 * Requires head_dim 128, bf16.  workspace >= nva_varlen_workspace_bytes(); same zero-filled-once contract as
 * nva_paged_decode's (the two may share one workspace).
 * The call enqueues up to three kernels on `stream` (the prefill work plan, the decode kernel for query runs of up
 * to 48 / group tokens, the prefill kernel for longer runs), each launched with a programmatic dependency on the one
 * before.  Together they keep the order of a single kernel: the first waits for the preceding work in the stream
 * before it touches memory, and the last completes only after the others.
 */
NVA_API int nva_varlen_attention(const void* q, int64_t q_row_stride, const void* key, int64_t key_row_stride,
                                 const void* value, int64_t value_row_stride, const void* k_cache,
                                 const void* v_cache, int32_t num_blocks, int32_t block_size,
                                 const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int32_t num_seqs,
                                 int32_t total_q, int32_t total_k, int32_t max_seqlen_q, int32_t max_seqlen_k,
                                 const int32_t* block_tables, int32_t bt_row_stride, int32_t num_heads,
                                 int32_t num_kv_heads, int32_t head_dim, float softmax_scale, void* out,
                                 int64_t out_row_stride, void* workspace, size_t workspace_bytes, void* stream);

NVA_API size_t nva_varlen_workspace_bytes(int32_t num_seqs, int32_t total_q, int32_t num_heads,
                                          int32_t num_kv_heads, int32_t head_dim);

/*
 * (c) Greedy accept length.  Replaces the greedy core of verify_drafts (nanovllm/layers/sampler.py:66-82) on
 * already-reduced target ids (row argmaxes of the verify logits):
 *     accepted[s, j] = target[s, j] == draft[s, j] && j < num_drafts[s]
 *     num_accepted[s] = length of the unbroken run of accepts from j = 0
 *     next_token[s]   = target[s, num_accepted[s]]
 * target [S, K+1], draft [S, K] (row strides in elements), num_drafts [S]; ids and outputs are int32 when
 * id_bytes == 4, int64 when id_bytes == 8 (num_drafts and num_accepted use the same width).  K may be 0.
 */
NVA_API int nva_greedy_accept(const void* target_ids, int64_t target_row_stride, const void* draft_ids,
                              int64_t draft_row_stride, const void* num_drafts, int32_t num_seqs, int32_t k,
                              int32_t id_bytes, void* num_accepted, void* next_tokens, void* stream);

/*
 * Qwen3's attention prologue in one pass.  Replaces, for every token, the q / k RMSNorm and rotary embedding of
 * Qwen3Attention.pre_attn (nanovllm/models/qwen3.py:88-97, layers/layernorm.py:16-26,
 * layers/rotary_embedding.py:6-14 and 37-48) and the KV scatter of Attention.forward (layers/attention.py:61-62):
 *   qkv [T, (H + 2 KVH) * D] bf16 (q heads, then k heads, then v heads; row stride in elements), positions [T] int64,
 *   cos_sin [max_position, D] float32 (cos of position p in columns [0, D/2), sin in [D/2, D)),
 *   q_norm_weight, k_norm_weight [D] bf16 ->
 *   q_out [T, H, D]:   rope(bf16(bf16(q * rsqrt(mean(q^2) + eps)) * q_norm_weight))
 *   k' (same with k_norm_weight), stored to k_out [T, KVH, D] when k_out != NULL,
 *   k_cache / v_cache rows (the nva_store_kvcache layout) at slot = slot_mapping[t] of k' and of v, when
 *   slot_mapping != NULL; slot -1 is skipped, slots past num_slots are skipped and set bit 1 of the error word.
 * rope: x1 = dims [0, D/2), x2 = dims [D/2, D): (x1 cos - x2 sin, x2 cos + x1 sin) in float32, rounded to bf16.
 * head_dim 128, num_heads + 2 * num_kv_heads <= 64.  Positions outside [0, max_position) are clamped.
 */
NVA_API int nva_qk_norm_rope_store(const void* qkv, int64_t qkv_row_stride, int32_t num_tokens, int32_t num_heads,
                                   int32_t num_kv_heads, int32_t head_dim, const int64_t* positions,
                                   const float* cos_sin, int32_t max_position, const void* q_norm_weight,
                                   const void* k_norm_weight, float eps, void* q_out, int64_t q_out_row_stride,
                                   void* k_out, int64_t k_out_row_stride, void* k_cache, void* v_cache,
                                   int64_t num_slots, const int32_t* slot_mapping, void* stream);

/*
 * Greedy verify from vocabulary shards.  Replaces, for all-greedy verify steps, the logits gather to rank 0 in
 * ParallelLMHead.forward (nanovllm/layers/embed_head.py:56-68) and the argmax + accept rule of verify_drafts
 * (nanovllm/layers/sampler.py:66-82).
 *
 * nva_shard_argmax: one rank's logits shard [rows, vocab_shard] (bf16 when elem_bytes == 2, float when 4, row
 * stride in elements) -> keys[rows], one uint64 per row:
 *     keys[r] = orderable(max_j logits[r, j]) << 32 | (0xFFFFFFFF - (vocab_offset + first j of that maximum))
 * where orderable() maps floats to unsigned integers in order (NaN above +inf, -0 equal to +0).  The largest key
 * over all shards names the argmax of the concatenated row with torch's tie rule (lowest index).  keys are
 * cleared in stream order by the call (one memset node, then the kernel).  rows <= 65535,
 * vocab_offset + vocab_shard < 2^32.
 *
 * nva_shard_accept: keys [num_shards, num_seqs * (k+1)] (shard-major, e.g. gathered from every rank) -> the target
 * ids (the merged argmaxes) and the greedy accept rule of nva_greedy_accept on them: num_accepted[s] = unbroken run
 * of target[s, j] == draft[s, j] with j < num_drafts[s], next_token[s] = target[s, num_accepted[s]].  Ids are
 * int32 (id_bytes 4) or int64 (8).  k == 0 gives plain greedy sampling (next_token = argmax of the row).
 */
NVA_API int nva_shard_argmax(const void* logits, int64_t row_stride, int32_t rows, int32_t vocab_shard,
                             int64_t vocab_offset, int32_t elem_bytes, uint64_t* keys, void* stream);
NVA_API int nva_shard_accept(const uint64_t* keys, int32_t num_shards, int32_t num_seqs, int32_t k,
                             const void* draft_ids, int64_t draft_row_stride, const void* num_drafts, int32_t id_bytes,
                             void* num_accepted, void* next_tokens, void* stream);

/*
 * Paged decode / verify attention without a caller workspace.  No counterpart in the reference: nano-vllm always
 * lets flash-attn allocate.  Same arguments and results as nva_paged_decode, minus the workspace.
 * It serves callers that cannot allocate device memory -- code running inside an allocator hook or a host callback
 * (where a cudaMalloc would recurse or deadlock), runtimes that carve all memory out of an arena reserved at start-up,
 * embedders whose memory manager has no device allocation -- by keeping the split-KV partials in a fixed array
 * compiled into the library: NVA_NOALLOC_SCRATCH_BYTES per GPU, held by every GPU that loads the library until the
 * process exits.  The call itself allocates nothing (no cudaMalloc / cudaFree, no allocating library routine).
 *  - The first call on each device looks up the array's device address (cudaGetSymbolAddress, that device current)
 *    and caches it: make that first call before any stream capture.
 *  - A call needing more than NVA_NOALLOC_SCRATCH_BYTES (2 x SMs x rows x 129 x 4 bytes, rows = q_per_seq x
 *    num_heads / num_kv_heads rounded up to 16, 32 or 48) returns NVA_ERR_WORKSPACE before launching anything; on a
 *    148-SM B200 that admits up to 32 rows (decode, and verify with up to 7 drafts at 4 q heads per kv head).
 *  - All calls on a device share the array and leave their contents in it.  The caller never clears it: each call
 *    first issues a small memset of the array's merge tickets on `stream`, then the kernel (two operations in stream
 *    order).  Calls that overlap on the GPU (e.g. on two streams) race on the array and must be serialised by the
 *    caller.
 */
#define NVA_NOALLOC_SCRATCH_BYTES (6u << 20)
NVA_API int nva_paged_decode_noalloc(const void* q, int64_t q_row_stride, const void* k_cache, const void* v_cache,
                                     int32_t num_blocks, int32_t block_size, const int32_t* context_lens,
                                     const int32_t* block_tables, int32_t bt_row_stride, int32_t num_seqs,
                                     int32_t q_per_seq, int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                                     float softmax_scale, void* out, int64_t out_row_stride, void* stream);

/*
 * Device error word.  Kernels never trap: a slot or block id out of range, or a pipeline wait that ran past its
 * time limit, sets a bit here and the kernel skips the access or returns.  Reading it synchronises the device.
 * Bits: 1 = scatter slot out of range, 2 = pipeline wait timed out, 4 = block id out of range.
 */
NVA_API int nva_get_device_error(uint32_t* out_bits);
NVA_API int nva_clear_device_error(void);

#ifdef __cplusplus
}
#endif

#endif /* NVATTN_H */
