/*
 * CPU oracle for the integer / byte parts of the attention hot path.  TEST INFRASTRUCTURE ONLY: the product
 * never links or calls this; tests, smoke() and bench.py's cpu_baseline use it as the checker.
 *
 * oracle_store_kvcache follows store_kvcache_kernel / store_kvcache (nanovllm/layers/attention.py:10-40).
 * oracle_greedy_accept follows the greedy core of verify_drafts (nanovllm/layers/sampler.py:66-82).
 */
#include <stdint.h>
#include <string.h>

/* attention.py:21-30: one program per token; slot == -1 skips the token; otherwise the D = KVH*head_dim
 * contiguous elements of key row i / value row i are copied to cache row `slot`. Bit copy of elem_bytes. */
int oracle_store_kvcache(const uint8_t* key, int64_t key_row_stride, const uint8_t* value, int64_t value_row_stride,
                         uint8_t* k_cache, uint8_t* v_cache, int64_t num_slots, const int32_t* slot_mapping,
                         int32_t num_tokens, int32_t row_elems, int32_t elem_bytes) {
  int skipped = 0;
  const int64_t row_bytes = (int64_t)row_elems * elem_bytes;
  for (int32_t i = 0; i < num_tokens; ++i) {
    const int64_t slot = slot_mapping[i];
    if (slot == -1) continue;                 /* attention.py:23 */
    if (slot < 0 || slot >= num_slots) {      /* the Triton kernel would write out of bounds; count instead */
      ++skipped;
      continue;
    }
    memcpy(k_cache + slot * row_bytes, key + (int64_t)i * key_row_stride * elem_bytes, (size_t)row_bytes);
    memcpy(v_cache + slot * row_bytes, value + (int64_t)i * value_row_stride * elem_bytes, (size_t)row_bytes);
  }
  return skipped;
}

/* sampler.py:66-82 (greedy rows): accepted = top1[:, :K] == drafts; accepted &= j < num_drafts;
 * num_accepted = cumprod(accepted).sum(); next = top1[s, num_accepted]. */
void oracle_greedy_accept(const int64_t* target, int64_t target_row_stride, const int64_t* drafts,
                          int64_t draft_row_stride, const int64_t* num_drafts, int32_t num_seqs, int32_t k,
                          int64_t* num_accepted, int64_t* next_token) {
  for (int32_t s = 0; s < num_seqs; ++s) {
    int64_t a = 0;
    for (int32_t j = 0; j < k; ++j) {
      const int ok = target[s * target_row_stride + j] == drafts[s * draft_row_stride + j] && j < num_drafts[s];
      if (!ok) break;   /* cumprod turns the first reject into zeros for the rest of the row */
      ++a;
    }
    num_accepted[s] = a;
    next_token[s] = target[s * target_row_stride + a];
  }
}
