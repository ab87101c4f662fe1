"""Drop-in replacement for nanovllm/layers/attention.py (Attention, store_kvcache) on B200.

Same constructor, attributes and forward contract as the reference's Attention (attention.py:43-79):
  * __init__(num_heads, head_dim, scale, num_kv_heads); k_cache / v_cache start empty and are assigned by
    ModelRunner.allocate_kv_cache (model_runner.py:258-267) as views [NB, BS, KVH, D] of one pool;
  * forward(q [T, H, D], k [T, KVH, D], v [T, KVH, D]) -> o [T, H, D], reading everything else from the
    per-step Context: slot_mapping for the KV scatter (skipped while the cache is empty, e.g. warmup),
    then either the varlen branch (is_prefill; paged cache when block_tables is set) or the decode / verify
    branch (every sequence brings T / num_seqs query tokens, causal bottom-right over context_lens).
The work runs in libnvattn.so kernels on the current stream; nothing here syncs or reads device values, so the
decode branch can be captured in CUDA graphs exactly as the reference's is.
"""
import torch
from torch import nn

from .context import get_context
from . import ops
from .ops import store_kvcache  # noqa: F401  (same name as the reference module exports)


class Attention(nn.Module):

    def __init__(self, num_heads, head_dim, scale, num_kv_heads):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.scale = scale
        self.num_kv_heads = num_kv_heads
        self.k_cache = self.v_cache = torch.tensor([])

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
        context = get_context()
        k_cache, v_cache = self.k_cache, self.v_cache
        if k_cache.numel() and v_cache.numel():
            ops.store_kvcache(k, v, k_cache, v_cache, context.slot_mapping)
        return self.forward_stored(q, k, v)

    def forward_stored(self, q: torch.Tensor, k: torch.Tensor | None, v: torch.Tensor | None):
        """forward() for a step whose K/V rows are already in the cache (written by the fused prologue,
        ops.qk_norm_rope_store).  k and v are read only by a prefill without a block table (contiguous K/V);
        otherwise they may be None."""
        context = get_context()
        k_cache, v_cache = self.k_cache, self.v_cache
        if context.is_prefill:
            if context.block_tables is not None:    # prefix cache / chunked prefill / mixed batch
                k, v = k_cache, v_cache
            o = ops.flash_attn_varlen_func(q, k, v, max_seqlen_q=context.max_seqlen_q,
                                           cu_seqlens_q=context.cu_seqlens_q, max_seqlen_k=context.max_seqlen_k,
                                           cu_seqlens_k=context.cu_seqlens_k, softmax_scale=self.scale, causal=True,
                                           block_table=context.block_tables)
        else:    # decode: every sequence brings the same number of query tokens (1, or 1+k when verifying)
            num_seqs = context.context_lens.size(0)
            q = q.reshape(num_seqs, -1, self.num_heads, self.head_dim)
            o = ops.flash_attn_with_kvcache(q, k_cache, v_cache, cache_seqlens=context.context_lens,
                                            block_table=context.block_tables, softmax_scale=self.scale, causal=True)
            o = o.view(-1, self.num_heads, self.head_dim)
        return o
