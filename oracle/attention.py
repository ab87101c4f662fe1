"""FP32 torch restatement of the attention hot path (test infrastructure only, see oracle/__init__.py).

Follows nanovllm/layers/attention.py:59-79 (Attention.forward) and the semantics flash-attn 2.8.3 documents for
the two calls it makes:
  * flash_attn_with_kvcache (decode / verify, attention.py:71-78): q [B, n, H, D] against the paged cache
    [NB, BS, KVH, D] through block_table [B, W]; cache_seqlens = context_lens include the n new tokens;
    causal mask aligned to the bottom right, so query i sees positions [0, len - n + i].
  * flash_attn_varlen_func (prefill / mixed, attention.py:64-70): q rows [cu_q[b], cu_q[b+1]), keys
    [0, Lk_b) from the contiguous k/v (block_table None) or the paged cache; causal bottom-right.
GQA: q head h uses kv head h // (H // KVH).  Softmax in FP32 with `scale`.  A query row with no visible key
gets a zero output ("If the row of the mask is all zero, the output will be zero").
"""
import numpy as np
import torch


def _gather_paged(cache: torch.Tensor, table_row: torch.Tensor, length: int) -> torch.Tensor:
    """Positions [0, length) of one sequence from the paged cache: block = table[p // BS], row p % BS
    (model_runner.py:338 slot rule)."""
    BS = cache.shape[1]
    nblk = (length + BS - 1) // BS
    blocks = table_row[:nblk].long()
    return cache[blocks].reshape(nblk * BS, *cache.shape[2:])[:length]


def _attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """q [n, H, D], k/v [L, KVH, D] (fp32) -> [n, H, D]; causal bottom-right over the L keys."""
    n, H, D = q.shape
    L, KVH, _ = k.shape
    G = H // KVH
    out = torch.zeros(n, H, D, dtype=torch.float32)
    if L == 0 or n == 0:
        return out
    kh = k.permute(1, 0, 2).repeat_interleave(G, dim=0)   # [H, L, D]: head h -> kv head h // G
    vh = v.permute(1, 0, 2).repeat_interleave(G, dim=0)
    s = torch.einsum("nhd,hld->hnl", q, kh) * scale        # [H, n, L]
    qi = torch.arange(n).unsqueeze(1)
    kj = torch.arange(L).unsqueeze(0)
    visible = kj <= (L - n + qi)                           # bottom-right aligned causal mask
    s = s.masked_fill(~visible.unsqueeze(0), float("-inf"))
    m = s.amax(dim=-1, keepdim=True)
    any_visible = visible.any(dim=-1)                      # [n]
    m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    p = torch.exp(s - m)
    l = p.sum(dim=-1, keepdim=True)
    o = torch.einsum("hnl,hld->nhd", p / torch.where(l > 0, l, torch.ones_like(l)), vh)
    return torch.where(any_visible.view(n, 1, 1), o, torch.zeros_like(o))


def paged_attention_ref(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, context_lens: torch.Tensor,
                        block_tables: torch.Tensor, scale: float) -> torch.Tensor:
    """flash_attn_with_kvcache(q, k_cache, v_cache, cache_seqlens=context_lens, block_table=block_tables,
    softmax_scale=scale, causal=True) restated in FP32.  q [B, n, H, D] -> [B, n, H, D] fp32."""
    B, n, H, D = q.shape
    out = torch.zeros(B, n, H, D, dtype=torch.float32)
    for b in range(B):
        L = int(context_lens[b])
        if L <= 0:
            continue
        k = _gather_paged(k_cache, block_tables[b], L).float()
        v = _gather_paged(v_cache, block_tables[b], L).float()
        out[b] = _attend(q[b].float(), k, v, scale)
    return out


def varlen_attention_ref(q: torch.Tensor, k: torch.Tensor | None, v: torch.Tensor | None, cu_seqlens_q: torch.Tensor,
                         cu_seqlens_k: torch.Tensor, scale: float, block_tables: torch.Tensor | None = None,
                         k_cache: torch.Tensor | None = None, v_cache: torch.Tensor | None = None) -> torch.Tensor:
    """flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, ..., softmax_scale=scale, causal=True,
    block_table=block_tables) restated in FP32.  With block_tables the keys come from k_cache/v_cache
    (attention.py:65-66).  q [Tq, H, D] -> [Tq, H, D] fp32."""
    Tq, H, D = q.shape
    out = torch.zeros(Tq, H, D, dtype=torch.float32)
    cq = cu_seqlens_q.tolist()
    ck = cu_seqlens_k.tolist()
    for b in range(len(cq) - 1):
        q0, q1 = cq[b], cq[b + 1]
        Lk = ck[b + 1] - ck[b]
        if q1 == q0:
            continue
        if block_tables is not None:
            kb = _gather_paged(k_cache, block_tables[b], Lk).float()
            vb = _gather_paged(v_cache, block_tables[b], Lk).float()
        else:
            kb = k[ck[b]:ck[b + 1]].float()
            vb = v[ck[b]:ck[b + 1]].float()
        out[q0:q1] = _attend(q[q0:q1].float(), kb, vb, scale)
    return out


def store_kvcache_ref(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                      slot_mapping: torch.Tensor) -> None:
    """store_kvcache (attention.py:33-40) as torch indexing on CPU: rows with slot -1 are skipped."""
    N, KVH, D = key.shape
    keep = slot_mapping.long() != -1
    slots = slot_mapping.long()[keep]
    k_cache.view(-1, KVH, D)[slots] = key[keep]
    v_cache.view(-1, KVH, D)[slots] = value[keep]


def greedy_accept_ref(target: np.ndarray, drafts: np.ndarray, num_drafts: np.ndarray):
    """verify_drafts greedy core (sampler.py:66-82) in numpy: returns (num_accepted, next_token) int64."""
    target = np.asarray(target, dtype=np.int64)
    S, K1 = target.shape
    K = K1 - 1
    drafts = np.asarray(drafts, dtype=np.int64).reshape(S, K)
    accepted = (target[:, :K] == drafts) & (np.arange(K)[None, :] < np.asarray(num_drafts)[:, None])
    num_accepted = np.cumprod(accepted.astype(np.int64), axis=1).sum(axis=1) if K else np.zeros(S, np.int64)
    next_token = target[np.arange(S), num_accepted]
    return num_accepted.astype(np.int64), next_token.astype(np.int64)
