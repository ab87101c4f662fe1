"""Torch-facing wrappers over the C ABI, with the signatures of the calls nano-vllm makes on its attention path.

  store_kvcache(key, value, k_cache, v_cache, slot_mapping)        nanovllm/layers/attention.py:33-40
  flash_attn_with_kvcache(q, k_cache, v_cache, cache_seqlens=, block_table=, softmax_scale=, causal=True)
                                                                    flash-attn call at attention.py:75-77
  flash_attn_varlen_func(q, k, v, max_seqlen_q=, cu_seqlens_q=, max_seqlen_k=, cu_seqlens_k=, softmax_scale=,
                         causal=True, block_table=)                 flash-attn call at attention.py:67-70
  greedy_accept(target_ids, draft_ids, num_drafts)                  greedy core of verify_drafts, sampler.py:66-82

Every op runs on the caller's current CUDA stream, allocates only its output and never syncs.  The attention ops
share one workspace per device (split-KV partials and the merge tickets, see _workspace); there is no CPU path:
non-CUDA tensors raise.
"""
import torch

from . import _lib


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("nvattn ops run on CUDA tensors only (no CPU fallback)")


# device index -> the attention workspace in use; earlier (smaller) ones stay referenced because captured CUDA
# graphs hold their addresses
_WORKSPACES: dict[int, torch.Tensor] = {}
_RETIRED: list[torch.Tensor] = []


def _workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """The decode / varlen workspace of a device.  Its merge-ticket words must be zero when a call starts and every
    call leaves them zero, so it is allocated zero-filled once (grown, zero-filled, when a call needs more) and then
    reused by every call and every captured graph.  Calls on one device are ordered by the stream they run on:
    nano-vllm runs attention from one stream; concurrent streams on one device need their own workspaces through
    the C ABI.  Growing it while a CUDA graph is being captured would allocate from the graph's pool and record the
    zero-fill into every replay, so that raises instead: size it first with reserve_workspace (the nano-vllm drop-in
    does so when the KV cache is allocated)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _WORKSPACES.get(idx)
    if ws is None or ws.numel() < nbytes:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError(f"nvattn: the attention workspace of cuda:{idx} must grow to {nbytes} bytes during a "
                               "CUDA graph capture; call nvattn.ops.reserve_workspace(...) before capturing")
        if ws is not None:
            _RETIRED.append(ws)
        ws = torch.zeros(max(nbytes, 16), dtype=torch.uint8, device=device)
        _WORKSPACES[idx] = ws
    return ws


def reserve_workspace(max_num_seqs: int, max_num_tokens: int, num_heads: int, num_kv_heads: int,
                      head_dim: int = 128, device: torch.device | None = None) -> int:
    """Allocate (zero-filled) the workspace every later decode / verify / varlen call of up to max_num_seqs
    sequences and max_num_tokens query rows needs on `device`, so that no call, captured or not, allocates.
    Returns its size in bytes.  nano-vllm: max_num_seqs and max_num_batched_tokens of its Config."""
    device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    lib = _lib.load()
    with torch.cuda.device(device):
        need = max(lib.nva_varlen_workspace_bytes(max_num_seqs, max_num_tokens, num_heads, num_kv_heads, head_dim),
                   max(lib.nva_paged_decode_workspace_bytes(max_num_seqs, n, num_heads, num_kv_heads, head_dim)
                       for n in range(1, 49)))
    return _workspace(need, device).numel()


def reset_workspaces() -> None:
    """Zero-fill every workspace again.  A call that gave up on a pipeline wait (bit 2 of the device error word) may
    leave merge tickets non-zero, after which later calls could merge split pieces wrongly; call this (outside any
    graph capture, after clearing the error word) before going on."""
    for ws in list(_WORKSPACES.values()) + _RETIRED:
        ws.zero_()


def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  slot_mapping: torch.Tensor) -> None:
    """Scatter this step's K/V rows into the paged cache (attention.py:33-40; same asserts)."""
    N, num_heads, head_dim = key.shape
    D = num_heads * head_dim
    assert key.stride(-1) == 1 and value.stride(-1) == 1
    assert key.stride(1) == head_dim and value.stride(1) == head_dim
    assert k_cache.stride(1) == D and v_cache.stride(1) == D
    assert slot_mapping.numel() == N
    _need_cuda(key, value, k_cache, v_cache, slot_mapping)
    assert key.dtype == value.dtype == k_cache.dtype == v_cache.dtype
    assert k_cache.is_contiguous() and v_cache.is_contiguous()
    assert slot_mapping.dtype == torch.int32 and slot_mapping.is_contiguous()
    num_slots = k_cache.numel() // D
    _lib.check(_lib.load().nva_store_kvcache(
        key.data_ptr(), key.stride(0), value.data_ptr(), value.stride(0), k_cache.data_ptr(), v_cache.data_ptr(),
        num_slots, slot_mapping.data_ptr(), N, num_heads, head_dim, key.element_size(), _stream()),
        "store_kvcache")


def flash_attn_with_kvcache(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, cache_seqlens: torch.Tensor,
                            block_table: torch.Tensor, softmax_scale: float, causal: bool = True,
                            out: torch.Tensor | None = None) -> torch.Tensor:
    """Paged decode / verify attention.  q [B, n, H, D] bf16; k_cache/v_cache [NB, BS, KVH, D]; cache_seqlens
    [B] int32 (including the n new tokens); block_table [B, W] int32.  Causal, bottom-right aligned."""
    assert causal, "nano-vllm always calls with causal=True"
    B, n, H, D = q.shape
    NB, BS, KVH, _ = k_cache.shape
    _need_cuda(q, k_cache, v_cache, cache_seqlens, block_table)
    assert q.dtype == k_cache.dtype == v_cache.dtype == torch.bfloat16
    assert q.stride(-1) == 1 and q.stride(2) == D and q.stride(0) == n * q.stride(1)
    assert k_cache.is_contiguous() and v_cache.is_contiguous()
    assert cache_seqlens.dtype == torch.int32 and cache_seqlens.is_contiguous() and cache_seqlens.numel() == B
    assert block_table.dtype == torch.int32 and block_table.stride(-1) == 1 and block_table.shape[0] == B
    if out is None:
        out = torch.empty(B, n, H, D, dtype=q.dtype, device=q.device)
    else:   # rows are addressed as (b * n + i) * out.stride(1): the same layout rules as q
        _need_cuda(out)
        assert out.dtype == q.dtype and out.shape == q.shape and out.device == q.device
        assert out.stride(-1) == 1 and out.stride(2) == D and out.stride(0) == n * out.stride(1)
    lib = _lib.load()
    ws_bytes = lib.nva_paged_decode_workspace_bytes(B, n, H, KVH, D)
    if ws_bytes == 0:
        raise _lib.NvattnError(f"paged decode does not support q_per_seq={n} with {H // KVH} q heads per kv head")
    ws = _workspace(ws_bytes, q.device)
    _lib.check(lib.nva_paged_decode(
        q.data_ptr(), q.stride(1), k_cache.data_ptr(), v_cache.data_ptr(), NB, BS, cache_seqlens.data_ptr(),
        block_table.data_ptr(), block_table.stride(0), B, n, H, KVH, D, float(softmax_scale), out.data_ptr(),
        out.stride(1), ws.data_ptr(), ws_bytes, _stream()), "paged decode")
    return out


def flash_attn_varlen_func(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, max_seqlen_q: int,
                           cu_seqlens_q: torch.Tensor, max_seqlen_k: int, cu_seqlens_k: torch.Tensor,
                           softmax_scale: float, causal: bool = True, block_table: torch.Tensor | None = None,
                           out: torch.Tensor | None = None) -> torch.Tensor:
    """Varlen causal attention.  q [Tq, H, D]; with block_table, k/v are the paged caches [NB, BS, KVH, D],
    else contiguous [Tk, KVH, D] rows (any row stride).  max_seqlen_* are upper bounds only."""
    assert causal, "nano-vllm always calls with causal=True"
    Tq, H, D = q.shape
    _need_cuda(q, k, v, cu_seqlens_q, cu_seqlens_k, block_table)
    assert q.dtype == k.dtype == v.dtype == torch.bfloat16
    assert q.stride(-1) == 1 and q.stride(1) == D
    assert cu_seqlens_q.dtype == torch.int32 and cu_seqlens_k.dtype == torch.int32
    assert cu_seqlens_q.is_contiguous() and cu_seqlens_k.is_contiguous()
    B = cu_seqlens_q.numel() - 1
    if out is None:
        out = torch.empty(Tq, H, D, dtype=q.dtype, device=q.device)
    else:
        _need_cuda(out)
        assert out.dtype == q.dtype and out.shape == q.shape and out.device == q.device
        assert out.stride(-1) == 1 and out.stride(1) == D
    lib = _lib.load()
    if block_table is not None:
        NB, BS, KVH, _ = k.shape
        assert k.is_contiguous() and v.is_contiguous()
        assert block_table.dtype == torch.int32 and block_table.stride(-1) == 1
        kp, kst, vp, vst, Tk = 0, 0, 0, 0, 0
        kc, vc, bt, bts = k.data_ptr(), v.data_ptr(), block_table.data_ptr(), block_table.stride(0)
    else:
        Tk, KVH, _ = k.shape
        assert k.stride(-1) == 1 and k.stride(1) == D and v.stride(-1) == 1 and v.stride(1) == D
        NB, BS = 0, 0
        kp, kst, vp, vst = k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0)
        kc, vc, bt, bts = 0, 0, 0, 0
    ws_bytes = lib.nva_varlen_workspace_bytes(B, Tq, H, KVH, D)
    ws = _workspace(ws_bytes, q.device)
    _lib.check(lib.nva_varlen_attention(
        q.data_ptr(), q.stride(0), kp, kst, vp, vst, kc, vc, NB, BS, cu_seqlens_q.data_ptr(),
        cu_seqlens_k.data_ptr(), B, Tq, Tk, int(max_seqlen_q), int(max_seqlen_k), bt, bts, H, KVH, D,
        float(softmax_scale), out.data_ptr(), out.stride(0), ws.data_ptr(), ws_bytes, _stream()), "varlen attention")
    return out


def greedy_accept(target_ids: torch.Tensor, draft_ids: torch.Tensor, num_drafts: torch.Tensor):
    """Integer greedy accept length: target [S, K+1], drafts [S, K], num_drafts [S] (all int32 or all int64).
    Returns (num_accepted [S], next_token [S]) in the same dtype."""
    _need_cuda(target_ids, draft_ids, num_drafts)
    S, K1 = target_ids.shape
    K = K1 - 1
    dt = target_ids.dtype
    assert dt in (torch.int32, torch.int64) and draft_ids.dtype == dt and num_drafts.dtype == dt
    assert target_ids.stride(-1) == 1 and num_drafts.is_contiguous() and num_drafts.numel() == S
    assert draft_ids.shape == (S, K) and (K == 0 or draft_ids.stride(-1) == 1)
    acc = torch.empty(S, dtype=dt, device=target_ids.device)
    nxt = torch.empty(S, dtype=dt, device=target_ids.device)
    _lib.check(_lib.load().nva_greedy_accept(
        target_ids.data_ptr(), target_ids.stride(0), draft_ids.data_ptr() if K else 0, draft_ids.stride(0) if K else 0,
        num_drafts.data_ptr(), S, K, target_ids.element_size(), acc.data_ptr(), nxt.data_ptr(), _stream()),
        "greedy accept")
    return acc, nxt


def shard_argmax(logits: torch.Tensor, vocab_offset: int = 0) -> torch.Tensor:
    """Per-row argmax keys of one vocabulary shard of logits [rows, V_shard] (bf16 or float32, unit column stride):
    int64 [rows] holding orderable(max) << 32 | (0xFFFFFFFF - (vocab_offset + first index of the max)) as raw bits.
    The largest key of a row over all shards (compared as unsigned) is the row's argmax with torch's tie rule; see
    shard_accept.  Replaces the per-rank part of the logits gather + argmax (embed_head.py:56-68, sampler.py:66)."""
    _need_cuda(logits)
    assert logits.dim() == 2 and logits.stride(-1) == 1
    assert logits.dtype in (torch.bfloat16, torch.float32)
    rows, vocab = logits.shape
    keys = torch.empty(rows, dtype=torch.int64, device=logits.device)
    _lib.check(_lib.load().nva_shard_argmax(logits.data_ptr(), logits.stride(0), rows, vocab, int(vocab_offset),
                                            logits.element_size(), keys.data_ptr(), _stream()), "shard argmax")
    return keys


def shard_accept(keys: torch.Tensor, draft_ids: torch.Tensor, num_drafts: torch.Tensor):
    """Greedy accept from argmax keys: keys [num_shards, S, K+1] (int64 raw bits from shard_argmax of each shard,
    contiguous), draft_ids [S, K], num_drafts [S] (int32 or int64, same dtype).  Returns (num_accepted [S],
    next_token [S]) in that dtype: verify_drafts' greedy result (sampler.py:66-82) on the concatenated shards."""
    _need_cuda(keys, draft_ids, num_drafts)
    num_shards, S, K1 = keys.shape
    K = K1 - 1
    dt = draft_ids.dtype
    assert keys.dtype == torch.int64 and keys.is_contiguous()
    assert dt in (torch.int32, torch.int64) and num_drafts.dtype == dt
    assert num_drafts.is_contiguous() and num_drafts.numel() == S
    assert draft_ids.shape == (S, K) and (K == 0 or draft_ids.stride(-1) == 1)
    acc = torch.empty(S, dtype=dt, device=keys.device)
    nxt = torch.empty(S, dtype=dt, device=keys.device)
    _lib.check(_lib.load().nva_shard_accept(
        keys.data_ptr(), num_shards, S, K, draft_ids.data_ptr() if K else 0, draft_ids.stride(0) if K else 0,
        num_drafts.data_ptr(), draft_ids.element_size(), acc.data_ptr(), nxt.data_ptr(), _stream()), "shard accept")
    return acc, nxt


def qk_norm_rope_store(qkv: torch.Tensor, positions: torch.Tensor, cos_sin_cache: torch.Tensor,
                       q_norm_weight: torch.Tensor, k_norm_weight: torch.Tensor, eps: float, num_heads: int,
                       num_kv_heads: int, k_cache: torch.Tensor | None = None, v_cache: torch.Tensor | None = None,
                       slot_mapping: torch.Tensor | None = None, want_k: bool = False):
    """Qwen3's attention prologue in one kernel: from the fused projection output qkv [T, (H + 2 KVH) * 128], the
    normalised and rotated q [T, H, 128] (returned), the same for k (returned when want_k, else None), and, with a
    cache, k and v scattered to slot_mapping's slots (qwen3.py:88-97 then attention.py:61-62).  cos_sin_cache is the
    reference RotaryEmbedding's [max_position, 1 or none, 128] float32 table.  Returns (q, k, v) with v a view of
    qkv, as Qwen3Attention.pre_attn returns them."""
    _need_cuda(qkv, positions, cos_sin_cache, q_norm_weight, k_norm_weight)
    D = 128
    T = qkv.shape[0]
    assert qkv.dim() == 2 and qkv.shape[1] == (num_heads + 2 * num_kv_heads) * D and qkv.stride(1) == 1
    assert qkv.dtype == torch.bfloat16 and q_norm_weight.dtype == k_norm_weight.dtype == torch.bfloat16
    assert positions.dtype == torch.int64 and positions.is_contiguous() and positions.numel() == T
    table = cos_sin_cache.reshape(-1, D)
    assert table.dtype == torch.float32 and table.is_contiguous()
    q = torch.empty(T, num_heads, D, dtype=qkv.dtype, device=qkv.device)
    k = torch.empty(T, num_kv_heads, D, dtype=qkv.dtype, device=qkv.device) if want_k else None
    if slot_mapping is not None:
        _need_cuda(k_cache, v_cache, slot_mapping)
        assert slot_mapping.dtype == torch.int32 and slot_mapping.is_contiguous() and slot_mapping.numel() == T
        assert k_cache.is_contiguous() and v_cache.is_contiguous() and k_cache.dtype == qkv.dtype
        assert k_cache.stride(1) == num_kv_heads * D
        num_slots = k_cache.numel() // (num_kv_heads * D)
    else:
        num_slots = 0
    _lib.check(_lib.load().nva_qk_norm_rope_store(
        qkv.data_ptr(), qkv.stride(0), T, num_heads, num_kv_heads, D, positions.data_ptr(), table.data_ptr(),
        table.shape[0], q_norm_weight.data_ptr(), k_norm_weight.data_ptr(), float(eps), q.data_ptr(), q.stride(0),
        k.data_ptr() if k is not None else 0, k.stride(0) if k is not None else 0,
        k_cache.data_ptr() if slot_mapping is not None else 0, v_cache.data_ptr() if slot_mapping is not None else 0,
        num_slots, slot_mapping.data_ptr() if slot_mapping is not None else 0, _stream()), "qk norm rope store")
    v = qkv[:, (num_heads + num_kv_heads) * D:].view(T, num_kv_heads, D)
    return q, k, v
