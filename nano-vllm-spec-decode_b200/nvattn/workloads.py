"""Seeded synthetic inputs for the five BASELINE configurations of the attention hot path.

All random values come from a CPU torch.Generator seeded per workload, so a CPU checker and the GPU see the same
numbers.  KV content is generated only for the blocks a sequence uses, block by block in sequence order, and
written straight into the paged pool on the target device; unused pool blocks are zero.  Shapes follow
Qwen3 (head_dim 128, block size 256) and the Context layout nano-vllm's ModelRunner builds
(model_runner.py:276-362 for prefill/decode, :31-63 for mixed batches).
"""
from dataclasses import dataclass, field
import math

import torch

BLOCK_SIZE = 256


@dataclass
class PagedBatch:
    """One attention step over a paged KV pool (the fields of nanovllm.utils.context.Context plus tensors)."""
    q: torch.Tensor                      # [T_q, H, D]
    k_new: torch.Tensor                  # [T_q, KVH, D] this step's keys (already stored in the cache)
    v_new: torch.Tensor                  # [T_q, KVH, D]
    k_cache: torch.Tensor                # [NB, BS, KVH, D]
    v_cache: torch.Tensor
    slot_mapping: torch.Tensor           # [T_q] int32
    block_tables: torch.Tensor           # [B, W] int32, -1 padded
    context_lens: torch.Tensor | None    # [B] int32 (decode / verify)
    cu_seqlens_q: torch.Tensor | None    # [B+1] int32 (varlen)
    cu_seqlens_k: torch.Tensor | None
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    q_per_seq: int = 1
    scale: float = 1.0 / math.sqrt(128)
    meta: dict = field(default_factory=dict)

    @property
    def num_seqs(self) -> int:
        return self.block_tables.shape[0]


def _table(gen, num_blocks: int, lens: list[int], width: int | None = None, block_size: int = BLOCK_SIZE):
    """Distinct random block ids per sequence: one seeded permutation of the pool, sliced in sequence order."""
    need = [(L + block_size - 1) // block_size for L in lens]
    assert sum(need) <= num_blocks, (sum(need), num_blocks)
    perm = torch.randperm(num_blocks, generator=gen).to(torch.int32)
    W = max([1] + need) if width is None else width
    table = torch.full((len(lens), W), -1, dtype=torch.int32)
    pos = 0
    for b, n in enumerate(need):
        table[b, :n] = perm[pos:pos + n]
        pos += n
    return table


def _fill_cache(gen, k_cache, v_cache, table, lens, std, block_size=BLOCK_SIZE):
    """Random K/V for every block a sequence uses (whole blocks, so the tail past the length holds finite
    stale values, like a reused block).  With a device generator the whole pool is filled on the device
    (fast; used by the benchmark, whose numbers do not depend on the values)."""
    KVH, D = k_cache.shape[2], k_cache.shape[3]
    if gen.device.type != "cpu":
        k_cache.normal_(0.0, std, generator=gen)
        v_cache.normal_(0.0, std, generator=gen)
        return
    for b, L in enumerate(lens):
        n = (L + block_size - 1) // block_size
        if n == 0:
            continue
        ids = table[b, :n].long().to(k_cache.device)
        kv = torch.randn(2, n, block_size, KVH, D, generator=gen) * std
        k_cache[ids] = kv[0].to(k_cache.dtype).to(k_cache.device)
        v_cache[ids] = kv[1].to(v_cache.dtype).to(v_cache.device)


def _slots(table, starts, ends, block_size=BLOCK_SIZE):
    out = []
    for b, (s, e) in enumerate(zip(starts, ends)):
        out.extend(int(table[b, p // block_size]) * block_size + p % block_size for p in range(s, e))
    return torch.tensor(out, dtype=torch.int32)


def paged_decode_batch(lens: list[int], q_per_seq: int = 1, num_heads: int = 32, num_kv_heads: int = 8,
                       head_dim: int = 128, num_blocks: int = 2048, std: float = 0.5, seed: int = 0,
                       dtype=torch.bfloat16, device="cpu", width: int | None = None, pad_seqs: int = 0,
                       device_fill: bool = False) -> PagedBatch:
    """Decode / verify step: every sequence brings q_per_seq query tokens whose KV is already in the cache
    at positions [len - q_per_seq, len) (prepare_decode, model_runner.py:319-362).  pad_seqs appends empty
    sequences (length 0, table -1, slot -1) like graph-bucket padding."""
    gen = torch.Generator().manual_seed(seed)
    B = len(lens)
    k_cache = torch.zeros(num_blocks, BLOCK_SIZE, num_kv_heads, head_dim, dtype=dtype, device=device)
    v_cache = torch.zeros_like(k_cache)
    table = _table(gen, num_blocks, lens, width)
    _fill_cache(torch.Generator(device).manual_seed(seed) if device_fill else gen, k_cache, v_cache, table, lens, std)
    T = B * q_per_seq
    q = (torch.randn(T, num_heads, head_dim, generator=gen) * std).to(dtype)
    slots = _slots(table, [L - q_per_seq for L in lens], lens)
    k_new = k_cache.view(-1, num_kv_heads, head_dim)[slots.long().to(device)].cpu()
    v_new = v_cache.view(-1, num_kv_heads, head_dim)[slots.long().to(device)].cpu()
    ctx = torch.tensor(lens, dtype=torch.int32)
    if pad_seqs:
        table = torch.cat([table, torch.full((pad_seqs, table.shape[1]), -1, dtype=torch.int32)])
        ctx = torch.cat([ctx, torch.zeros(pad_seqs, dtype=torch.int32)])
        q = torch.cat([q, torch.zeros(pad_seqs * q_per_seq, num_heads, head_dim, dtype=dtype)])
        k_new = torch.cat([k_new, torch.zeros(pad_seqs * q_per_seq, num_kv_heads, head_dim, dtype=dtype)])
        v_new = torch.cat([v_new, torch.zeros(pad_seqs * q_per_seq, num_kv_heads, head_dim, dtype=dtype)])
        slots = torch.cat([slots, torch.full((pad_seqs * q_per_seq,), -1, dtype=torch.int32)])
    return PagedBatch(q=q.to(device), k_new=k_new.to(device), v_new=v_new.to(device), k_cache=k_cache,
                      v_cache=v_cache, slot_mapping=slots.to(device), block_tables=table.to(device),
                      context_lens=ctx.to(device), cu_seqlens_q=None, cu_seqlens_k=None, q_per_seq=q_per_seq,
                      scale=1.0 / math.sqrt(head_dim), meta=dict(lens=list(lens)))


def decode_config(seed: int = 0, device="cpu", B: int = 64, num_heads: int = 32, num_kv_heads: int = 8,
                  num_blocks: int = 2048, device_fill: bool = False) -> PagedBatch:
    """Qwen3-8B decode, B=64, context U[512, 4096], pool 2048 blocks, N(0,1)*0.5."""
    gen = torch.Generator().manual_seed(seed)
    lens = torch.randint(512, 4097, (B,), generator=gen).tolist()
    return paged_decode_batch(lens, 1, num_heads, num_kv_heads, 128, num_blocks, 0.5, seed + 1, device=device,
                              device_fill=device_fill)


def verify_config(k: int, seed: int = 0, device="cpu", B: int = 32, num_heads: int = 32, num_kv_heads: int = 8,
                  num_blocks: int = 2048, device_fill: bool = False) -> PagedBatch:
    """BASELINE config 3 (attention part): B=32, context U[256, 2048], k+1 query tokens per sequence."""
    gen = torch.Generator().manual_seed(seed)
    lens = torch.randint(256, 2049, (B,), generator=gen).tolist()
    return paged_decode_batch(lens, k + 1, num_heads, num_kv_heads, 128, num_blocks, 0.5, seed + 1, device=device,
                              device_fill=device_fill)


def accept_config(k: int, S: int = 32, p_match: float = 0.7, vocab: int = 151936, seed: int = 0):
    """BASELINE config 3 (accept part): int32 target argmax ids [S, k+1] and draft ids [S, k]; each draft equals
    the target at its position with probability p_match, else a different random id.  num_drafts = k."""
    gen = torch.Generator().manual_seed(seed)
    target = torch.randint(0, vocab, (S, k + 1), generator=gen, dtype=torch.int64)
    other = torch.randint(1, vocab, (S, k), generator=gen, dtype=torch.int64)
    match = torch.rand(S, k, generator=gen) < p_match
    drafts = torch.where(match, target[:, :k], (target[:, :k] + other) % vocab)
    num_drafts = torch.full((S,), k, dtype=torch.int64)
    return target.to(torch.int32), drafts.to(torch.int32), num_drafts.to(torch.int32)


def varlen_batch(q_lens: list[int], k_lens: list[int], num_heads: int = 32, num_kv_heads: int = 8,
                 head_dim: int = 128, num_blocks: int = 2048, std: float = 0.5, seed: int = 0,
                 dtype=torch.bfloat16, device="cpu", paged: bool = True) -> PagedBatch:
    """Varlen step (prepare_prefill / mixed_batch layout): sequence b brings q_lens[b] query tokens at
    positions [k_lens[b] - q_lens[b], k_lens[b]); all of its KV is in the paged cache (paged=True) or, for a
    prefill without prefix (paged=False, q_len == k_len), in contiguous k/v rows cu_seqlens_k[b] + pos."""
    gen = torch.Generator().manual_seed(seed)
    B = len(q_lens)
    assert all(0 <= q <= k for q, k in zip(q_lens, k_lens))
    k_cache = torch.zeros(num_blocks, BLOCK_SIZE, num_kv_heads, head_dim, dtype=dtype, device=device)
    v_cache = torch.zeros_like(k_cache)
    table = _table(gen, num_blocks, k_lens)
    _fill_cache(gen, k_cache, v_cache, table, k_lens, std)
    Tq = sum(q_lens)
    q = (torch.randn(Tq, num_heads, head_dim, generator=gen) * std).to(dtype)
    slots = _slots(table, [k - q for q, k in zip(q_lens, k_lens)], k_lens)
    k_new = k_cache.view(-1, num_kv_heads, head_dim)[slots.long().to(device)].cpu()
    v_new = v_cache.view(-1, num_kv_heads, head_dim)[slots.long().to(device)].cpu()
    cu_q = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0).tolist()), dtype=torch.int32)
    cu_k = torch.tensor([0] + list(torch.tensor(k_lens).cumsum(0).tolist()), dtype=torch.int32)
    if not paged:
        assert q_lens == k_lens, "contiguous K/V only without a prefix (prepare_prefill without block_tables)"
    return PagedBatch(q=q.to(device), k_new=k_new.to(device), v_new=v_new.to(device), k_cache=k_cache,
                      v_cache=v_cache, slot_mapping=slots.to(device),
                      block_tables=table.to(device) if paged else table[:, :0].to(device), context_lens=None,
                      cu_seqlens_q=cu_q.to(device), cu_seqlens_k=cu_k.to(device), max_seqlen_q=max(q_lens),
                      max_seqlen_k=max(k_lens), scale=1.0 / math.sqrt(head_dim),
                      meta=dict(q_lens=list(q_lens), k_lens=list(k_lens), paged=paged))


def mixed_config(seed: int = 0, device="cpu", num_heads: int = 32, num_kv_heads: int = 8,
                 num_blocks: int = 2048) -> PagedBatch:
    """2048-token mixed step.  Decode rows first (run_mixed orders decode before prefill,
    model_runner.py:512): 256 decode sequences, q_len 1, context log-normal(median 600, sigma 0.8) clamped to
    [16, 4096]; then three prefill chunks of 512, 640, 640 new tokens with prefixes 0, 256, 1024."""
    gen = torch.Generator().manual_seed(seed)
    z = torch.randn(256, generator=gen, dtype=torch.float64)
    dec = torch.exp(math.log(600.0) + 0.8 * z).round().clamp(16, 4096).long().tolist()
    chunks, prefixes = [512, 640, 640], [0, 256, 1024]
    q_lens = [1] * 256 + chunks
    k_lens = dec + [c + p for c, p in zip(chunks, prefixes)]
    b = varlen_batch(q_lens, k_lens, num_heads, num_kv_heads, 128, num_blocks, 0.5, seed + 1, device=device)
    b.meta.update(num_decode=256, chunks=chunks, prefixes=prefixes)
    return b


def config1(seed: int = 0) -> dict:
    """BASELINE config 0 (CPU-runnable reference): Qwen3-0.6B attention shape in fp32, 4 sequences with context
    lengths 37, 256, 513, 1000 over a 64-block pool; each block table a seeded random slice of distinct ids;
    q, k, v ~ N(0, 1); the 4 new tokens are scattered with slot = block_id * 256 + offset."""
    lens = [37, 256, 513, 1000]
    b = paged_decode_batch(lens, 1, 16, 8, 128, 64, 1.0, seed, dtype=torch.float32)
    return dict(batch=b, lens=lens)


def flops_decode(lens, q_per_seq, num_heads, head_dim=128) -> float:
    """Algorithmic FLOPs of causal paged attention: 4*H*D per visible (query, key) pair."""
    n = q_per_seq
    pairs = sum(n * L - n * (n - 1) // 2 for L in lens if L > 0)
    return 4.0 * num_heads * head_dim * pairs


def bytes_decode(lens, q_per_seq, num_heads, num_kv_heads, head_dim=128, elem=2) -> float:
    """Algorithmic HBM bytes of paged decode: each visible K/V row once per kv head, plus q and o."""
    kv = sum(lens) * 2 * num_kv_heads * head_dim * elem
    qo = 2 * len(lens) * q_per_seq * num_heads * head_dim * elem
    return float(kv + qo)


def shard_heads(b: PagedBatch, rank: int, world: int) -> PagedBatch:
    """Rank `rank`'s tensor-parallel shard of a batch (qwen3.py:29-39 head split; model_runner.py:251 cache of
    num_kv_heads // world heads): q heads [r*H/t, (r+1)*H/t) and kv heads [r*KVH/t, (r+1)*KVH/t).  The block tables,
    slots and lengths are shared by all ranks."""
    H, KVH = b.q.shape[1], b.k_cache.shape[2]
    assert H % world == 0 and KVH % world == 0
    h0, h1 = rank * H // world, (rank + 1) * H // world
    k0, k1 = rank * KVH // world, (rank + 1) * KVH // world
    return PagedBatch(q=b.q[:, h0:h1].contiguous(), k_new=b.k_new[:, k0:k1].contiguous(),
                      v_new=b.v_new[:, k0:k1].contiguous(), k_cache=b.k_cache[:, :, k0:k1].contiguous(),
                      v_cache=b.v_cache[:, :, k0:k1].contiguous(), slot_mapping=b.slot_mapping,
                      block_tables=b.block_tables, context_lens=b.context_lens, cu_seqlens_q=b.cu_seqlens_q,
                      cu_seqlens_k=b.cu_seqlens_k, max_seqlen_q=b.max_seqlen_q, max_seqlen_k=b.max_seqlen_k,
                      q_per_seq=b.q_per_seq, scale=b.scale, meta=dict(b.meta, rank=rank, world=world))
