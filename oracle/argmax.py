"""Numpy restatement of greedy verify over vocabulary shards (test infrastructure only, see oracle/__init__.py).

The reference gathers every rank's logits shard to rank 0 (nanovllm/layers/embed_head.py:56-68), takes the row
argmax of the concatenation (sampler.py:66, torch's argmax: the first index of the maximum, NaN above every number,
-0 equal to +0) and applies the greedy accept rule (sampler.py:79-82).  The sharded form computes per shard one key
per row, key = orderable(max) << 32 | (0xFFFFFFFF - global index of the first maximum), merges the shards by the
largest key and reads the index back; shard_argmax_keys and merge_keys restate that, argmax_ref is the unsharded
rule it must equal, accept_from_keys the accept rule on the merged ids.
"""
import numpy as np


def orderable(values: np.ndarray) -> np.ndarray:
    """float32 -> uint32 in the same order (NaN above +inf, -0 mapped to +0's value)."""
    v = np.asarray(values, dtype=np.float32).copy()
    v[np.isnan(v)] = np.float32(np.nan)
    u = v.view(np.uint32).copy()
    u[np.isnan(v)] = 0x7FC00000
    u[u == 0x80000000] = 0
    neg = (u & 0x80000000) != 0
    return np.where(neg, ~u, u | 0x80000000).astype(np.uint32)


def argmax_ref(logits: np.ndarray) -> np.ndarray:
    """Row argmax with torch's rule (first index of the maximum, NaN counts as the largest)."""
    x = np.asarray(logits, dtype=np.float32)
    out = np.empty(x.shape[0], dtype=np.int64)
    for r in range(x.shape[0]):
        nan = np.flatnonzero(np.isnan(x[r]))
        out[r] = nan[0] if len(nan) else int(np.argmax(x[r]))
    return out


def shard_argmax_keys(logits_shard: np.ndarray, vocab_offset: int) -> np.ndarray:
    """uint64 [rows]: orderable(row max) << 32 | (0xFFFFFFFF - (vocab_offset + first index of the max))."""
    x = np.asarray(logits_shard, dtype=np.float32)
    idx = argmax_ref(x)
    best = x[np.arange(x.shape[0]), idx]
    hi = orderable(best).astype(np.uint64) << np.uint64(32)
    lo = (np.uint64(0xFFFFFFFF) - (np.uint64(vocab_offset) + idx.astype(np.uint64)))
    return hi | lo


def merge_keys(keys: np.ndarray) -> np.ndarray:
    """keys [num_shards, rows] uint64 -> global argmax ids [rows] (int64)."""
    best = np.asarray(keys, dtype=np.uint64).max(axis=0)
    return (np.uint64(0xFFFFFFFF) - (best & np.uint64(0xFFFFFFFF))).astype(np.int64)


def accept_from_keys(keys: np.ndarray, drafts: np.ndarray, num_drafts: np.ndarray):
    """keys [num_shards, S, K+1] -> (num_accepted [S], next_token [S]) by sampler.py:79-82 on the merged ids."""
    nsh, S, K1 = keys.shape
    target = merge_keys(keys.reshape(nsh, S * K1)).reshape(S, K1)
    acc = np.zeros(S, dtype=np.int64)
    nxt = np.zeros(S, dtype=np.int64)
    for s in range(S):
        a = 0
        while a < K1 - 1 and a < num_drafts[s] and target[s, a] == drafts[s, a]:
            a += 1
        acc[s], nxt[s] = a, target[s, a]
    return acc, nxt
