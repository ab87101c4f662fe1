"""Golden attention outputs from the reference's own attention library, flash-attn 2.8.3, called exactly the way
nanovllm/layers/attention.py calls it:
  decode / verify (attention.py:75-77):  flash_attn_with_kvcache(q[B, n, H, D], k_cache, v_cache,
                                          cache_seqlens=context_lens, block_table=block_tables,
                                          softmax_scale=scale, causal=True)
  prefill / mixed (attention.py:67-70):  flash_attn_varlen_func(q, k, v, max_seqlen_q=, cu_seqlens_q=,
                                          max_seqlen_k=, cu_seqlens_k=, softmax_scale=scale, causal=True,
                                          block_table=block_tables)   (k, v = the paged caches, or contiguous rows)
Needs a CUDA GPU with flash-attn installed (the B200 image has 2.8.3).  Inputs come from nvattn.workloads with fixed
seeds on the CPU generator, so only their checksums and the outputs (raw bf16 bits) are stored; the tests rebuild the
inputs and fail loudly if the checksums drift.

Usage: python tests/golden/make_golden_fa2.py [--out tests/golden/attention_fa2_golden.npz]
"""
import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "nano-vllm-spec-decode_b200"))

# (name, kind, arguments for the workload generator); geometry H=8, KVH=2 (group 4, as Qwen3-8B), D=128, 8-block pool
CASES = [
    ("decode", "paged_decode", dict(lens=[37, 300, 513], q_per_seq=1, seed=11)),
    ("verify_k3", "paged_decode", dict(lens=[40, 256, 700], q_per_seq=4, seed=12)),
    ("verify_k8_padded", "paged_decode", dict(lens=[9, 1000, 130], q_per_seq=9, seed=13, pad_seqs=1)),
    ("mixed_paged", "varlen", dict(q_lens=[1, 3, 130, 1], k_lens=[200, 40, 400, 1], seed=14, paged=True)),
    ("prefill_contiguous", "varlen", dict(q_lens=[5, 129, 64], k_lens=[5, 129, 64], seed=15, paged=False)),
]
GEOM = dict(num_heads=8, num_kv_heads=2, head_dim=128, num_blocks=8)


def build(kind, args, device="cpu"):
    from nvattn.workloads import paged_decode_batch, varlen_batch
    if kind == "paged_decode":
        a = dict(args)
        return paged_decode_batch(a.pop("lens"), a.pop("q_per_seq"), GEOM["num_heads"], GEOM["num_kv_heads"],
                                  GEOM["head_dim"], GEOM["num_blocks"], 0.5, device=device, **a)
    a = dict(args)
    return varlen_batch(a.pop("q_lens"), a.pop("k_lens"), GEOM["num_heads"], GEOM["num_kv_heads"], GEOM["head_dim"],
                        GEOM["num_blocks"], 0.5, device=device, **a)


def checksum(b) -> np.ndarray:
    return np.array([float(b.q.double().sum()), float(b.k_cache.double().sum()), float(b.v_cache.double().sum()),
                     float(b.q.double().abs().sum())])


def run_fa2(kind, b):
    from flash_attn import flash_attn_varlen_func, flash_attn_with_kvcache
    if kind == "paged_decode":
        B, n = b.num_seqs, b.q_per_seq
        H, D = b.q.shape[1], b.q.shape[2]
        o = flash_attn_with_kvcache(b.q.view(B, n, H, D), b.k_cache, b.v_cache, cache_seqlens=b.context_lens,
                                    block_table=b.block_tables, softmax_scale=b.scale, causal=True)
        return o.reshape(B * n, H, D)
    if b.meta["paged"]:
        k, v, bt = b.k_cache, b.v_cache, b.block_tables
    else:
        k, v, bt = b.k_new, b.v_new, None
    return flash_attn_varlen_func(b.q, k, v, max_seqlen_q=b.max_seqlen_q, cu_seqlens_q=b.cu_seqlens_q,
                                  max_seqlen_k=b.max_seqlen_k, cu_seqlens_k=b.cu_seqlens_k, softmax_scale=b.scale,
                                  causal=True, block_table=bt)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(HERE, "attention_fa2_golden.npz"))
    args = ap.parse_args()
    import flash_attn
    out = {"flash_attn_version": np.array(flash_attn.__version__)}
    for name, kind, a in CASES:
        cpu = build(kind, a)
        dev = build(kind, a, device="cuda")
        o = run_fa2(kind, dev)
        torch.cuda.synchronize()
        out[f"{name}/out"] = o.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
        out[f"{name}/checksum"] = checksum(cpu)
        print(name, tuple(o.shape), float(o.float().abs().mean()))
    np.savez_compressed(args.out, **out)
    print("wrote", args.out)


if __name__ == "__main__":
    main()
