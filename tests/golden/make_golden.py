"""Generate golden vectors for the byte / integer parts of the hot path from the reference itself.

Runs the reference's own code on CPU (so it needs a checkout of R3pere/nano-vllm-spec-decode, passed as
--reference or REFERENCE_DIR; it is not needed to run the tests):
  * store_kvcache (nanovllm/layers/attention.py:33-40) under TRITON_INTERPRET=1 -> scatter_golden.npz
  * verify_drafts (nanovllm/layers/sampler.py:28-103), greedy rows, fed one-hot logits whose argmax is the
    target id (the logits_with_top1 pattern of tests/test_spec_unit.py:64-69) -> accept_golden.npz

Inputs are seeded; bf16 tensors are stored as their raw uint16 bits.
Usage: TRITON_INTERPRET=1 python tests/golden/make_golden.py --reference <path to the reference checkout>
"""
import argparse
import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "nano-vllm-spec-decode_b200"))


def raw(t: torch.Tensor) -> np.ndarray:
    t = t.contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def scatter_cases(store_kvcache):
    from nvattn.workloads import config1
    cases = {}

    def run(name, key, value, NB, slots, init="zeros"):
        N, KVH, D = key.shape
        if init == "zeros":
            kc = torch.zeros(NB, 256, KVH, D, dtype=key.dtype)
            vc = torch.zeros_like(kc)
        else:    # a periodic pattern (compresses well, still shows any stray write)
            n = NB * 256 * KVH * D
            kc = (((torch.arange(n) % 997) - 498) * 0.01).view(NB, 256, KVH, D).to(key.dtype)
            vc = (((torch.arange(n) % 991) - 495) * -0.01).view(NB, 256, KVH, D).to(key.dtype)
        kin, vin = kc.clone(), vc.clone()
        store_kvcache(key, value, kc, vc, slots)
        # key/value stored compact; their row strides recorded so the test rebuilds the same views
        cases[name] = dict(key_base=raw(key._base if key._base is not None else key),
                           value_base=raw(value._base if value._base is not None else value),
                           key_offset=key.storage_offset(), value_offset=value.storage_offset(),
                           key_row_stride=key.stride(0), value_row_stride=value.stride(0),
                           shape=np.array([N, KVH, D, NB]), dtype=str(key.dtype), slots=slots.numpy(),
                           k_in=raw(kin), v_in=raw(vin), k_out=raw(kc), v_out=raw(vc), init=init)

    # config 0 of BASELINE: 0.6B shape, fp32, pool 64 blocks, the 4 new tokens at slot = block*256 + offset
    c1 = config1(0)["batch"]
    gen = torch.Generator().manual_seed(100)
    key = torch.randn(4, 8, 128, generator=gen)
    value = torch.randn(4, 8, 128, generator=gen)
    run("config1_fp32", key, value, 64, c1.slot_mapping.clone())

    # bf16, value a column slice of a fused qkv row (attention.py:36-37 allows any row stride), slots with -1
    gen = torch.Generator().manual_seed(101)
    N, KVH, D = 37, 2, 64
    qkv = torch.randn(N, 4 * KVH * D, generator=gen).to(torch.bfloat16)
    key = qkv[:, KVH * D:2 * KVH * D].view(N, KVH, D)
    value = qkv[:, 2 * KVH * D:3 * KVH * D].view(N, KVH, D)
    slots = torch.randperm(4 * 256, generator=gen)[:N].to(torch.int32)
    slots[torch.tensor([0, 5, 17, 36])] = -1
    run("bf16_strided", key, value, 4, slots, init="pattern")

    # decode-like with padding rows (slot -1 at the tail), fp32 random cache
    gen = torch.Generator().manual_seed(103)
    N, KVH, D = 12, 4, 128
    key = torch.randn(N, KVH, D, generator=gen)
    value = torch.randn(N, KVH, D, generator=gen)
    slots = torch.tensor([3, 300, 511, 256, 0, 767, 10, 11, -1, -1, -1, -1], dtype=torch.int32)
    run("fp32_padded", key, value, 3, slots, init="pattern")

    # Qwen3-8B row (KVH 8 x 128) in bf16, a full decode batch of 64 tokens at distinct random slots
    gen = torch.Generator().manual_seed(105)
    N, KVH, D = 64, 8, 128
    key = torch.randn(N, KVH, D, generator=gen).to(torch.bfloat16)
    value = torch.randn(N, KVH, D, generator=gen).to(torch.bfloat16)
    slots = torch.randperm(8 * 256, generator=gen)[:N].to(torch.int32)
    run("bf16_qwen3_8b", key, value, 8, slots)
    return cases


def accept_cases(verify_drafts):
    from nvattn.workloads import accept_config
    cases = {}

    def run(name, target, drafts, num_drafts, V):
        S, K1 = target.shape
        logits = torch.zeros(S * K1, V)
        logits.scatter_(1, target.reshape(-1, 1).long(), 1.0)   # argmax = target (unique max)
        a, t = verify_drafts(logits, drafts.long(), num_drafts.long(), torch.zeros(S))
        cases[name] = dict(target=target.numpy().astype(np.int64), drafts=drafts.numpy().astype(np.int64),
                           num_drafts=num_drafts.numpy().astype(np.int64), num_accepted=a.numpy(),
                           next_token=t.numpy())

    # test_verify_greedy's hand case (tests/test_spec_unit.py:72-83)
    run("hand", torch.tensor([[3, 4, 5, 6]] * 4), torch.tensor([[3, 4, 5], [3, 9, 5], [1, 4, 5], [3, 4, 5]]),
        torch.tensor([3, 3, 3, 1]), 10)
    # K = 0 is plain greedy decoding (test_spec_unit.py:85-87)
    run("k0", torch.tensor([[7], [2]]), torch.zeros(2, 0, dtype=torch.int64), torch.zeros(2, dtype=torch.int64), 10)
    gen = torch.Generator().manual_seed(7)
    for k in (1, 2, 4, 8):
        target, drafts, nd = accept_config(k, seed=k)
        run(f"config3_k{k}", target, drafts, nd, 151936)
        # padded drafts: fewer real guesses than k (run_verify pads drafts with 0, model_runner.py:477-479)
        nd2 = torch.randint(0, k + 1, (32,), generator=gen).to(torch.int32)
        run(f"config3_k{k}_padded", target, torch.where(torch.arange(k) < nd2[:, None], drafts, target[:, :k]),
            nd2, 151936)
    return cases


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("REFERENCE_DIR"))
    args = ap.parse_args()
    assert args.reference and os.path.isdir(args.reference), "pass --reference <reference checkout>"
    sys.path.insert(0, args.reference)
    from nanovllm.layers.attention import store_kvcache
    from nanovllm.layers.sampler import verify_drafts

    sc = scatter_cases(store_kvcache)
    flat = {f"{c}/{k}": v for c, d in sc.items() for k, v in d.items()}
    np.savez_compressed(os.path.join(HERE, "scatter_golden.npz"), **flat)
    ac = accept_cases(verify_drafts)
    flat = {f"{c}/{k}": v for c, d in ac.items() for k, v in d.items()}
    np.savez_compressed(os.path.join(HERE, "accept_golden.npz"), **flat)
    print("scatter cases:", list(sc), "accept cases:", list(ac))


if __name__ == "__main__":
    main()
