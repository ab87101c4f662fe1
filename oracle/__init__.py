"""CPU oracle for the attention hot path of nano-vllm-spec-decode.

TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm
import this package, and only as the checker or the timed CPU baseline.  The product (the nvattn package and
libnvattn.so) never imports, links or calls it, and has no CPU fallback.

Contents:
  oracle.c       C restatement of the byte / integer work: the KV scatter (attention.py:10-40) and the greedy
                 accept length (sampler.py:66-82).  Built by build_c() into oracle/_build/liboracle.so.
  argmax.py      numpy restatement of greedy verify over vocabulary shards: per-shard (max, index) keys, their
                 merge and the accept rule (embed_head.py:56-68, sampler.py:66-82).
  attention.py   FP32 torch restatement of Attention.forward's math (attention.py:59-79) with flash-attn's
                 documented semantics: paged KV through block tables, GQA head mapping h -> h // (H/KVH),
                 causal mask aligned to the bottom right, empty rows give zero output.

Pinning: the scatter and accept-length restatements are checked against golden vectors produced by the
reference's own store_kvcache (Triton interpreter on CPU) and verify_drafts (tests/golden/make_golden.py).
The attention restatement is checked against outputs of the reference's attention library (flash-attn 2.8.3,
run on a B200 by tests/golden/make_golden_fa2.py) stored in tests/golden/attention_fa2_golden.npz.
"""
from .lib import build_c, store_kvcache, greedy_accept  # noqa: F401
from .attention import (  # noqa: F401
    paged_attention_ref,
    varlen_attention_ref,
    store_kvcache_ref,
    greedy_accept_ref,
)
