"""nvattn: B200 (sm_100a) attention hot path for nano-vllm-spec-decode.

Public surface (mirrors the reference's module names):
  nvattn.attention.Attention, nvattn.attention.store_kvcache     <- nanovllm/layers/attention.py
  nvattn.context.{Context, set_context, get_context, reset_context, bind}  <- nanovllm/utils/context.py
  nvattn.ops.{flash_attn_with_kvcache, flash_attn_varlen_func, greedy_accept}
  nvattn.sampler.verify_drafts_greedy                             <- all-greedy verify_drafts (layers/sampler.py)
The kernels live in libnvattn.so (C ABI: include/nvattn.h), loaded on first use.
"""
__version__ = "0.1.0"


def __getattr__(name):
    if name in ("Attention", "store_kvcache"):
        from . import attention
        return getattr(attention, name)
    raise AttributeError(name)
