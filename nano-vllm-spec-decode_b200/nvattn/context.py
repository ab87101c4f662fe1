"""Per-step batch descriptor read by Attention.forward: the Context of nanovllm/utils/context.py:5-28, with the
same fields, defaults and set/get/reset functions, so ModelRunner code that builds it works unchanged.

Inside nano-vllm, bind() makes Attention read nano-vllm's own module-global context instead of this one:
    import nanovllm.utils.context, nvattn.context
    nvattn.context.bind(nanovllm.utils.context.get_context)
"""
from dataclasses import dataclass

import torch


@dataclass(slots=True)
class Context:
    is_prefill: bool = False
    cu_seqlens_q: torch.Tensor | None = None
    cu_seqlens_k: torch.Tensor | None = None
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    slot_mapping: torch.Tensor | None = None
    context_lens: torch.Tensor | None = None
    block_tables: torch.Tensor | None = None
    logits_indices: torch.Tensor | None = None    # mixed batching: the rows the LM head computes logits for


_CONTEXT = Context()
_getter = None


def get_context() -> Context:
    return _getter() if _getter is not None else _CONTEXT


def set_context(is_prefill, cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q=0, max_seqlen_k=0, slot_mapping=None,
                context_lens=None, block_tables=None, logits_indices=None):
    global _CONTEXT
    _CONTEXT = Context(is_prefill, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, slot_mapping, context_lens,
                       block_tables, logits_indices)


def reset_context():
    global _CONTEXT
    _CONTEXT = Context()


def bind(getter) -> None:
    """Read the context through `getter` (e.g. nanovllm.utils.context.get_context); None restores this module's."""
    global _getter
    _getter = getter
