"""Greedy speculative verify: the all-greedy case of nano-vllm's verify_drafts (nanovllm/layers/sampler.py:28-103).

verify_drafts_greedy(logits, draft_token_ids, num_drafts) returns what verify_drafts returns when every
temperature is 0: the target ids are the row argmaxes of logits [S*(K+1), V] (torch's argmax, first index of the
maximum, as sampler.py:66), and the accept length and next token come from the integer kernel behind
ops.greedy_accept (sampler.py:67, 79-82).  Unlike the reference it reads no device value on the host (the
reference's all-greedy test at sampler.py:64 syncs), so a verify step stays capturable in a CUDA graph.

The random-temperature branch (speculative sampling, sampler.py:68-78, 83-102) has no counterpart here.
"""
import torch

from . import ops


def verify_drafts_greedy(logits: torch.Tensor, draft_token_ids: torch.Tensor, num_drafts: torch.Tensor):
    """logits [S*(K+1), V], draft_token_ids [S, K], num_drafts [S] -> (num_accepted [S], next_token [S]) int64,
    the dtype the reference returns.  Sequence s keeps draft_token_ids[s, :num_accepted[s]], then next_token[s]."""
    S, K = draft_token_ids.shape
    top1 = logits.view(S, K + 1, logits.size(-1)).argmax(dim=-1)    # [S, K+1] int64
    return ops.greedy_accept(top1, draft_token_ids.to(top1.dtype), num_drafts.to(top1.dtype))
