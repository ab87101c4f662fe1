"""Install this package into a running nano-vllm-spec-decode (the `nanovllm` package) without editing its files.

install_attention()
    The attention swap: nano-vllm's `Attention` (nanovllm/layers/attention.py:43-79) and `store_kvcache`
    (:33-40) are replaced by nvattn's, which read nano-vllm's own module-global Context
    (nanovllm/utils/context.py:18-28).  Done before the model is built, every `Qwen3Attention`
    (nanovllm/models/qwen3.py:63-68) constructs the nvattn module, and ModelRunner's cache binding
    (model_runner.py:258-267), decode graph capture (:646-675), verify step (:465-485) and piecewise mixed steps
    (:563-589) call it unchanged.

install_tp_speculative()
    n-gram speculative decoding with tensor parallelism > 1.  The reference refuses it
    (nanovllm/config.py:39-41: "drafting needs each request's full token list, which TP>1 doesn't send to the
    worker processes").  The proposer only needs the full token list on rank 0, where it runs
    (llm_engine.py:107-146); the workers need just this step's guesses, so three changes suffice:
      * Sequence pickling (sequence.py:81-92) also carries `draft_token_ids` of decode sequences and the
        temperature (so every rank takes the same path in install_greedy_argmax);
      * ModelRunner.run_verify (model_runner.py:465-485) verifies on rank 0 only: the workers run the same model
        pass and the same logits gather (embed_head.py:56-68), whose result exists on rank 0 only;
      * ModelRunner.warmup_verify (model_runner.py:219-238) likewise skips `verify_drafts` on the workers;
    and Config's TP=1 assertion is lifted for n-gram drafting (a draft model still needs TP=1: its sampler also
    runs on rank 0 only, model_runner.py:441).  Mixed batching keeps its own TP=1 assertion (config.py:58-59).

install_greedy_argmax()
    Greedy verify without the full-vocabulary logits on rank 0 (the LM-head half of `verify_drafts`,
    sampler.py:66-82, and the logits gather of ParallelLMHead.forward, embed_head.py:56-68): when every request of
    a verify step is greedy, each rank reduces its vocabulary shard of the logits to one (maximum, index) pair per
    row on the GPU (`nva_shard_argmax`), rank 0 gathers the pairs (8 bytes per row and rank instead of V / tp x 2
    bytes) and a second kernel merges them into the target ids and the accept lengths (`nva_shard_accept`).  Ties
    go to the lowest vocabulary index, as torch's argmax over the concatenated logits does, so the result is the
    reference's bit for bit.

Each function is idempotent and must run in every process that builds a model: in the TP worker processes too
(they are started with multiprocessing's spawn, which imports the parent's main module first; call these at module
level there, as nvattn.e2e does).
"""
import sys

_installed: set[str] = set()


def install_attention() -> None:
    """Swap nano-vllm's attention module and KV scatter for nvattn's (see module docstring)."""
    if "attention" in _installed:
        return
    import nanovllm.utils.context as nctx
    import nanovllm.layers.attention as nattn
    from . import context as vctx
    from . import attention as vattn
    vctx.bind(nctx.get_context)
    nattn.Attention = vattn.Attention
    nattn.store_kvcache = vattn.store_kvcache
    qwen3 = sys.modules.get("nanovllm.models.qwen3")
    if qwen3 is None:
        import nanovllm.models.qwen3 as qwen3
    qwen3.Attention = vattn.Attention

    # Size the attention workspace with the KV cache (model_runner.py:240-267), before capture_cudagraph and the
    # piecewise graphs, so that no attention call allocates later (under a graph capture that would raise).
    from nanovllm.engine import model_runner as mr
    from . import ops
    allocate_kv_cache = mr.ModelRunner.allocate_kv_cache

    def runner_allocate_kv_cache(self):
        allocate_kv_cache(self)
        attn = next(m for m in self.model.modules() if isinstance(m, vattn.Attention))
        ops.reserve_workspace(self.config.max_num_seqs, self.config.max_num_batched_tokens, attn.num_heads,
                              attn.num_kv_heads, attn.head_dim)

    mr.ModelRunner.allocate_kv_cache = runner_allocate_kv_cache
    _installed.add("attention")


def install_tp_speculative() -> None:
    """Let n-gram speculative decoding run with tensor_parallel_size > 1 (see module docstring)."""
    if "tp_spec" in _installed:
        return
    import torch
    from nanovllm.config import Config
    from nanovllm.engine.sequence import Sequence
    from nanovllm.engine import model_runner as mr
    from nanovllm.utils.context import set_context, reset_context

    post_init = Config.__post_init__

    def config_post_init(self):
        tp = self.tensor_parallel_size
        if tp > 1 and self.speculative_method == "ngram":
            # the reference's checks with the TP assertion for drafting taken out; mixed batching keeps its own
            assert not self.enable_mixed_batching, "mixed batching is not supported with tensor parallelism"
            self.tensor_parallel_size = 1
            try:
                post_init(self)
            finally:
                self.tensor_parallel_size = tp
        else:
            post_init(self)

    Config.__post_init__ = config_post_init

    get_state, set_state = Sequence.__getstate__, Sequence.__setstate__

    def seq_getstate(self):
        return get_state(self) + (list(self.draft_token_ids) if not self.is_prefill else [], self.temperature)

    def seq_setstate(self, state):
        set_state(self, state[:-2])
        self.draft_token_ids, self.temperature = state[-2], state[-1]

    Sequence.__getstate__, Sequence.__setstate__ = seq_getstate, seq_setstate

    run_verify = mr.ModelRunner.run_verify

    @torch.inference_mode()
    def runner_run_verify(self, seqs, k):
        if self.rank == 0:
            return run_verify(self, seqs, k)
        assert self.draft_model is None, "draft-model drafting needs tensor_parallel_size 1"
        input_ids, positions = self.prepare_decode(seqs, 1 + k)
        hidden_states = self.run_model(input_ids, positions, False)[:len(seqs) * (1 + k)]
        self.model.compute_logits(hidden_states)    # this rank's part of the logits gather
        reset_context()
        return None

    mr.ModelRunner.run_verify = runner_run_verify

    warmup_verify = mr.ModelRunner.warmup_verify

    @torch.inference_mode()
    def runner_warmup_verify(self):
        if self.rank == 0:
            return warmup_verify(self)
        for k in self.config.spec_k_choices:
            if k == 0:
                continue
            num_seqs = self.config.spec_batch_limit(k)
            set_context(False)
            hidden_states = torch.zeros(num_seqs * (1 + k), self.config.hf_config.hidden_size)
            self.model.compute_logits(hidden_states)
            del hidden_states
            reset_context()

    mr.ModelRunner.warmup_verify = runner_warmup_verify
    _installed.add("tp_spec")


def install_greedy_argmax() -> None:
    """All-greedy verify steps reduce the logits to (maximum, index) per row and rank (see module docstring)."""
    if "greedy_argmax" in _installed:
        return
    import torch
    import torch.distributed as dist
    from nanovllm.engine import model_runner as mr
    from nanovllm.layers.embed_head import ParallelLMHead
    from nanovllm.utils.context import reset_context
    from . import ops

    run_verify = mr.ModelRunner.run_verify

    @torch.inference_mode()
    def runner_run_verify(self, seqs, k):
        # model_runner.py:465-485 with the logits gather and verify_drafts replaced (greedy steps only)
        if any(seq.temperature != 0 for seq in seqs):
            return run_verify(self, seqs, k)
        S = len(seqs)
        if self.draft_model is not None:    # a draft model guesses first (TP 1 only, like the reference)
            drafts, _ = self.run_draft(seqs, k, self.prepare_sample(seqs))
            for seq, guesses in zip(seqs, drafts.tolist()):
                seq.draft_token_ids = guesses[:seq.max_drafts(k)]
        elif self.rank == 0:
            drafts = [seq.draft_token_ids + [0] * (k - len(seq.draft_token_ids)) for seq in seqs]
            drafts = torch.tensor(drafts, dtype=torch.int64, pin_memory=True).cuda(non_blocking=True).view(S, k)
        if self.rank == 0:
            num_drafts = torch.tensor([len(seq.draft_token_ids) for seq in seqs], dtype=torch.int64,
                                      pin_memory=True).cuda(non_blocking=True)
        input_ids, positions = self.prepare_decode(seqs, 1 + k)
        hidden_states = self.run_model(input_ids, positions, False)[:S * (1 + k)]
        head: ParallelLMHead = self.model.lm_head
        logits = torch.nn.functional.linear(hidden_states, head.weight)    # this rank's vocabulary shard
        keys = ops.shard_argmax(logits, head.vocab_start_idx)               # [S(1+k)] (max, index) keys
        del logits
        if head.tp_size > 1:
            gathered = [torch.empty_like(keys) for _ in range(head.tp_size)] if self.rank == 0 else None
            dist.gather(keys, gathered, 0)
            keys = torch.stack(gathered) if self.rank == 0 else None
        else:
            keys = keys.unsqueeze(0)
        reset_context()
        if self.rank != 0:
            return None
        num_accepted, next_tokens = ops.shard_accept(keys.view(-1, S, 1 + k), drafts, num_drafts)
        return [seq.draft_token_ids[:a] + [t] for seq, a, t in zip(seqs, num_accepted.tolist(), next_tokens.tolist())]

    mr.ModelRunner.run_verify = runner_run_verify
    _installed.add("greedy_argmax")
