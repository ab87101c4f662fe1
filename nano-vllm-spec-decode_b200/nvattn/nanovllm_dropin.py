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

install_fused_prologue()
    Qwen3's attention prologue in one kernel (`nva_qk_norm_rope_store`): the q / k RMSNorm and rotary embedding of
    Qwen3Attention.pre_attn (nanovllm/models/qwen3.py:88-97) and the KV scatter of Attention.forward
    (attention.py:61-62) become one pass over the projection output.  Qwen3Attention.forward (whole-model steps:
    prefill, decode / verify and their CUDA graphs) scatters in the same kernel; pre_attn (the piecewise segments of
    mixed steps, recorded without a Context) fuses the norms and rotary only and leaves the scatter to the
    attention call, as the reference does.  Needs install_attention.

install_mixed_step_graph()
    Mixed steps (enable_mixed_batching with mixed_cuda_graph) as one CUDA graph per token bucket.  The reference
    records the L + 1 segments between the attentions as separate graphs and runs every attention eagerly in
    between (ModelRunner.run_piecewise, model_runner.py:563-589, 677-687), because flash-attn's varlen call reads
    host values of the step's batch.  nvattn's varlen attention reads its batch layout from device memory only and
    keeps a fixed launch geometry for a fixed sequence capacity, so the whole step -- segments and attentions -- is
    recorded once per bucket over static Context buffers (cu_seqlens for max_num_seqs sequences, padded with empty
    ones; the slot mapping padded with -1; a max_num_seqs x max_num_blocks block table) and replayed after the step's
    Context is copied into them.  Rows of the bucket past the step's tokens belong to no sequence: attention neither
    reads nor writes them, and nothing else mixes rows.  Steps the graphs do not cover (more sequences than
    max_num_seqs, or eager mode) take the reference's path.  Needs install_attention.

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


def install_fused_prologue() -> None:
    """q / k RMSNorm + rotary (+ the KV scatter in whole-model steps) in one kernel (see module docstring)."""
    if "fused_prologue" in _installed:
        return
    assert "attention" in _installed, "install_attention first"
    from nanovllm.models import qwen3
    from nanovllm.utils.context import get_context
    from . import ops

    def prologue(self, positions, hidden_states, scatter):
        qkv = self.qkv_proj(hidden_states)
        attn = self.attn
        ctx = get_context() if scatter else None
        cache = scatter and attn.k_cache.numel() > 0
        contiguous_kv = not scatter or (ctx.is_prefill and ctx.block_tables is None)
        q, k, v = ops.qk_norm_rope_store(
            qkv, positions, self.rotary_emb.cos_sin_cache, self.q_norm.weight, self.k_norm.weight, self.q_norm.eps,
            self.num_heads, self.num_kv_heads, attn.k_cache if cache else None, attn.v_cache if cache else None,
            ctx.slot_mapping if cache else None, want_k=contiguous_kv)
        return q, k, v

    def attention_forward(self, positions, hidden_states):
        assert not self.qkv_bias, "the fused prologue is Qwen3's (q / k norms, no qkv bias)"
        q, k, v = prologue(self, positions, hidden_states, True)
        o = self.attn.forward_stored(q, k, v)
        return self.post_attn(o)

    def attention_pre_attn(self, positions, hidden_states):
        assert not self.qkv_bias, "the fused prologue is Qwen3's (q / k norms, no qkv bias)"
        return prologue(self, positions, hidden_states, False)

    qwen3.Qwen3Attention.forward = attention_forward
    qwen3.Qwen3Attention.pre_attn = attention_pre_attn
    _installed.add("fused_prologue")


def install_mixed_step_graph() -> None:
    """Whole mixed steps (segments + attentions) as one CUDA graph per token bucket (see module docstring)."""
    if "mixed_step_graph" in _installed:
        return
    assert "attention" in _installed, "install_attention first"
    import torch
    from nanovllm.engine import model_runner as mr
    from nanovllm.utils.context import get_context, set_context, reset_context

    capture_cudagraph = mr.ModelRunner.capture_cudagraph
    run_piecewise = mr.ModelRunner.run_piecewise

    def whole_step(self, n):
        layers = self.model.model.layers
        pv = self.piecewise_vars
        for i in range(len(layers) + 1):
            if i:
                pv["o"][:n] = layers[i - 1].self_attn.attn(pv["q"][:n], pv["k"][:n], pv["v"][:n])
            self.run_segment(i, n)

    @torch.inference_mode()
    def runner_capture_cudagraph(self):
        capture_cudagraph(self)
        self.mixed_step_graphs = {}
        if not self.mixed_buckets:
            return
        S, N = self.config.max_num_seqs, self.mixed_buckets[-1]
        sv = dict(cu_q=torch.zeros(S + 1, dtype=torch.int32), cu_k=torch.zeros(S + 1, dtype=torch.int32),
                  slots=torch.full((N,), -1, dtype=torch.int32),
                  bt=torch.full((S, self.max_num_blocks), -1, dtype=torch.int32))
        self.mixed_step_vars = sv
        for n in reversed(self.mixed_buckets):
            # recorded with every sequence empty; max_seqlen_q = n is an upper bound for any step of this bucket
            set_context(True, sv["cu_q"], sv["cu_k"], n, self.config.max_model_len, sv["slots"][:n], None, sv["bt"])
            whole_step(self, n)    # warmup
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, self.graph_pool):
                whole_step(self, n)
            self.mixed_step_graphs[n] = graph
            reset_context()
        torch.cuda.synchronize()

    @torch.inference_mode()
    def runner_run_piecewise(self, input_ids, positions):
        graphs = getattr(self, "mixed_step_graphs", None)
        ctx = get_context()
        n = input_ids.size(0)
        B = ctx.cu_seqlens_q.numel() - 1
        if self.enforce_eager or not graphs or B > self.config.max_num_seqs or n > self.mixed_buckets[-1]:
            return run_piecewise(self, input_ids, positions)
        bucket = next(x for x in self.mixed_buckets if x >= n)
        pv, sv = self.piecewise_vars, self.mixed_step_vars
        pv["input_ids"][:n] = input_ids
        pv["input_ids"][n:bucket] = 0
        pv["positions"][:n] = positions
        pv["positions"][n:bucket] = 0
        pv["o"][n:bucket] = 0
        for name, src in (("cu_q", ctx.cu_seqlens_q), ("cu_k", ctx.cu_seqlens_k)):
            sv[name][:B + 1] = src
            sv[name][B + 1:] = src[-1:]      # empty sequences after the last one
        sv["slots"][:n] = ctx.slot_mapping
        sv["slots"][n:bucket] = -1
        W = ctx.block_tables.size(1)
        if W > sv["bt"].size(1):
            return run_piecewise(self, input_ids, positions)
        sv["bt"][:B, :W] = ctx.block_tables
        graphs[bucket].replay()
        return pv["hidden"][:n]

    exit_runner = mr.ModelRunner.exit

    def runner_exit(self):
        self.mixed_step_graphs = {}    # released before the graph pool, as the reference releases its own graphs
        exit_runner(self)

    mr.ModelRunner.capture_cudagraph = runner_capture_cudagraph
    mr.ModelRunner.run_piecewise = runner_run_piecewise
    mr.ModelRunner.exit = runner_exit
    _installed.add("mixed_step_graph")
