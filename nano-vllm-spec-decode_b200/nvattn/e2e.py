"""BASELINE config 5 end to end: greedy n-gram speculative decoding of a random-init Qwen3-8B under
nano-vllm-spec-decode's own engine (LLMEngine, Scheduler, ModelRunner with its CUDA graphs, the n-gram proposer and
dynamic k), with the attention of one of two arms:

  reference   the unmodified reference: flash-attn 2.8.3 + its Triton KV scatter (nanovllm/layers/attention.py)
  nvattn      this package swapped in by nvattn.nanovllm_dropin.install_attention
  nvattn+argmax  the same, plus nanovllm_dropin.install_greedy_argmax (greedy verify from per-rank (max, index) pairs)
  nvattn+all  the same, plus nanovllm_dropin.install_fused_prologue (q / k norm + rotary + KV scatter in one kernel)
              and install_mixed_step_graph (whole mixed steps as one CUDA graph)

At tensor_parallel_size > 1 both arms also get nanovllm_dropin.install_tp_speculative (the reference refuses
speculative decoding with TP > 1, config.py:39-41).

Reproducibility: torch.compile's Inductor is set to deterministic mode in every arm (no kernel configs chosen by
timing), so repeated runs of a variant give the same tokens.

What stands in for what the reference would load (no checkpoint, tokenizer or network here):
  * the model directory holds only a config.json with Qwen3-8B's published shape (36 layers, hidden 4096,
    32 q / 8 kv heads of 128, SwiGLU 12288, vocab 151936, RoPE theta 1e6, bf16);
  * the weights come from `seeded_weight`: every tensor of the Hugging Face checkpoint layout drawn from
    N(0, 0.02) (RMSNorm weights 1) by a CUDA generator seeded from (seed, tensor name), rounded to bf16, and fed
    through the model's own weight_loaders exactly as nanovllm/utils/loader.py:12-28 feeds a checkpoint;
  * prompts are token ids (`config5_prompts`), so the tokenizer is replaced by a stub with Qwen3's EOS id;
  * dynamic k chooses k from a step-cost table (llm_engine.py:36-38 measures it at start-up, dynamic_k.py); a
    measured table makes the choice depend on timing, so `--step-costs FILE` injects one fixed table into every
    arm (and `--save-step-costs FILE` keeps what an arm measured).  With the same table, two arms whose tokens
    agree take the same k at every step.

Run one arm per process (each takes most of the GPU memory for its KV cache, like the reference's test_greedy.py):
    python -m nvattn.e2e --arm nvattn --variant spec_ngram_dynk_graph --tp 1 --out result.json
Worker processes of TP > 1 re-import this module (multiprocessing spawn) and install the same patches from the
NVA_E2E_* environment variables set by the parent.
"""
import argparse
import json
import os
import sys
import time
import zlib

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF_INSTALL = os.path.join(REPO, "baseline", "_ref")    # pip install --target of the reference (git-ignored)

QWEN3_8B = {
    "architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "attention_bias": False, "attention_dropout": 0.0,
    "bos_token_id": 151643, "eos_token_id": 151645, "head_dim": 128, "hidden_act": "silu", "hidden_size": 4096,
    "initializer_range": 0.02, "intermediate_size": 12288, "max_position_embeddings": 40960, "max_window_layers": 36,
    "num_attention_heads": 32, "num_hidden_layers": 36, "num_key_value_heads": 8, "rms_norm_eps": 1e-06,
    "rope_scaling": None, "rope_theta": 1000000, "sliding_window": None, "tie_word_embeddings": False,
    "torch_dtype": "bfloat16", "use_cache": True, "use_sliding_window": False, "vocab_size": 151936,
}
EOS = QWEN3_8B["eos_token_id"]

# the reference's test_greedy.py variants that n-gram drafting and the attention path touch (tests/test_greedy.py:69-90)
VARIANTS = {
    "eager": dict(enforce_eager=True),
    "graph": dict(enforce_eager=False),
    "spec_ngram": dict(enforce_eager=True, speculative_method="ngram", num_speculative_tokens=4),
    "spec_ngram_graph": dict(enforce_eager=False, speculative_method="ngram", num_speculative_tokens=4),
    "spec_ngram_dynk_graph": dict(enforce_eager=False, speculative_method="ngram", num_speculative_tokens=8,
                                  spec_dynamic_k=True),
    # the model guesses for itself (draft_model = the model's own directory and weights): nearly every guess is
    # accepted, so verify steps run on every decode step whatever the model generates
    "spec_draft": dict(enforce_eager=True, speculative_method="draft", draft_model="SELF", num_speculative_tokens=4),
    "spec_draft_graph": dict(enforce_eager=False, speculative_method="draft", draft_model="SELF",
                             num_speculative_tokens=4),
    "mixed_eager": dict(enforce_eager=True, enable_mixed_batching=True, max_num_batched_tokens=256),
    "mixed_graph": dict(enforce_eager=False, enable_mixed_batching=True, max_num_batched_tokens=256),
    "mixed_spec_ngram_graph": dict(enforce_eager=False, enable_mixed_batching=True, max_num_batched_tokens=256,
                                   speculative_method="ngram", num_speculative_tokens=4),
}
ARMS = ("reference", "nvattn", "nvattn+argmax", "nvattn+all")

ENV_ARM, ENV_TP, ENV_COSTS, ENV_SEED = "NVA_E2E_ARM", "NVA_E2E_TP", "NVA_E2E_STEP_COSTS", "NVA_E2E_WEIGHT_SEED"


def ensure_reference_importable() -> None:
    """Put the reference install (baseline/_ref, from `pip install --target baseline/_ref <reference>`) on the
    path; raise if nanovllm cannot be imported."""
    if os.path.isdir(REF_INSTALL) and REF_INSTALL not in sys.path:
        sys.path.insert(0, REF_INSTALL)
    try:
        import nanovllm  # noqa: F401
    except ImportError as e:
        raise RuntimeError(f"nano-vllm-spec-decode is not importable (expected under {REF_INSTALL}): {e}") from e


def write_model_dir(path: str, **overrides) -> str:
    """A model directory nano-vllm's Config accepts (config.py:34-37): config.json only."""
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(dict(QWEN3_8B, **overrides), f, indent=1)
    return path


def checkpoint_shapes(cfg: dict) -> dict[str, tuple[int, ...]]:
    """Name -> shape of every tensor of a Qwen3 checkpoint in the Hugging Face layout (what load_model reads)."""
    H, L, V = cfg["hidden_size"], cfg["num_hidden_layers"], cfg["vocab_size"]
    D, nq, nkv, I = cfg["head_dim"], cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["intermediate_size"]
    shapes = {"model.embed_tokens.weight": (V, H), "model.norm.weight": (H,)}
    if not cfg.get("tie_word_embeddings", False):
        shapes["lm_head.weight"] = (V, H)
    for i in range(L):
        p = f"model.layers.{i}."
        shapes.update({
            p + "self_attn.q_proj.weight": (nq * D, H), p + "self_attn.k_proj.weight": (nkv * D, H),
            p + "self_attn.v_proj.weight": (nkv * D, H), p + "self_attn.o_proj.weight": (H, nq * D),
            p + "self_attn.q_norm.weight": (D,), p + "self_attn.k_norm.weight": (D,),
            p + "mlp.gate_proj.weight": (I, H), p + "mlp.up_proj.weight": (I, H), p + "mlp.down_proj.weight": (H, I),
            p + "input_layernorm.weight": (H,), p + "post_attention_layernorm.weight": (H,),
        })
    return shapes


def seeded_weight(name: str, shape, seed: int, dtype=None, device="cuda"):
    """The random-init checkpoint tensor `name`: N(0, 0.02) from a CUDA generator seeded by (seed, crc32(name)),
    rounded to bf16 (norm weights: ones), returned in `dtype` (default bf16)."""
    import torch
    dtype = dtype or torch.bfloat16
    if name.endswith("norm.weight"):
        return torch.ones(shape, dtype=dtype, device=device)
    g = torch.Generator(device=device)
    g.manual_seed((seed * 1_000_003 + zlib.crc32(name.encode())) % (1 << 63))
    w = torch.randn(shape, generator=g, device=device, dtype=torch.float32).mul_(0.02)
    return w.to(torch.bfloat16).to(dtype)


def load_seeded(model, path: str) -> None:
    """Stand-in for nanovllm.utils.loader.load_model (loader.py:12-28): the same name -> packed parameter mapping and
    weight_loader calls, with seeded_weight tensors in place of the safetensors files."""
    with open(os.path.join(path, "config.json")) as f:
        cfg = json.load(f)
    seed = int(os.environ.get(ENV_SEED, "0"))
    packed = getattr(model, "packed_modules_mapping", {})
    for name, shape in checkpoint_shapes(cfg).items():
        w = seeded_weight(name, shape, seed)
        for k, (v, shard_id) in packed.items():
            if k in name:
                param = model.get_parameter(name.replace(k, v))
                param.weight_loader(param, w, shard_id)
                break
        else:
            param = model.get_parameter(name)
            loader = getattr(param, "weight_loader", None)
            if loader is None:
                param.data.copy_(w)
            else:
                loader(param, w)
        del w


def config5_prompts(num: int = 64, prompt_len: int = 1024, span: int = 128, repeats: int = 4, seed: int = 0,
                    vocab: int = 151643) -> list[list[int]]:
    """BASELINE config 5's requests: `prompt_len` seeded random ids whose last span * repeats tokens are one
    seeded `span`-token run repeated `repeats` times, so the n-gram proposer finds matches from the first step.
    Ids stay below Qwen3's special tokens (151643)."""
    import numpy as np
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(num):
        ids = rng.integers(0, vocab, prompt_len)
        run = rng.integers(0, vocab, span)
        ids[prompt_len - span * repeats:] = np.tile(run, repeats)
        out.append(ids.tolist())
    return out


def synthetic_step_costs(k_choices=(0, 1, 2, 4, 8), max_num_seqs: int = 512):
    """A fixed dynamic-k cost table (costs[k][i] = ms at bucket i, buckets as model_runner.batch_buckets): a step
    reading 16 GB of weights plus a per-token cost, 2.6 ms + 0.02 ms x tokens.  Used by tests, where measuring
    the table would dominate the run."""
    def buckets(max_bs):
        return [x for x in [1, 2, 4, 8] if x < max_bs] + list(range(16, max_bs, 16)) + [max_bs]
    limits = {k: min(512 // (1 + k), max_num_seqs) for k in k_choices if k}
    most = max(limits.values())
    costs, bks = {}, {}
    for k in k_choices:
        sizes = buckets(limits[k] if k else min(max_num_seqs, 512))
        if k == 0:
            sizes = [x for x in sizes if x < most] + [next(x for x in sizes if x >= most)]
        bks[k] = sizes
        costs[k] = [2.6 + 0.02 * bs * (1 + k) for bs in sizes]
    return costs, bks


class _StubTokenizer:
    """Prompts arrive as ids; generate() only needs eos_token_id and a decode()."""
    eos_token_id = EOS

    @classmethod
    def from_pretrained(cls, *a, **k):
        return cls()

    def decode(self, ids):
        return ""


def _apply_from_env() -> None:
    """Install the arm's patches in this process (parent and spawned TP workers alike)."""
    arm = os.environ.get(ENV_ARM)
    if not arm:
        return
    ensure_reference_importable()
    pkg = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if pkg not in sys.path:
        sys.path.insert(0, pkg)
    # torch.compile (RMSNorm, rotary, SiluAndMul, Sampler) otherwise picks some Triton kernel configs by timing them
    # at run time, so two processes running the same variant can round differently (seen as different tokens, the
    # reference arm included); with this set, every process compiles the same kernels.  It applies to every arm.
    import torch._inductor.config
    torch._inductor.config.deterministic = True
    import nanovllm.engine.model_runner as mr
    import nanovllm.engine.llm_engine as le
    from nvattn import nanovllm_dropin
    mr.load_model = load_seeded
    le.AutoTokenizer = _StubTokenizer
    if int(os.environ.get(ENV_TP, "1")) > 1:
        nanovllm_dropin.install_tp_speculative()
    if arm.startswith("nvattn"):
        nanovllm_dropin.install_attention()
    if arm in ("nvattn+argmax", "nvattn+all"):
        nanovllm_dropin.install_greedy_argmax()
    if arm == "nvattn+all":
        nanovllm_dropin.install_fused_prologue()
        nanovllm_dropin.install_mixed_step_graph()
    costs_file = os.environ.get(ENV_COSTS)
    if costs_file and os.path.exists(costs_file):
        with open(costs_file) as f:
            table = json.load(f)
        costs = {int(k): v for k, v in table["costs"].items()}
        bks = {int(k): v for k, v in table["buckets"].items()}
        mr.ModelRunner.measure_step_costs = lambda self, *a, **k: (costs, bks)


def install_proposer(llm, kind: str, prompts: list[list[int]], replay: list[list[int]] | None = None,
                     seed: int = 0) -> None:
    """Replace the engine's n-gram guesses (on rank 0, where the proposer runs), as the reference's bench.py does for
    its worst case (--spec-proposer random, bench.py:143-146):
      random  uniformly random token ids: almost never accepted, so every decode step verifies k guesses and
              keeps only the model's own token;
      replay  the tokens a plain greedy run produced for the same prompt (`replay`), i.e. the guesses a perfect
              proposer would make: accepted until the first bf16 near-tie between the two runs' batch shapes.
    Either way the speculative path (guesses shipped to every rank, verify, accept) runs on every decode step,
    which n-gram lookups on a random-init model (whose output does not repeat itself) rarely reach."""
    import random
    if kind == "ngram":
        return
    assert llm.proposer is not None, "proposer replacement needs speculative_method='ngram'"
    if kind == "random":
        rng = random.Random(seed)
        vocab = llm.config.hf_config.vocab_size
        llm.proposer.propose = lambda seq, k: [rng.randrange(vocab) for _ in range(max(k, 0))]
        return
    assert kind == "replay" and replay is not None
    by_prompt = {tuple(p): r for p, r in zip(prompts, replay)}

    def propose(seq, k):
        done = seq.num_completion_tokens
        future = by_prompt.get(tuple(seq.prompt_token_ids), [])
        return list(future[done:done + max(k, 0)])
    llm.proposer.propose = propose


def run_arm(arm: str, variant: str, prompts: list[list[int]], max_tokens: int, model_path: str, tp: int = 1,
            step_costs_file: str | None = None, save_step_costs: str | None = None, weight_seed: int = 0,
            proposer: str = "ngram", replay: list[list[int]] | None = None,
            shape_warmup: list[list[int]] | None = None, **engine_overrides) -> dict:
    """One engine run in this process: build LLM(model_path, ...) with the arm's attention, generate greedily
    (ignore_eos, exactly max_tokens per request) and return tokens, timing and speculative-decoding counters.
    `shape_warmup`: requests shaped like the measured ones (other ids, so no prefix-cache block is shared), run for
    32 new tokens before the measurement, so that the first calls at the measured batch sizes (torch.compile of the
    sampler and norms for those shapes) happen outside the timed generate()."""
    assert arm in ARMS, arm
    os.environ[ENV_ARM], os.environ[ENV_TP], os.environ[ENV_SEED] = arm, str(tp), str(weight_seed)
    if step_costs_file:
        os.environ[ENV_COSTS] = os.path.abspath(step_costs_file)
    _apply_from_env()
    if tp > 1:    # a leftover block from a run that died would stop ModelRunner from creating it
        from multiprocessing import shared_memory
        try:
            shared_memory.SharedMemory(name="nanovllm").unlink()
        except FileNotFoundError:
            pass
    import torch
    from nanovllm import LLM, SamplingParams
    kwargs = dict(VARIANTS[variant], tensor_parallel_size=tp)
    if kwargs.get("draft_model") == "SELF":
        kwargs["draft_model"] = model_path
    kwargs.update(engine_overrides)
    t0 = time.perf_counter()
    llm = LLM(model_path, **kwargs)
    init_s = time.perf_counter() - t0
    install_proposer(llm, proposer, prompts, replay)
    if save_step_costs and llm.step_costs is not None:
        with open(save_step_costs, "w") as f:
            json.dump({"costs": llm.step_costs, "buckets": llm.step_cost_buckets}, f)
    # Warm-up of the reference's own bench.py (bench.py:248-253): first calls with new shapes are slow (torch.compile
    # of the sampler and norms, kernel setup), so one request, then four of 64-256 tokens, 32 new tokens each; their
    # tokens share no prefix-cache block with the measured prompts.  Counters are reset after it.
    warm = [[100 + i % (3 + j) for i in range(64 * (j + 1))] for j in range(4)]
    for batch in (warm[:1], warm) + ((shape_warmup,) if shape_warmup else ()):
        llm.generate(batch, SamplingParams(temperature=0, max_tokens=32, ignore_eos=True), use_tqdm=False)
    llm.reset_spec_stats()
    llm.num_mixed_steps = 0
    sp = SamplingParams(temperature=0, max_tokens=max_tokens, ignore_eos=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    outputs = llm.generate(prompts, sp, use_tqdm=False)
    torch.cuda.synchronize()
    gen_s = time.perf_counter() - t0
    tokens = [o["token_ids"] for o in outputs]
    n_out = sum(len(t) for t in tokens)
    result = {
        "arm": arm, "variant": variant, "tp": tp, "proposer": proposer, "tokens": tokens, "output_tokens": n_out,
        "generate_s": gen_s, "output_tok_per_s": n_out / gen_s, "init_s": init_s,
        "num_kvcache_blocks": llm.config.num_kvcache_blocks, "mixed_steps": llm.num_mixed_steps,
        "spec": llm.get_spec_stats() if llm.spec_method else None,
    }
    if arm.startswith("nvattn"):
        from nvattn import _lib
        result["device_error"] = _lib.device_error()
    llm.exit()
    import atexit
    atexit.unregister(llm.exit)
    return result


_apply_from_env()    # spawned TP workers: install the parent's patches before ModelRunner is unpickled


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("--arm", choices=ARMS, required=True)
    p.add_argument("--variant", choices=list(VARIANTS), default="spec_ngram_dynk_graph")
    p.add_argument("--tp", type=int, default=1)
    p.add_argument("--num-prompts", type=int, default=64)
    p.add_argument("--prompt-len", type=int, default=1024)
    p.add_argument("--max-tokens", type=int, default=256)
    p.add_argument("--seed", type=int, default=0, help="prompt seed")
    p.add_argument("--weight-seed", type=int, default=0)
    p.add_argument("--model-dir", default=None, help="where to write config.json (default: a temporary directory)")
    p.add_argument("--step-costs", default=None, help="inject this dynamic-k cost table (JSON) if the file exists")
    p.add_argument("--synthetic-step-costs", action="store_true", help="write synthetic_step_costs() to --step-costs first")
    p.add_argument("--save-step-costs", default=None, help="write the table this arm measured")
    p.add_argument("--proposer", choices=["ngram", "random", "replay"], default="ngram",
                   help="replace the n-gram guesses (n-gram variants only), see install_proposer")
    p.add_argument("--replay-from", default=None, help="--proposer replay: a result JSON of a plain greedy run")
    p.add_argument("--max-num-seqs", type=int, default=None)
    p.add_argument("--gpu-memory-utilization", type=float, default=None)
    p.add_argument("--shape-warmup", action="store_true",
                   help="also warm up on requests of the measured shape (prompt seed + 1, 32 new tokens)")
    p.add_argument("--out", required=True)
    a = p.parse_args(argv)
    import tempfile
    model_path = write_model_dir(a.model_dir or tempfile.mkdtemp(prefix="qwen3_8b_random_"))
    if a.synthetic_step_costs:
        assert a.step_costs, "--synthetic-step-costs needs --step-costs FILE"
        costs, bks = synthetic_step_costs(max_num_seqs=a.max_num_seqs or 512)
        with open(a.step_costs, "w") as f:
            json.dump({"costs": costs, "buckets": bks}, f)
    overrides = {}
    if a.max_num_seqs:
        overrides["max_num_seqs"] = a.max_num_seqs
    if a.gpu_memory_utilization:
        overrides["gpu_memory_utilization"] = a.gpu_memory_utilization
    prompts = config5_prompts(a.num_prompts, a.prompt_len, seed=a.seed)
    replay = None
    if a.replay_from:
        with open(a.replay_from) as f:
            replay = json.load(f)["tokens"]
    shape_warmup = config5_prompts(a.num_prompts, a.prompt_len, seed=a.seed + 1) if a.shape_warmup else None
    res = run_arm(a.arm, a.variant, prompts, a.max_tokens, model_path, a.tp, a.step_costs, a.save_step_costs,
                  a.weight_seed, a.proposer, replay, shape_warmup, **overrides)
    res["prompts_seed"], res["num_prompts"], res["prompt_len"] = a.seed, a.num_prompts, a.prompt_len
    res["shape_warmup"] = bool(shape_warmup)
    with open(a.out, "w") as f:
        json.dump(res, f)
    print(json.dumps({k: v for k, v in res.items() if k != "tokens"}))


if __name__ == "__main__":
    main()
