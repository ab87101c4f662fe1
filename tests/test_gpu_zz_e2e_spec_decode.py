"""End to end on a B200: nano-vllm-spec-decode's own engine with this package's attention swapped in, greedy
speculative decoding of a random-init Qwen3-8B (BASELINE config 5's model and prompt shape, a smaller workload:
8 requests of 1024 tokens, 48 new tokens each), against the unmodified reference (flash-attn 2.8.3 + Triton scatter)
on the same seeds.  Drafts come from the n-gram proposer (config 5's method; with random weights the model rarely
repeats itself within 48 tokens, so these runs are mostly plain decode steps) and from the model guessing for
itself (the reference's spec_draft variants: nearly every guess accepted, so every decode step is a k = 4 verify
step), plus mixed-batching runs (decode requests and prefill chunks in one step).  Arms: the reference; nvattn's
attention alone (nvattn); with the sharded greedy verify (nvattn+argmax); and the whole drop-in (nvattn+all: also
the fused q/k-norm + rotary + KV-scatter prologue, and mixed steps recorded as one CUDA graph each).

Checks, following the reference's tests/test_greedy.py (the method and its 0.5 tolerance, :1-30, 244-248):
  * every run's tokens face a float32 referee (tests/e2e_referee.py): each generated token must be the referee's
    top-1 or within 0.5 of its top-1 logit;
  * runs that compute exactly the same thing must give identical tokens: CUDA-graph vs eager steps with nvattn
    (the reference's MUST_MATCH pairs; with nvattn+all the graph side is the whole-step mixed graph, the eager side
    the reference's segment-by-segment path), and nvattn with and without the per-rank (max, index) greedy verify
    (which is bit-exact by construction);
  * self-drafting accepts at least 85% of the tested guesses in both arms (a wrong verify attention would reject
    guesses the draft pass, which shares no state with it, agrees on); the device error word of the nvattn kernels
    stays 0; the mixed run did run mixed steps.
Where the nvattn arm and the reference arm part ways, the first diverging position of each request is printed
with both tokens' referee gaps: a bf16 near-tie, not an error, when both are within the tolerance.

Needs the reference importable from baseline/_ref (pip install --target of the reference); skipped otherwise.
Each engine runs in its own process (each takes most of the GPU memory for its KV cache).
"""
import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "nano-vllm-spec-decode_b200")
sys.path.insert(0, PKG)

TOL = 0.5                 # max allowed float32 logit gap below top-1 (the reference's test_greedy.py default)
NUM_PROMPTS, PROMPT_LEN, MAX_TOKENS = 8, 1024, 48
RUNS = [                  # (name, arm, variant)
    ("ref_spec_graph", "reference", "spec_ngram_graph"),
    ("nva_spec_graph", "nvattn", "spec_ngram_graph"),
    ("nva_spec_eager", "nvattn", "spec_ngram"),
    ("ref_draft_graph", "reference", "spec_draft_graph"),
    ("nva_draft_graph", "nvattn", "spec_draft_graph"),
    ("nva_draft_eager", "nvattn", "spec_draft"),
    ("nva_argmax_draft_graph", "nvattn+argmax", "spec_draft_graph"),
    ("nva_mixed_graph", "nvattn", "mixed_graph"),
    ("nva_mixed_eager", "nvattn", "mixed_eager"),
    ("all_draft_graph", "nvattn+all", "spec_draft_graph"),
    ("all_mixed_graph", "nvattn+all", "mixed_graph"),
    ("all_mixed_eager", "nvattn+all", "mixed_eager"),
]
MUST_MATCH = {"nva_spec_eager": "nva_spec_graph", "nva_draft_eager": "nva_draft_graph",
              "nva_argmax_draft_graph": "nva_draft_graph", "nva_mixed_eager": "nva_mixed_graph",
              "all_mixed_eager": "all_mixed_graph"}
# A model guessing for itself: the guesses come from the same weights with other batch shapes, so only bf16
# near-ties reject one (0.92-0.93 measured in both arms with these random weights; the reference's test_greedy.py
# asks 0.95 of real weights).  A wrong verify attention rejects far more.
MIN_ACCEPTANCE = 0.85


def _reference_available() -> bool:
    return os.path.isdir(os.path.join(REPO, "baseline", "_ref", "nanovllm"))


def _run(cmd, timeout):
    env = dict(os.environ, PYTHONPATH=PKG + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, f"{' '.join(cmd)} failed:\n{r.stdout[-3000:]}\n{r.stderr[-6000:]}"


def first_diff(a, b):
    n = min(len(a), len(b))
    return next((j for j in range(n) if a[j] != b[j]), n if len(a) != len(b) else None)


@pytest.mark.gpu
def test_spec_decode_end_to_end(tmp_path):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    if not _reference_available():
        pytest.skip("the reference is not installed under baseline/_ref")
    from nvattn.e2e import write_model_dir, config5_prompts
    model_dir = write_model_dir(str(tmp_path / "qwen3_8b_random"))
    results = {}
    for name, arm, variant in RUNS:
        out = tmp_path / f"{name}.json"
        _run([sys.executable, "-m", "nvattn.e2e", "--arm", arm, "--variant", variant, "--model-dir", model_dir,
              "--num-prompts", str(NUM_PROMPTS), "--prompt-len", str(PROMPT_LEN), "--max-tokens", str(MAX_TOKENS),
              "--max-num-seqs", "16", "--out", str(out)], timeout=1200)
        results[name] = json.loads(out.read_text())
    prompts = config5_prompts(NUM_PROMPTS, PROMPT_LEN)
    runs = {name: r["tokens"] for name, r in results.items()}
    (tmp_path / "runs.json").write_text(json.dumps({"prompts": prompts, "runs": runs}))
    _run([sys.executable, os.path.join(REPO, "tests", "e2e_referee.py"), "--model-dir", model_dir,
          "--inp", str(tmp_path / "runs.json"), "--out", str(tmp_path / "gaps.json")], timeout=1200)
    gaps = json.loads((tmp_path / "gaps.json").read_text())

    report = {}
    for name, r in results.items():
        flat = [g for seq in gaps[name] for g in seq]
        same_ref = sum(first_diff(a, b) is None for a, b in zip(runs["ref_spec_graph"], runs[name]))
        report[name] = dict(tokens=len(flat), not_top1=sum(g > 0 for g in flat), worst_gap=max(flat),
                            same_as_reference=f"{same_ref}/{NUM_PROMPTS}", tok_per_s=round(r["output_tok_per_s"], 1),
                            spec=r["spec"] and {k: r["spec"][k] for k in ("num_drafts", "num_accepted", "num_rejected",
                                                                          "k_steps")},
                            mixed_steps=r["mixed_steps"], device_error=r.get("device_error"))
    divergences = []
    for ref_name, nva_name in (("ref_spec_graph", "nva_spec_graph"), ("ref_draft_graph", "nva_draft_graph")):
        for i, (a, b) in enumerate(zip(runs[ref_name], runs[nva_name])):
            j = first_diff(a, b)
            if j is not None:
                divergences.append(dict(runs=f"{ref_name} / {nva_name}", request=i, position=j, reference_token=a[j],
                                        nvattn_token=b[j], reference_gap=gaps[ref_name][i][j],
                                        nvattn_gap=gaps[nva_name][i][j]))
    print(json.dumps({"runs": report, "reference_vs_nvattn_divergences": divergences}, indent=1))

    for name in results:
        assert report[name]["worst_gap"] <= TOL, f"{name}: a token {report[name]['worst_gap']:.3f} below the referee's top-1"
        if name.startswith("nva"):
            assert results[name]["device_error"] == 0, f"{name}: device error word {results[name]['device_error']}"
    for name, partner in MUST_MATCH.items():
        same = sum(first_diff(a, b) is None for a, b in zip(runs[partner], runs[name]))
        assert same == NUM_PROMPTS, f"{name} differs from {partner} on {NUM_PROMPTS - same} of {NUM_PROMPTS} requests"
    for name in ("ref_draft_graph", "nva_draft_graph", "nva_draft_eager", "nva_argmax_draft_graph", "all_draft_graph"):
        s = results[name]["spec"]
        rate = s["num_accepted"] / max(s["num_accepted"] + s["num_rejected"], 1)
        assert s["num_drafts"] > 0 and rate >= MIN_ACCEPTANCE, f"{name}: acceptance {rate:.3f} of {s['num_drafts']}"
    for name in ("nva_mixed_graph", "all_mixed_graph"):
        assert results[name]["mixed_steps"] > 0, f"{name}: no mixed step ran"
    for d in divergences:
        assert d["reference_gap"] <= TOL and d["nvattn_gap"] <= TOL
