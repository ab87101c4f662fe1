"""Float32 referee for the end-to-end greedy runs (test infrastructure, used by test_gpu_zz_e2e_spec_decode.py).

The method is the reference's own (tests/test_greedy.py:1-30, 161-173): bf16 engines cannot promise identical
tokens (logits are rounded to a few significant digits, so near-ties flip with any change in computation order),
so every generated token is checked against a float32 run of the same model instead.  The referee is Hugging Face
transformers' Qwen3ForCausalLM in float32 with the same seeded weights (nvattn.e2e.seeded_weight, the bf16 values
widened to float32); for every generated token it reports how far the token's float32 logit lies below the float32
top-1 logit at that position (0 = the token is the referee's top-1).  A wrong KV cache, position or block gives
tokens far from top-1 within a few steps.

    python tests/e2e_referee.py --model-dir DIR --inp runs.json --out gaps.json
runs.json: {"prompts": [[ids]...], "runs": {name: [[generated ids]...]}}; gaps.json: {name: [[gap per token]...]}.
"""
import argparse
import json
import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(REPO, "nano-vllm-spec-decode_b200"))


def build_referee(model_dir: str, weight_seed: int):
    import torch
    from transformers import AutoConfig, Qwen3ForCausalLM
    from nvattn.e2e import checkpoint_shapes, seeded_weight
    cfg = AutoConfig.from_pretrained(model_dir)
    cfg.dtype = torch.float32
    torch.set_default_dtype(torch.float32)
    with torch.device("cuda"):
        model = Qwen3ForCausalLM(cfg)
    with open(os.path.join(model_dir, "config.json")) as f:
        raw = json.load(f)
    with torch.no_grad():
        for name, shape in checkpoint_shapes(raw).items():
            model.get_parameter(name).copy_(seeded_weight(name, shape, weight_seed, dtype=torch.float32))
    return model.eval()


def gaps_for(model, prompts, runs):
    import torch
    out = {}
    with torch.inference_mode():
        for name, outputs in runs.items():
            out[name] = []
            for prompt, gen in zip(prompts, outputs):
                x = torch.tensor([prompt + gen], device="cuda")
                logits = model(input_ids=x).logits[0, len(prompt) - 1:-1].float()
                chosen = logits.gather(1, torch.tensor(gen, device="cuda").unsqueeze(1)).squeeze(1)
                out[name].append((logits.max(dim=1).values - chosen).tolist())
    return out


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--model-dir", required=True)
    p.add_argument("--weight-seed", type=int, default=0)
    p.add_argument("--inp", required=True)
    p.add_argument("--out", required=True)
    a = p.parse_args()
    with open(a.inp) as f:
        data = json.load(f)
    model = build_referee(a.model_dir, a.weight_seed)
    with open(a.out, "w") as f:
        json.dump(gaps_for(model, data["prompts"], data["runs"]), f)


if __name__ == "__main__":
    main()
