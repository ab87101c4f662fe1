"""Golden vectors for the fused attention prologue (nva_qk_norm_rope_store), made with the reference's own layers:
nanovllm.layers.layernorm.RMSNorm and nanovllm.layers.rotary_embedding.get_rope, run eagerly on the CPU (their
torch.compile is switched off: it needs a compiler toolchain for the CPU backend), applied as
Qwen3Attention.pre_attn applies them (nanovllm/models/qwen3.py:88-97).  Needs the reference importable (the
baseline/_ref install or the reference tree on PYTHONPATH).

    python tests/golden/make_golden_prologue.py  ->  tests/golden/prologue_golden.npz
"""
import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "baseline", "_ref"))
import torch._dynamo  # noqa: E402
torch._dynamo.config.disable = True
from nanovllm.layers.layernorm import RMSNorm  # noqa: E402
from nanovllm.layers.rotary_embedding import get_rope  # noqa: E402

CASES = {   # name: (tokens, q heads, kv heads, max position, rope base, seed)
    "qwen3_8b_decode": (32, 32, 8, 4096, 1000000.0, 0),
    "qwen3_8b_tp4": (37, 8, 2, 4096, 1000000.0, 1),
    "qwen3_0p6b": (19, 16, 8, 40960, 1000000.0, 2),
}


def main():
    out = {}
    for name, (T, H, KVH, max_pos, base, seed) in CASES.items():
        g = torch.Generator().manual_seed(seed)
        D = 128
        qkv = (torch.randn(T, (H + 2 * KVH) * D, generator=g) * 2.0).to(torch.bfloat16)
        positions = torch.randint(0, max_pos, (T,), generator=g, dtype=torch.int64)
        q_norm, k_norm = RMSNorm(D, 1e-6), RMSNorm(D, 1e-6)
        with torch.no_grad():
            q_norm.weight.copy_(1.0 + 0.25 * torch.randn(D, generator=g))
            k_norm.weight.copy_(1.0 + 0.25 * torch.randn(D, generator=g))
        q_norm, k_norm = q_norm.to(torch.bfloat16), k_norm.to(torch.bfloat16)
        get_rope.cache_clear()
        rope = get_rope(D, D, max_pos, base)
        q, k, v = qkv.split([H * D, KVH * D, KVH * D], dim=-1)
        with torch.no_grad():
            q = q_norm(q.reshape(-1, H, D))
            k = k_norm(k.reshape(-1, KVH, D))
            q, k = rope(positions, q, k)
        table = rope.cos_sin_cache.reshape(max_pos, D).contiguous()
        out[f"{name}/qkv"] = qkv.view(torch.int16).numpy()
        out[f"{name}/positions"] = positions.numpy()
        out[f"{name}/q_w"] = q_norm.weight.detach().view(torch.int16).numpy()
        out[f"{name}/k_w"] = k_norm.weight.detach().view(torch.int16).numpy()
        out[f"{name}/q"] = q.view(torch.int16).numpy()
        out[f"{name}/k"] = k.view(torch.int16).numpy()
        out[f"{name}/geometry"] = np.array([T, H, KVH, max_pos], dtype=np.int64)
        out[f"{name}/base"] = np.array([base])
        out[f"{name}/table_sha256"] = np.frombuffer(hashlib.sha256(table.numpy().tobytes()).digest(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, "prologue_golden.npz"), **out)
    print("wrote", len(out), "arrays")


if __name__ == "__main__":
    main()
