"""Torch restatement of Qwen3's attention prologue (test infrastructure only, see oracle/__init__.py).

qwen3.py:88-97 on the fused projection output: q / k split into heads, RMSNorm of each head over its 128 dims
(layers/layernorm.py:16-26: float32 x * rsqrt(mean(x^2) + eps), rounded to bf16, times the bf16 weight), rotary
embedding (layers/rotary_embedding.py:6-14 and 37-48: rotate-half in float32 with the float32 cos / sin table of
positions, rounded to bf16), then the KV scatter of Attention.forward (attention.py:61-62).  Eager torch ops on the
CPU, in the reference's own order.
"""
import torch


def rope_table(head_dim: int, max_position: int, base: float) -> torch.Tensor:
    """[max_position, head_dim] float32: cos of the rotation angles in the first half of each row, sin in the
    second (RotaryEmbedding.__init__, rotary_embedding.py:27-35)."""
    inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float) / head_dim))
    t = torch.arange(max_position, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    dt = x.dtype
    x = x.float()
    var = x.pow(2).mean(dim=-1, keepdim=True)
    x = x * torch.rsqrt(var + eps)
    return x.to(dt) * weight


def rotary(x: torch.Tensor, table: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
    cos, sin = table[positions].unsqueeze(1).chunk(2, dim=-1)
    x1, x2 = torch.chunk(x.float(), 2, dim=-1)
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1).to(x.dtype)


def qk_prologue_ref(qkv: torch.Tensor, positions: torch.Tensor, table: torch.Tensor, q_w: torch.Tensor,
                    k_w: torch.Tensor, eps: float, H: int, KVH: int, D: int = 128):
    """qkv [T, (H + 2 KVH) D] bf16 -> (q [T, H, D], k [T, KVH, D], v [T, KVH, D]) as Qwen3Attention.pre_attn."""
    q, k, v = qkv.split([H * D, KVH * D, KVH * D], dim=-1)
    q = rms_norm(q.reshape(-1, H, D), q_w, eps)
    k = rms_norm(k.reshape(-1, KVH, D), k_w, eps)
    return rotary(q, table, positions), rotary(k, table, positions), v.reshape(-1, KVH, D)
