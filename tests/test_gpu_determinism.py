"""The kernels' results do not depend on scheduling.  Each work item of the prefill kernels is computed whole by
the CTA that takes it from the work counter, and the decode kernel's split and merge order follow from the lengths
alone, so a call gives bitwise the same output however its CTAs are placed and timed.  Checked here by repeating
calls while a GEMM on another stream holds a varying share of the SMs (so CTAs start late, in other orders, and the
work counter hands items to other CTAs), on the mixed step of BASELINE config 4, a chunked-prefill batch of the
shape nano-vllm's mixed batching makes (256-token budget: chunks of up to 256 tokens over paged prefixes plus decode
rows), the two-tile prefill kernel and verify k = 8."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _cases():
    from nvattn.workloads import mixed_config, varlen_batch, verify_config
    yield "mixed_config4", mixed_config(seed=0, device="cuda"), "varlen"
    q_lens = [1] * 6 + [5] * 4 + [200, 256, 37]
    k_lens = [300 + 97 * i for i in range(10)] + [1224, 520, 37]
    yield "mixed_budget256", varlen_batch(q_lens, k_lens, 32, 8, 128, 64, 0.5, 5, device="cuda"), "varlen"
    yield "prefill_pair_16x1024", varlen_batch([1024] * 16, [1024] * 16, 32, 8, 128, 64, 0.5, 42, device="cuda",
                                               paged=False), "varlen"
    yield "verify_k8", verify_config(8, seed=0, device="cuda", device_fill=True), "decode"


@pytest.mark.parametrize("which", ["mixed_config4", "mixed_budget256", "prefill_pair_16x1024", "verify_k8"])
def test_outputs_independent_of_sm_share(cuda, which):
    from nvattn import ops, _lib
    name, b, kind = next(c for c in _cases() if c[0] == which)
    if kind == "varlen":
        paged = b.meta.get("paged", True)
        k, v, bt = (b.k_cache, b.v_cache, b.block_tables) if paged else (b.k_new, b.v_new, None)

        def call():
            return ops.flash_attn_varlen_func(b.q, k, v, max_seqlen_q=b.max_seqlen_q, cu_seqlens_q=b.cu_seqlens_q,
                                              max_seqlen_k=b.max_seqlen_k, cu_seqlens_k=b.cu_seqlens_k,
                                              softmax_scale=b.scale, causal=True, block_table=bt)
    else:
        q = b.q.view(b.num_seqs, b.q_per_seq, b.q.shape[1], b.q.shape[2])

        def call():
            return ops.flash_attn_with_kvcache(q, b.k_cache, b.v_cache, cache_seqlens=b.context_lens,
                                               block_table=b.block_tables, softmax_scale=b.scale)
    _lib.clear_device_error()
    ref = call()
    torch.cuda.synchronize()
    a = torch.randn(4096, 4096, device=cuda, dtype=torch.bfloat16)
    side = torch.cuda.Stream()
    for i in range(24):
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(i % 6):
                a = (a @ a).clamp_(-1, 1)
        out = call()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        assert torch.equal(out, ref), f"{name}: call {i} differs"
    assert _lib.device_error() == 0
