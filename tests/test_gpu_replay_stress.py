"""Long CUDA-graph replay runs of the full-size decode (config 2), verify (config 3, k = 8) and mixed (config 4)
steps, of a prefill of sixteen 1024-token prompts and of the two-tile prefill kernel on sixty-four prompts of at most
128 tokens (every item one tile), as nano-vllm replays its captured steps: every replay must finish without any bounded wait giving up (the
device error word stays 0) and give bitwise the same output as the eager call (the kernels are deterministic:
the split, the merge order and each item's arithmetic depend only on the inputs).  Timing-dependent races between
the kernels' warp roles, or between the chained kernels of a varlen call, would show up here as a set error bit or
a changed output."""
import pytest
import torch

pytestmark = pytest.mark.gpu

REPLAYS = 300


def _capture(fn):
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g


def _decode_call(b, out):
    from nvattn import ops
    n = b.q_per_seq
    q = b.q.view(b.num_seqs, n, b.q.shape[1], b.q.shape[2])

    def call():
        ops.flash_attn_with_kvcache(q, b.k_cache, b.v_cache, cache_seqlens=b.context_lens,
                                    block_table=b.block_tables, softmax_scale=b.scale, out=out)
    return call


def _varlen_call(b, out):
    from nvattn import ops
    paged = b.meta.get("paged", True)
    k, v, bt = (b.k_cache, b.v_cache, b.block_tables) if paged else (b.k_new, b.v_new, None)

    def call():
        ops.flash_attn_varlen_func(b.q, k, v, max_seqlen_q=b.max_seqlen_q, cu_seqlens_q=b.cu_seqlens_q,
                                   max_seqlen_k=b.max_seqlen_k, cu_seqlens_k=b.cu_seqlens_k, softmax_scale=b.scale,
                                   causal=True, block_table=bt, out=out)
    return call


@pytest.mark.parametrize("case", ["decode_config2", "verify_config3_k8", "mixed_config4", "prefill_16x1024",
                                  "prefill_pair_short_items"])
def test_graph_replays_stay_clean_and_bitwise_stable(cuda, case):
    from nvattn import _lib
    from nvattn.workloads import decode_config, mixed_config, varlen_batch, verify_config
    if case in ("mixed_config4", "prefill_16x1024", "prefill_pair_short_items"):
        if case == "mixed_config4":
            b = mixed_config(seed=0, device="cuda")
        elif case == "prefill_16x1024":
            b = varlen_batch([1024] * 16, [1024] * 16, 32, 8, 128, 64, 0.5, 42, device="cuda", paged=False)
        else:    # the two-tile kernel with one-tile items only (loose max_seqlen_q): the item ring laps group 1
            lens = [100 + (11 * i) % 29 for i in range(64)]
            b = varlen_batch(lens, lens, 32, 8, 128, 64, 0.5, 43, device="cuda", paged=False)
            b.max_seqlen_q = 4096
        out = torch.empty_like(b.q)
        call = _varlen_call(b, out)
    else:
        b = (decode_config(seed=0, device="cuda", device_fill=True) if case == "decode_config2"
             else verify_config(8, seed=0, device="cuda", device_fill=True))
        out = torch.empty(b.num_seqs, b.q_per_seq, b.q.shape[1], b.q.shape[2], dtype=b.q.dtype, device=cuda)
        call = _decode_call(b, out)
    _lib.clear_device_error()
    call()
    torch.cuda.synchronize()
    ref = out.clone()
    assert _lib.device_error() == 0
    g = _capture(call)
    for i in range(REPLAYS):
        out.fill_(float("nan"))
        g.replay()
        if i % 50 == 49 or i == REPLAYS - 1:
            torch.cuda.synchronize()
            assert _lib.device_error() == 0, f"a bounded wait gave up by replay {i}"
            assert torch.equal(out, ref), f"replay {i} differs from the eager call"
    g.reset()
