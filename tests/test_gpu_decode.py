"""GPU parity of paged decode (n = 1) and speculative verify (n = k + 1) attention against the FP32 oracle,
plus the properties nano-vllm relies on: batch-padding invariance (scripts/check_padding.py), zero output for
empty sequences, robustness to stale NaN past the context length, and CUDA-graph replay == eager."""
import pytest
import torch

import oracle
from conftest import assert_attn_close

pytestmark = pytest.mark.gpu


def run_decode(b):
    from nvattn import ops
    B = b.num_seqs
    n = b.q_per_seq
    H, D = b.q.shape[1], b.q.shape[2]
    q = b.q.view(B, n, H, D)
    return ops.flash_attn_with_kvcache(q, b.k_cache, b.v_cache, cache_seqlens=b.context_lens,
                                       block_table=b.block_tables, softmax_scale=b.scale)


def ref_decode(b):
    B, n = b.num_seqs, b.q_per_seq
    H, D = b.q.shape[1], b.q.shape[2]
    return oracle.paged_attention_ref(b.q.cpu().view(B, n, H, D), b.k_cache.cpu(), b.v_cache.cpu(),
                                      b.context_lens.cpu(), b.block_tables.cpu(), b.scale)


def batch(lens, n=1, H=32, KVH=8, NB=256, seed=0, **kw):
    from nvattn.workloads import paged_decode_batch
    return paged_decode_batch(lens, n, H, KVH, 128, NB, 0.5, seed, device="cuda", **kw)


@pytest.mark.parametrize("lens", [[1], [127], [128], [129], [256], [257], [1, 2, 3, 300, 511, 512, 513, 1000]])
def test_decode_small(cuda, lens):
    b = batch(lens, seed=len(lens))
    assert_attn_close(run_decode(b), ref_decode(b), f"lens={lens}")


def test_decode_config1_shape(cuda):
    """BASELINE config 0 geometry (16 q heads, 8 kv heads: group 2) in bf16."""
    from nvattn.workloads import paged_decode_batch
    b = paged_decode_batch([37, 256, 513, 1000], 1, 16, 8, 128, 64, 1.0, 0, device="cuda")
    assert_attn_close(run_decode(b), ref_decode(b), "config1")


def test_decode_config2_full(cuda):
    """Qwen3-8B decode, B=64, context U[512, 4096], 2048-block pool."""
    from nvattn.workloads import decode_config
    b = decode_config(seed=0, device="cuda")
    assert_attn_close(run_decode(b), ref_decode(b), "config2")


def test_decode_long_single_sequence_splits(cuda):
    """One 4096-token sequence: its 8 kv-head segments are cut across many CTAs (more than 16 pieces each) and
    merged in the kernel."""
    b = batch([4096], NB=32, seed=5)
    assert_attn_close(run_decode(b), ref_decode(b), "split")


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_decode_tp_head_shards(cuda, tp):
    """Per-rank head shard at TP=t (qwen3.py:29-39): 32/t q heads over 8/t kv heads."""
    b = batch([700, 1500, 64, 3000], H=32 // tp, KVH=8 // tp, seed=tp)
    assert_attn_close(run_decode(b), ref_decode(b), f"tp{tp}")


@pytest.mark.parametrize("k", [1, 2, 4, 8, 11])
def test_verify(cuda, k):
    b = batch([k + 1, 200, 256, 257, 1024, 1500], n=k + 1, seed=10 + k)
    assert_attn_close(run_decode(b), ref_decode(b), f"verify k={k}")


@pytest.mark.parametrize("lens", [[9], [127], [128, 136], [137, 263], [264, 265], [383, 384, 385]])
def test_verify_k8_tile_edges(cuda, lens):
    """k = 8 (36 rows, the 48-row variant) where the last draft position's visible range ends at, just before and
    just after a 128-key tile edge: tiles every row sees in full take the unmasked path, the rest the masked one."""
    b = batch(lens, n=9, seed=len(lens) + lens[0])
    assert_attn_close(run_decode(b), ref_decode(b), f"k=8 tile edges {lens}")


@pytest.mark.parametrize("k", [1, 2, 4, 8])
def test_verify_config3_full(cuda, k):
    """B=32, context U[256, 2048], k+1 causal queries per sequence."""
    from nvattn.workloads import verify_config
    b = verify_config(k, seed=k, device="cuda")
    assert_attn_close(run_decode(b), ref_decode(b), f"config3 k={k}")


@pytest.mark.parametrize("n", [1, 5, 9, 12])
def test_rising_scores_rescale_and_merge(cuda, n):
    """Scores that rise along the keys (dim 0 of every query is 4, dim 0 of key p gains 0.3 p: ~9.8 in log2 units
    per 64 keys): every tile moves the row maxima past the 2^8 rescale threshold, and the pieces of a split sequence
    reach the in-kernel merge with log-sum-exps hundreds of log2 units apart.  n = 9 and 12 (36 and 48 rows) run the
    48-row variant whose O stays in TMEM: every tile there scales the accumulated O by alpha before its PV product."""
    lens = [2000, 700, 129, 4000]
    b = batch(lens, n=n, seed=41)
    for i, L in enumerate(lens):
        pos = torch.arange(L, device=cuda)
        pages = b.block_tables[i, pos // 256].long()
        b.k_cache[pages, pos % 256, :, 0] += (0.3 * pos.float())[:, None].to(b.k_cache.dtype)
    b.q[:, :, 0] = 4.0
    assert_attn_close(run_decode(b), ref_decode(b), f"rising scores n={n}")


@pytest.mark.parametrize("n", [3, 9])
def test_padding_sequences_zero_and_invariant(cuda, n):
    """Padded sequences (length 0, table -1) output zeros, and real rows are bitwise identical with and without
    the padding (the check_padding.py property that eager == CUDA-graph runs rely on)."""
    lens = [300, 1200, 4000]
    a = batch(lens, n=n, seed=3)
    p = batch(lens, n=n, seed=3, pad_seqs=13)
    oa = run_decode(a)
    op = run_decode(p)
    assert torch.equal(oa, op[:3])
    assert op[3:].abs().sum() == 0


@pytest.mark.parametrize("n", [2, 9])
def test_stale_nan_past_context_is_ignored(cuda, n):
    """Cache rows past a sequence's length inside its last block may hold anything (torch.empty pool, rejected
    drafts); they must not leak into the output."""
    lens = [100, 300, 129]
    b = batch(lens, n=n, seed=4)
    ref = ref_decode(b)
    for i, L in enumerate(lens):
        nblk = (L + 255) // 256
        last = int(b.block_tables[i, nblk - 1])
        b.k_cache[last, L % 256 or 256:] = float("nan")
        b.v_cache[last, L % 256 or 256:] = float("nan")
    assert_attn_close(run_decode(b), ref, "nan tail")


@pytest.mark.parametrize("n", [5, 12])
def test_cuda_graph_replay_matches_eager(cuda, n):
    from nvattn import ops
    b = batch([513, 77, 2048, 1], n=n, seed=6)
    eager = run_decode(b)
    B, H, D = b.num_seqs, 32, 128
    q_static = b.q.view(B, n, H, D).clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        run_decode(b)   # warm-up on the side stream
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = ops.flash_attn_with_kvcache(q_static, b.k_cache, b.v_cache, cache_seqlens=b.context_lens,
                                          block_table=b.block_tables, softmax_scale=b.scale)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    # new lengths in the same static buffers: the replay follows the device data
    b.context_lens.copy_(torch.tensor([400, 77, 1000, 0], dtype=torch.int32))
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, run_decode(b))


def test_no_device_error_after_runs(cuda):
    from nvattn import _lib
    _lib.clear_device_error()
    b = batch([300, 600], n=2, seed=8)
    run_decode(b)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("name", ["decode", "verify_k3", "verify_k8_padded", "mixed_paged", "prefill_contiguous"])
def test_kernels_match_flash_attn_golden(cuda, name):
    """Our kernels against flash-attn 2.8.3's outputs (the reference's attention library) on the same inputs."""
    from nvattn import ops
    from test_oracle import fa2_case
    kind, args, _, fa2_out = fa2_case(name)      # also puts tests/golden on sys.path
    import make_golden_fa2 as mg
    b = mg.build(kind, args, device="cuda")
    if kind == "paged_decode":
        B, n = b.num_seqs, b.q_per_seq
        got = ops.flash_attn_with_kvcache(b.q.view(B, n, 8, 128), b.k_cache, b.v_cache, cache_seqlens=b.context_lens,
                                          block_table=b.block_tables, softmax_scale=b.scale).reshape(B * n, 8, 128)
    else:
        paged = b.meta["paged"]
        k, v, bt = (b.k_cache, b.v_cache, b.block_tables) if paged else (b.k_new, b.v_new, None)
        got = ops.flash_attn_varlen_func(b.q, k, v, max_seqlen_q=b.max_seqlen_q, cu_seqlens_q=b.cu_seqlens_q,
                                         max_seqlen_k=b.max_seqlen_k, cu_seqlens_k=b.cu_seqlens_k,
                                         softmax_scale=b.scale, causal=True, block_table=bt)
    assert_attn_close(got, fa2_out.float(), f"kernels vs flash-attn: {name}")


@pytest.mark.parametrize("pieces_case", ["two_pieces", "table", "many_pieces", "wide_two_pieces"])
def test_merge_tickets_left_zero_and_repeatable(cuda, pieces_case):
    """The workspace contract: the merge tickets (first block of the workspace) are zero again after every call,
    whichever merge path ran (two pieces, the weight table for 3..16 pieces, the plain loop beyond), and repeated
    calls sharing the workspace give bitwise identical outputs.  A varlen call in between shares the workspace."""
    from nvattn import ops
    from nvattn.workloads import varlen_batch
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    ticket_bytes = (2 * sms * 4 + 255) // 256 * 256
    lens = {"two_pieces": [1500] * 40, "table": [2048 * 3] * 4, "many_pieces": [4096],
            "wide_two_pieces": [1500] * 40}[pieces_case]
    n = {"two_pieces": 3, "wide_two_pieces": 10}.get(pieces_case, 1)   # (10 x 4 rows: the 48-row variant)
    b = batch(lens, n=n, NB=512, seed=21)
    first = run_decode(b).clone()
    ws = ops._WORKSPACES[torch.cuda.current_device()]
    torch.cuda.synchronize()
    assert int(ws[:ticket_bytes].count_nonzero()) == 0, "tickets not left at zero"
    v = varlen_batch([1, 3, 200], [300, 40, 900], 32, 8, 128, 64, 0.5, 3, device="cuda")
    ops.flash_attn_varlen_func(v.q, v.k_cache, v.v_cache, max_seqlen_q=v.max_seqlen_q, cu_seqlens_q=v.cu_seqlens_q,
                               max_seqlen_k=v.max_seqlen_k, cu_seqlens_k=v.cu_seqlens_k, softmax_scale=v.scale,
                               causal=True, block_table=v.block_tables)
    torch.cuda.synchronize()
    assert int(ws[:ticket_bytes].count_nonzero()) == 0, "tickets not zero after a varlen call"
    again = run_decode(b)
    assert torch.equal(first, again)
    assert_attn_close(again, ref_decode(b), f"tickets {pieces_case}")
