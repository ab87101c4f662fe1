"""GPU parity of varlen attention (flash_attn_varlen_func's role at attention.py:64-70): prefill without a prefix
(contiguous K/V), chunked prefill over a paged prefix, the mixed prefill+decode batch of BASELINE config 4, and the
Attention module itself driven through the Context, all against the FP32 oracle."""
import pytest
import torch

import oracle
from conftest import assert_attn_close

pytestmark = pytest.mark.gpu


def run_varlen(b, paged=True):
    from nvattn import ops
    if paged:
        k, v, bt = b.k_cache, b.v_cache, b.block_tables
    else:
        k, v, bt = b.k_new, b.v_new, None
    return ops.flash_attn_varlen_func(b.q, k, v, max_seqlen_q=b.max_seqlen_q, cu_seqlens_q=b.cu_seqlens_q,
                                      max_seqlen_k=b.max_seqlen_k, cu_seqlens_k=b.cu_seqlens_k,
                                      softmax_scale=b.scale, causal=True, block_table=bt)


def ref_varlen(b, paged=True):
    if paged:
        return oracle.varlen_attention_ref(b.q.cpu(), None, None, b.cu_seqlens_q.cpu(), b.cu_seqlens_k.cpu(),
                                           b.scale, block_tables=b.block_tables.cpu(), k_cache=b.k_cache.cpu(),
                                           v_cache=b.v_cache.cpu())
    return oracle.varlen_attention_ref(b.q.cpu(), b.k_new.cpu(), b.v_new.cpu(), b.cu_seqlens_q.cpu(),
                                       b.cu_seqlens_k.cpu(), b.scale)


def batch(q_lens, k_lens, H=32, KVH=8, NB=512, seed=0, paged=True):
    from nvattn.workloads import varlen_batch
    return varlen_batch(q_lens, k_lens, H, KVH, 128, NB, 0.5, seed, device="cuda", paged=paged)


@pytest.mark.parametrize("lens", [[1], [13], [64, 127, 128, 129], [300, 1, 1000, 5, 700]])
def test_prefill_contiguous(cuda, lens):
    """Prefill without a prefix: keys from the contiguous k/v rows (block_table None)."""
    b = batch(lens, lens, seed=len(lens), paged=False)
    assert_attn_close(run_varlen(b, paged=False), ref_varlen(b, paged=False), f"contiguous {lens}")


@pytest.mark.parametrize("q_lens,prefix", [([200], [0]), ([512, 640, 640], [0, 256, 1024]),
                                           ([129, 300, 77], [1, 383, 2000])])
def test_prefill_paged_prefix(cuda, q_lens, prefix):
    """Chunked prefill / prefix-cache hits: keys [0, prefix + q) from the paged cache."""
    k_lens = [q + p for q, p in zip(q_lens, prefix)]
    b = batch(q_lens, k_lens, seed=7)
    assert_attn_close(run_varlen(b), ref_varlen(b), f"paged prefix {q_lens}/{prefix}")


# Calls with rows x heads >= 4 x SMs x 256 (4736 rows at 32 heads on 148 SMs) take the kernel with two query tiles
# per work item (prefill_pair.cu); the cases above take the single-tile kernel.
@pytest.mark.parametrize("lens", [[1024, 1000, 1300, 129, 1500]])
def test_prefill_pair_contiguous(cuda, lens):
    """Two-tile items: full pairs, a partial second tile (1000, 129 rows) and a lone last tile (1300, 1500 rows)."""
    b = batch(lens, lens, seed=21, paged=False)
    assert_attn_close(run_varlen(b, paged=False), ref_varlen(b, paged=False), f"pair contiguous {lens}")


def test_prefill_pair_paged_prefix(cuda):
    q_lens, prefix = [1024, 640, 1500, 1700], [0, 256, 1024, 300]
    b = batch(q_lens, [q + p for q, p in zip(q_lens, prefix)], seed=22)
    assert_attn_close(run_varlen(b), ref_varlen(b), "pair paged prefix")


def test_prefill_pair_stale_nan_past_context(cuda):
    q_lens, k_lens = [1300, 1200, 1100, 1200], [1400, 1333, 1900, 1250]
    b = batch(q_lens, k_lens, seed=23)
    ref = ref_varlen(b)
    for i, L in enumerate(k_lens):
        last = int(b.block_tables[i, (L + 255) // 256 - 1])
        b.k_cache[last, L % 256 or 256:] = float("nan")
        b.v_cache[last, L % 256 or 256:] = float("nan")
    assert_attn_close(run_varlen(b), ref, "pair nan tail")


def test_prefill_pair_single_tile_items_only(cuda):
    """The two-tile kernel on a call whose every item has one query tile: 48 prompts of 100-128 tokens (5k rows at
    32 heads, above the two-tile threshold) with a loose max_seqlen_q bound (4096), which the C ABI takes as "some
    run may fill two tiles".  Softmax group 1 then skips every item, so the producer laps the 8-entry item ring
    many times while group 1 only reads and releases entries: the ring's read barrier is what keeps the entries
    valid.  Parity with the oracle and a clean device error word."""
    from nvattn import _lib
    lens = [100 + (7 * i) % 29 for i in range(48)]
    b = batch(lens, lens, seed=24, paged=False)
    b.max_seqlen_q = 4096
    _lib.clear_device_error()
    out = run_varlen(b, paged=False)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert_attn_close(out, ref_varlen(b, paged=False), "pair kernel, single-tile items")


def test_varlen_padding_sequences_invariant(cuda):
    """Batch padding in a mixed varlen step (the property the reference's scripts/check_padding.py:28-55 checks for
    decode): appending empty sequences (no query rows, no keys, block-table rows of -1) leaves every real row's
    output bitwise unchanged, on a mixed batch with decode rows, verify runs and prefill chunks."""
    from nvattn import ops
    q_lens = [1] * 40 + [5] * 8 + [300, 129]
    k_lens = [60 + 53 * i for i in range(48)] + [300 + 256, 129 + 1000]
    b = batch(q_lens, k_lens, seed=12)
    alone = run_varlen(b)
    pad = 6
    cu_q = torch.cat([b.cu_seqlens_q, b.cu_seqlens_q[-1:].repeat(pad)])
    cu_k = torch.cat([b.cu_seqlens_k, b.cu_seqlens_k[-1:].repeat(pad)])
    bt = torch.cat([b.block_tables, torch.full((pad, b.block_tables.shape[1]), -1, dtype=torch.int32, device=cuda)])
    padded = ops.flash_attn_varlen_func(b.q, b.k_cache, b.v_cache, max_seqlen_q=b.max_seqlen_q, cu_seqlens_q=cu_q,
                                        max_seqlen_k=b.max_seqlen_k, cu_seqlens_k=cu_k, softmax_scale=b.scale,
                                        causal=True, block_table=bt)
    assert torch.equal(alone, padded)
    assert_attn_close(alone, ref_varlen(b), "mixed batch before padding")


@pytest.mark.parametrize("lens", [[700, 300], [1200, 1200, 1200, 1200]])
def test_prefill_rising_scores_rescale_every_half_tile(cuda, lens):
    """Scores that rise along the keys: dim 0 of every query is 4 and dim 0 of key p gains 0.3 p, so each 64 keys
    raise a row's log2 score by ~9.8, past the 2^8 rescale threshold.  Every key tile then rescales O, and every
    second 64-key half rescales the first half's P (the two-tile kernel) or takes the exact vote path (the single-tile
    kernel).  [700, 300] runs the single-tile kernel, 4 x 1200 rows the two-tile one."""
    b = batch(lens, lens, seed=31, paged=False)
    cu = b.cu_seqlens_k.tolist()
    for i in range(len(lens)):
        pos = torch.arange(lens[i], device=cuda, dtype=torch.float32)
        b.k_new[cu[i]:cu[i + 1], :, 0] += (0.3 * pos)[:, None].to(b.k_new.dtype)
    b.q[:, :, 0] = 4.0
    assert_attn_close(run_varlen(b, paged=False), ref_varlen(b, paged=False), f"rising scores {lens}")


def test_varlen_decode_rows_only(cuda):
    """A mixed step whose every run is short (decode rows with 1+k tokens): handled by the decode kernel."""
    q_lens = [1] * 20 + [5] * 10 + [12] * 3
    k_lens = [50 + 37 * i for i in range(len(q_lens))]
    b = batch(q_lens, k_lens, seed=3)
    assert_attn_close(run_varlen(b), ref_varlen(b), "varlen decode rows")


def test_mixed_config4_full(cuda):
    """256 decode rows (log-normal contexts) + prefill chunks 512/640/640 with prefixes
    0/256/1024 in one varlen batch."""
    from nvattn.workloads import mixed_config
    b = mixed_config(seed=0, device="cuda")
    assert_attn_close(run_varlen(b), ref_varlen(b), "config4")


def test_mixed_group2_geometry(cuda):
    """Qwen3-0.6B geometry (16 q heads, 8 kv heads: group 2) in a mixed batch: short runs up to 24 rows."""
    q_lens = [1, 3, 24, 25, 300]
    k_lens = [40, 300, 500, 600, 900]
    b = batch(q_lens, k_lens, H=16, KVH=8, seed=11)
    assert_attn_close(run_varlen(b), ref_varlen(b), "group 2")


def test_prefill_stale_nan_past_context(cuda):
    q_lens, k_lens = [300, 140], [300, 1100]
    b = batch(q_lens, k_lens, seed=5)
    ref = ref_varlen(b)
    for i, L in enumerate(k_lens):
        last = int(b.block_tables[i, (L + 255) // 256 - 1])
        b.k_cache[last, L % 256 or 256:] = float("nan")
        b.v_cache[last, L % 256 or 256:] = float("nan")
    assert_attn_close(run_varlen(b), ref, "nan tail prefill")


def test_attention_module_prefill_and_decode(cuda):
    """nvattn.attention.Attention.forward reading the Context, as nano-vllm calls it: a prefill step (KV scattered
    then attention over the contiguous k/v), then a prefix-cache prefill step over the paged cache."""
    from nvattn.attention import Attention
    from nvattn.context import set_context, reset_context
    from nvattn.workloads import varlen_batch
    H, KVH = 32, 8
    attn = Attention(H, 128, 128 ** -0.5, KVH)
    # empty cache (warmup): no scatter, contiguous keys
    lens = [100, 37]
    b = varlen_batch(lens, lens, H, KVH, 128, 64, 0.5, 1, device="cuda", paged=False)
    set_context(True, b.cu_seqlens_q, b.cu_seqlens_k, b.max_seqlen_q, b.max_seqlen_k, b.slot_mapping)
    o = attn(b.q, b.k_new, b.v_new)
    reset_context()
    assert_attn_close(o, ref_varlen(b, paged=False), "module prefill")
    # with a cache: the step's K/V are scattered first, then the paged prefix is read
    q_lens, k_lens = [64, 200], [64 + 300, 200 + 20]
    b = varlen_batch(q_lens, k_lens, H, KVH, 128, 64, 0.5, 2, device="cuda")
    ref = ref_varlen(b)
    kc, vc = b.k_cache.clone(), b.v_cache.clone()
    kc.view(-1, KVH, 128)[b.slot_mapping.long()] = 0     # the step's rows are not there yet
    vc.view(-1, KVH, 128)[b.slot_mapping.long()] = 0
    attn.k_cache, attn.v_cache = kc, vc
    set_context(True, b.cu_seqlens_q, b.cu_seqlens_k, b.max_seqlen_q, b.max_seqlen_k, b.slot_mapping, None,
                b.block_tables)
    o = attn(b.q, b.k_new, b.v_new)
    reset_context()
    assert torch.equal(kc, b.k_cache) and torch.equal(vc, b.v_cache)
    assert_attn_close(o, ref, "module prefix prefill")


def test_attention_module_decode_graph(cuda):
    """The decode branch of Attention.forward captured in a CUDA graph (ModelRunner.capture_cudagraph) and replayed
    with new static inputs."""
    from nvattn.attention import Attention
    from nvattn.context import set_context, reset_context
    from nvattn.workloads import paged_decode_batch
    H, KVH, n = 32, 8, 3
    b = paged_decode_batch([500, 1200, 31], n, H, KVH, 128, 64, 0.5, 9, device="cuda")
    attn = Attention(H, 128, b.scale, KVH)
    attn.k_cache, attn.v_cache = b.k_cache, b.v_cache
    q, k, v = b.q.clone(), b.k_new.clone(), b.v_new.clone()
    set_context(False, slot_mapping=b.slot_mapping, context_lens=b.context_lens, block_tables=b.block_tables)
    eager = attn(q, k, v).clone()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        attn(q, k, v)
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = attn(q, k, v)
    reset_context()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    ref = oracle.paged_attention_ref(b.q.cpu().view(3, n, H, 128), b.k_cache.cpu(), b.v_cache.cpu(),
                                     b.context_lens.cpu(), b.block_tables.cpu(), b.scale)
    assert_attn_close(out.view(3, n, H, 128), ref, "graph decode")


def test_workspace_reserved_before_capture_and_never_grown_in_one(cuda):
    """nvattn.ops keeps one attention workspace per device.  A call that needs a bigger one while a CUDA graph is
    being captured raises instead of allocating inside the capture (which would give the graph a private
    allocation and record a zero-fill into every replay); after ops.reserve_workspace(max_num_seqs,
    max_num_batched_tokens, ...) -- what the nano-vllm drop-in does when the KV cache is allocated -- a larger call
    captures without allocating and replays equal to the eager call."""
    from nvattn import ops
    from nvattn.workloads import mixed_config
    saved = dict(ops._WORKSPACES)
    ops._WORKSPACES.clear()
    try:
        small = batch([1, 40], [100, 300], seed=13)
        run_varlen(small)                       # sizes a workspace for 2 sequences
        big = mixed_config(seed=0, device="cuda")   # 259 sequences: needs more
        out = torch.empty_like(big.q)

        def call():
            ops.flash_attn_varlen_func(big.q, big.k_cache, big.v_cache, max_seqlen_q=big.max_seqlen_q,
                                       cu_seqlens_q=big.cu_seqlens_q, max_seqlen_k=big.max_seqlen_k,
                                       cu_seqlens_k=big.cu_seqlens_k, softmax_scale=big.scale, causal=True,
                                       block_table=big.block_tables, out=out)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with pytest.raises(RuntimeError, match="reserve_workspace"):
            with torch.cuda.graph(g):
                call()
        del g
        ops.reserve_workspace(512, 16384, 32, 8)
        ws = ops._WORKSPACES[torch.cuda.current_device()]
        call()
        torch.cuda.synchronize()
        ref = out.clone()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        g2 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g2):
            call()
        out.fill_(float("nan"))
        g2.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        assert ops._WORKSPACES[torch.cuda.current_device()] is ws     # nothing was allocated or grown
        del g2
    finally:
        ops._WORKSPACES.clear()
        ops._WORKSPACES.update(saved)
