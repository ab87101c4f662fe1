"""nva_paged_decode_noalloc: paged decode / verify for callers that cannot allocate device memory.

Such callers (an allocator hook or host callback where cudaMalloc would recurse or deadlock, a runtime that owns all
memory through a fixed arena, an embedder without device allocation) cannot pass the workspace nva_paged_decode
needs; this entry point keeps the split-KV partials in scratch compiled into the library instead.  The test calls it
through the C ABI and checks it against nva_paged_decode and against the FP32 oracle within the attention tolerance,
on two calls in a row.  The verify case includes a sequence shorter than its query run (3 keys, 5 query tokens):
its first two rows see no key and must come out zero, as the oracle (flash-attn's semantics) gives them.

The file name makes pytest collect it last, so a run that stops at the first failure has run every other test."""
import pytest
import torch

import oracle
from conftest import assert_attn_close

pytestmark = pytest.mark.gpu

NVA_ERR_WORKSPACE = 4


def _batch(lens, n, seed):
    from nvattn.workloads import paged_decode_batch
    return paged_decode_batch(lens, n, 32, 8, 128, 512, 0.5, seed, device="cuda")


def _noalloc(b, out):
    from nvattn import _lib
    B, n = b.num_seqs, b.q_per_seq
    NB, BS, KVH, D = b.k_cache.shape
    return _lib.load().nva_paged_decode_noalloc(
        b.q.data_ptr(), 32 * 128, b.k_cache.data_ptr(), b.v_cache.data_ptr(), NB, BS, b.context_lens.data_ptr(),
        b.block_tables.data_ptr(), b.block_tables.stride(0), B, n, 32, KVH, D, b.scale, out.data_ptr(), 32 * 128,
        torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("lens,n", [([4096, 3000, 17, 900, 1], 1),      # long sequences: split across CTAs
                                    ([2048, 700, 129, 3], 5)])        # verify, 5 x 4 = 20 rows (32-row tile)
def test_noalloc_matches_workspace_entry_point(cuda, lens, n):
    from nvattn import ops, _lib
    _lib.clear_device_error()
    b = _batch(lens, n, seed=n)
    B = b.num_seqs
    ref = ops.flash_attn_with_kvcache(b.q.view(B, n, 32, 128), b.k_cache, b.v_cache, cache_seqlens=b.context_lens,
                                      block_table=b.block_tables, softmax_scale=b.scale)
    fp32 = oracle.paged_attention_ref(b.q.view(B, n, 32, 128).cpu(), b.k_cache.cpu(), b.v_cache.cpu(),
                                      b.context_lens.cpu(), b.block_tables.cpu(), b.scale)
    for call in range(2):   # the second call reuses the scratch the first one left behind
        out = torch.full((B * n, 32, 128), float("nan"), dtype=torch.bfloat16, device=cuda)
        assert _noalloc(b, out) == 0, f"call {call}"
        torch.cuda.synchronize()
        assert_attn_close(out.view(B, n, 32, 128), ref, f"no-alloc call {call}")
        assert_attn_close(out.view(B, n, 32, 128), fp32, f"no-alloc call {call} vs the oracle")
    assert _lib.device_error() == 0


def test_noalloc_rejects_calls_beyond_its_scratch(cuda):
    """9 query tokens x 4 q heads = 36 rows -> the 48-row tile needs more than the static scratch holds."""
    b = _batch([300, 600], 9, seed=3)
    out = torch.zeros(b.q.shape, dtype=torch.bfloat16, device=cuda)
    assert _noalloc(b, out) == NVA_ERR_WORKSPACE
    torch.cuda.synchronize()
    assert out.abs().sum() == 0    # nothing was launched
