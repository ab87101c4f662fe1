"""Host logic of the torch-facing wrappers (nvattn/ops.py) without a GPU: the arguments each wrapper hands to
the C ABI (row strides, null pointers for the absent operands, the workspace size the library's size query
returned) and the layout checks on caller-provided outputs, which must fail before any entry point is called.

The library is replaced by a recorder: every compute entry point only records its arguments and returns NVA_OK.
The real size queries scale with the device's SM count, so the recorder answers them itself: 0 (unsupported)
above 48 packed query rows per kv head, as the decode tile does, else a fixed size."""
import pytest
import torch


WS_BYTES = 1 << 20


class _Recorder:
    def __init__(self):
        self.calls = []

    @staticmethod
    def nva_paged_decode_workspace_bytes(B, n, H, KVH, D):
        return 0 if n * (H // KVH) > 48 else WS_BYTES

    @staticmethod
    def nva_varlen_workspace_bytes(B, Tq, H, KVH, D):
        return WS_BYTES

    def __getattr__(self, name):
        def call(*args):
            self.calls.append((name, args))
            return 0
        return call


@pytest.fixture()
def rec(monkeypatch):
    from nvattn import _lib, ops
    r = _Recorder()
    monkeypatch.setattr(_lib, "load", lambda: r)
    monkeypatch.setattr(ops, "_need_cuda", lambda *ts: None)
    monkeypatch.setattr(ops, "_stream", lambda: 0)
    monkeypatch.setattr(ops, "_workspace", lambda nbytes, device: torch.zeros(max(nbytes, 16), dtype=torch.uint8))
    return r


def _decode_inputs(B=3, n=2, H=32, KVH=8, D=128, NB=4, BS=256):
    q = torch.zeros(B, n, H, D, dtype=torch.bfloat16)
    kc = torch.zeros(NB, BS, KVH, D, dtype=torch.bfloat16)
    lens = torch.ones(B, dtype=torch.int32)
    bt = torch.zeros(B, 2, dtype=torch.int32)
    return q, kc, lens, bt


# nva_paged_decode argument positions (include/nvattn.h)
_DQ_STRIDE, _DB, _DN, _DH, _DKVH, _DD, _DOUT, _DOUT_STRIDE, _DWS_BYTES = 1, 9, 10, 11, 12, 13, 15, 16, 18


def test_decode_marshals_strides_and_workspace(rec):
    from nvattn import ops
    q, kc, lens, bt = _decode_inputs()
    out = ops.flash_attn_with_kvcache(q, kc, kc, cache_seqlens=lens, block_table=bt, softmax_scale=0.1)
    (name, a), = rec.calls
    assert name == "nva_paged_decode"
    assert (a[_DB], a[_DN], a[_DH], a[_DKVH], a[_DD]) == (3, 2, 32, 8, 128)
    assert a[_DQ_STRIDE] == a[_DOUT_STRIDE] == 32 * 128
    assert a[_DOUT] == out.data_ptr() and out.shape == q.shape and out.dtype == torch.bfloat16
    assert a[_DWS_BYTES] == WS_BYTES


def test_decode_accepts_padded_output_rows(rec):
    from nvattn import ops
    q, kc, lens, bt = _decode_inputs()
    base = torch.zeros(3 * 2, 32 * 128 + 64, dtype=torch.bfloat16)
    out = base[:, :32 * 128].view(3, 2, 32, 128)
    got = ops.flash_attn_with_kvcache(q, kc, kc, cache_seqlens=lens, block_table=bt, softmax_scale=0.1, out=out)
    (_, a), = rec.calls
    assert got is out and a[_DOUT] == out.data_ptr() and a[_DOUT_STRIDE] == 32 * 128 + 64


@pytest.mark.parametrize("bad", ["dtype", "shape", "batch_stride", "head_stride"])
def test_decode_rejects_output_layouts_it_cannot_address(rec, bad):
    from nvattn import ops
    q, kc, lens, bt = _decode_inputs()
    out = {
        "dtype": lambda: torch.zeros(3, 2, 32, 128, dtype=torch.float16),
        "shape": lambda: torch.zeros(3, 1, 32, 128, dtype=torch.bfloat16),
        # the query rows of one sequence are not adjacent to the next sequence's
        "batch_stride": lambda: torch.zeros(3, 4, 32, 128, dtype=torch.bfloat16)[:, :2],
        # heads interleaved with another tensor
        "head_stride": lambda: torch.zeros(3, 2, 32, 256, dtype=torch.bfloat16)[..., :128],
    }[bad]()
    with pytest.raises(AssertionError):
        ops.flash_attn_with_kvcache(q, kc, kc, cache_seqlens=lens, block_table=bt, softmax_scale=0.1, out=out)
    assert rec.calls == []


def test_decode_unsupported_row_count_raises_before_launch(rec):
    from nvattn import _lib, ops
    q, kc, lens, bt = _decode_inputs(n=17)      # 17 query rows x 4 heads exceed the 48-row tile
    with pytest.raises(_lib.NvattnError):
        ops.flash_attn_with_kvcache(q, kc, kc, cache_seqlens=lens, block_table=bt, softmax_scale=0.1)
    assert rec.calls == []


# nva_varlen_attention argument positions (include/nvattn.h)
_VK, _VK_STRIDE, _VV, _VKC, _VVC, _VNB, _VBS, _VB, _VTQ, _VTK, _VBT, _VBT_STRIDE = 2, 3, 4, 6, 7, 8, 9, 12, 13, 14, 17, 18
_VOUT, _VOUT_STRIDE, _VWS_BYTES = 23, 24, 26


def test_varlen_paged_passes_cache_and_table_only(rec):
    from nvattn import ops
    q = torch.zeros(10, 32, 128, dtype=torch.bfloat16)
    kc = torch.zeros(4, 256, 8, 128, dtype=torch.bfloat16)
    cu = torch.tensor([0, 3, 10], dtype=torch.int32)
    bt = torch.zeros(2, 5, dtype=torch.int32)
    out = ops.flash_attn_varlen_func(q, kc, kc, 7, cu, 600, cu, 0.1, causal=True, block_table=bt)
    (name, a), = rec.calls
    assert name == "nva_varlen_attention"
    assert a[_VK] == a[_VK_STRIDE] == a[_VV] == a[_VTK] == 0
    assert (a[_VKC], a[_VVC]) == (kc.data_ptr(), kc.data_ptr())
    assert (a[_VNB], a[_VBS], a[_VB], a[_VTQ]) == (4, 256, 2, 10)
    assert (a[_VBT], a[_VBT_STRIDE]) == (bt.data_ptr(), 5)
    assert a[_VOUT] == out.data_ptr() and a[_VOUT_STRIDE] == 32 * 128
    assert a[_VWS_BYTES] == WS_BYTES


def test_varlen_contiguous_passes_row_strides_and_no_cache(rec):
    from nvattn import ops
    q = torch.zeros(10, 32, 128, dtype=torch.bfloat16)
    kv = torch.zeros(12, 2, 8, 128, dtype=torch.bfloat16)      # K and V interleaved per row: row stride 2 x 8 x 128
    k, v = kv[:, 0], kv[:, 1]
    cu_q = torch.tensor([0, 3, 10], dtype=torch.int32)
    cu_k = torch.tensor([0, 5, 12], dtype=torch.int32)
    ops.flash_attn_varlen_func(q, k, v, 7, cu_q, 7, cu_k, 0.1, causal=True)
    (_, a), = rec.calls
    assert (a[_VK], a[_VV]) == (k.data_ptr(), v.data_ptr()) and a[_VK_STRIDE] == 2 * 8 * 128
    assert a[_VKC] == a[_VVC] == a[_VNB] == a[_VBS] == a[_VBT] == a[_VBT_STRIDE] == 0
    assert a[_VTK] == 12


def test_varlen_rejects_mismatched_output(rec):
    from nvattn import ops
    q = torch.zeros(10, 32, 128, dtype=torch.bfloat16)
    k = torch.zeros(12, 8, 128, dtype=torch.bfloat16)
    cu = torch.tensor([0, 10], dtype=torch.int32)
    cu_k = torch.tensor([0, 12], dtype=torch.int32)
    for out in (torch.zeros(9, 32, 128, dtype=torch.bfloat16), torch.zeros(10, 32, 256, dtype=torch.bfloat16)[..., :128]):
        with pytest.raises(AssertionError):
            ops.flash_attn_varlen_func(q, k, k, 10, cu, 12, cu_k, 0.1, out=out)
    assert rec.calls == []


def test_store_kvcache_counts_slots(rec):
    from nvattn import ops
    key = torch.zeros(5, 8, 128, dtype=torch.bfloat16)
    kc = torch.zeros(3, 256, 8, 128, dtype=torch.bfloat16)
    slots = torch.arange(5, dtype=torch.int32)
    ops.store_kvcache(key, key, kc, kc, slots)
    (name, a), = rec.calls
    assert name == "nva_store_kvcache"
    assert a[6] == 3 * 256 and a[8:12] == (5, 8, 128, 2)


def test_greedy_accept_without_drafts_passes_null(rec):
    from nvattn import ops
    t = torch.zeros(4, 1, dtype=torch.int64)
    acc, nxt = ops.greedy_accept(t, torch.zeros(4, 0, dtype=torch.int64), torch.zeros(4, dtype=torch.int64))
    (name, a), = rec.calls
    assert name == "nva_greedy_accept" and a[2] == a[3] == 0 and a[6] == 0 and a[7] == 8
    assert acc.dtype == nxt.dtype == torch.int64 and acc.shape == nxt.shape == (4,)


def test_verify_drafts_greedy_hands_int64_argmax_ids_to_accept(rec):
    from nvattn.sampler import verify_drafts_greedy
    S, K, V = 3, 2, 11
    logits = torch.zeros(S * (K + 1), V, dtype=torch.bfloat16)
    acc, nxt = verify_drafts_greedy(logits, torch.zeros(S, K, dtype=torch.int32), torch.full((S,), K))
    (name, a), = rec.calls
    assert name == "nva_greedy_accept" and (a[5], a[6], a[7]) == (S, K, 8)
    assert acc.dtype == nxt.dtype == torch.int64 and acc.shape == (S,)
