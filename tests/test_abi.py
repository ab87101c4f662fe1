"""The C-ABI library loads without a GPU, exports every entry point include/nvattn.h declares, and rejects
invalid arguments before touching the device (no compute calls here)."""
import ctypes
import os
import re

import pytest

from conftest import REPO

HEADER = os.path.join(REPO, "include", "nvattn.h")


def declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"NVA_API\s+[\w\s\*]+?\b(nva_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared()
    for n in ("nva_store_kvcache", "nva_paged_decode", "nva_varlen_attention", "nva_greedy_accept"):
        assert n in names


def test_library_exports_every_declared_symbol():
    from nvattn import _lib
    lib = _lib.load()
    for name in declared():
        assert hasattr(lib, name), name
    assert set(declared()) <= set(_lib.SIGNATURES)


def test_status_strings():
    from nvattn import _lib
    lib = _lib.load()
    assert lib.nva_status_string(0) == b"ok"
    assert b"workspace" in lib.nva_status_string(4)
    assert lib.nva_version() >= 1


def test_invalid_arguments_rejected_on_host():
    from nvattn import _lib
    lib = _lib.load()
    # negative token count
    assert lib.nva_store_kvcache(0, 0, 0, 0, 0, 0, 0, 0, -1, 8, 128, 2, 0) == 1
    # 8-byte elements are not a KV dtype
    assert lib.nva_store_kvcache(0, 0, 0, 0, 0, 0, 0, 0, 1, 8, 128, 8, 0) == 2
    # zero tokens: nothing to do
    assert lib.nva_store_kvcache(0, 0, 0, 0, 0, 0, 0, 0, 0, 8, 128, 2, 0) == 0
    # head_dim 64 unsupported by the attention kernels
    assert lib.nva_paged_decode(0, 0, 0, 0, 1, 256, 0, 0, 1, 1, 1, 32, 8, 64, 1.0, 0, 0, 0, 0, 0) == 2
    # H not a multiple of KVH
    assert lib.nva_paged_decode(0, 0, 0, 0, 1, 256, 0, 0, 1, 1, 1, 30, 8, 128, 1.0, 0, 0, 0, 0, 0) == 1
    # block size not a multiple of 128
    assert lib.nva_paged_decode(16, 4096, 16, 16, 1, 100, 16, 16, 1, 1, 1, 32, 8, 128, 1.0, 16, 4096, 16, 1 << 30, 0) == 2
    # the softmax scale must be positive and finite (decode, varlen, no-workspace decode)
    for bad in (0.0, -0.088, float("nan"), float("inf")):
        assert lib.nva_paged_decode(16, 4096, 16, 16, 1, 256, 16, 16, 1, 1, 1, 32, 8, 128, bad, 16, 4096, 16,
                                    1 << 30, 0) == 1
        assert lib.nva_varlen_attention(16, 4096, 0, 0, 0, 0, 16, 16, 1, 256, 16, 16, 1, 1, 1, 1, 1, 16, 1, 32, 8,
                                        128, bad, 16, 4096, 16, 1 << 30, 0) == 1
        assert lib.nva_paged_decode_noalloc(16, 4096, 16, 16, 1, 256, 16, 16, 1, 1, 1, 32, 8, 128, bad, 16, 4096,
                                            0) == 1
    # 64 draft tokens x 4 heads does not fit the 48-row tile
    assert lib.nva_paged_decode(16, 4096, 16, 16, 1, 256, 16, 16, 1, 1, 16, 32, 8, 128, 1.0, 16, 4096, 16, 1 << 30, 0) == 2
    # greedy accept: bad id width, negative k
    assert lib.nva_greedy_accept(0, 0, 0, 0, 0, 1, 1, 2, 0, 0, 0) == 2
    assert lib.nva_greedy_accept(0, 0, 0, 0, 0, 1, -1, 4, 0, 0, 0) == 1


def test_ops_refuse_cpu_tensors():
    import torch
    from nvattn import ops
    q = torch.zeros(1, 1, 32, 128, dtype=torch.bfloat16)
    kc = torch.zeros(2, 256, 8, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.flash_attn_with_kvcache(q, kc, kc, torch.ones(1, dtype=torch.int32), torch.zeros(1, 1, dtype=torch.int32),
                                    0.1)
    with pytest.raises(ValueError, match="CUDA"):
        ops.store_kvcache(torch.zeros(1, 8, 128), torch.zeros(1, 8, 128), torch.zeros(1, 256, 8, 128),
                          torch.zeros(1, 256, 8, 128), torch.zeros(1, dtype=torch.int32))


def test_store_kvcache_keeps_reference_asserts():
    """Same asserts as attention.py:36-39 (checked before anything else)."""
    import torch
    from nvattn import ops
    k = torch.zeros(2, 8, 128)[:, :, :64]          # head stride != head_dim
    with pytest.raises(AssertionError):
        ops.store_kvcache(k, k, torch.zeros(1, 256, 8, 64), torch.zeros(1, 256, 8, 64), torch.zeros(2, dtype=torch.int32))
