"""ctypes loader for oracle/oracle.c (test infrastructure only, see oracle/__init__.py)."""
import ctypes
import os
import subprocess

import numpy as np
import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None


def build_c(force: bool = False) -> str:
    """Compile oracle.c with gcc into oracle/_build/liboracle.so (skipped when up to date)."""
    src = os.path.join(_HERE, "oracle.c")
    if force or not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(src):
        os.makedirs(os.path.dirname(_SO), exist_ok=True)
        subprocess.check_call(["gcc", "-O2", "-shared", "-fPIC", "-o", _SO, src])
    return _SO


def _load():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build_c())
        _lib.oracle_store_kvcache.restype = ctypes.c_int
        _lib.oracle_store_kvcache.argtypes = [
            ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_int64, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]
        _lib.oracle_greedy_accept.restype = None
        _lib.oracle_greedy_accept.argtypes = [
            ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int32,
            ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]
    return _lib


def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  slot_mapping: torch.Tensor) -> int:
    """In-place C scatter on CPU tensors (attention.py:33-40 contract). Returns the number of out-of-range
    slots skipped."""
    N, KVH, D = key.shape
    assert key.stride(-1) == 1 and value.stride(-1) == 1
    assert key.stride(1) == D and value.stride(1) == D
    assert k_cache.is_contiguous() and v_cache.is_contiguous()
    slots = slot_mapping.to(torch.int32).contiguous()
    num_slots = k_cache.numel() // (KVH * D)
    return _load().oracle_store_kvcache(
        key.data_ptr(), key.stride(0), value.data_ptr(), value.stride(0), k_cache.data_ptr(), v_cache.data_ptr(),
        num_slots, slots.data_ptr(), N, KVH * D, key.element_size())


def greedy_accept(target: np.ndarray, drafts: np.ndarray, num_drafts: np.ndarray):
    """C greedy accept length on int64 arrays: target [S, K+1], drafts [S, K], num_drafts [S]."""
    target = np.ascontiguousarray(target, dtype=np.int64)
    S = target.shape[0]
    K = target.shape[1] - 1
    drafts = np.ascontiguousarray(drafts, dtype=np.int64).reshape(S, K)
    num_drafts = np.ascontiguousarray(num_drafts, dtype=np.int64)
    acc = np.zeros(S, np.int64)
    nxt = np.zeros(S, np.int64)
    _load().oracle_greedy_accept(target.ctypes.data, K + 1, drafts.ctypes.data, K,
                                 num_drafts.ctypes.data, S, K, acc.ctypes.data, nxt.ctypes.data)
    return acc, nxt
