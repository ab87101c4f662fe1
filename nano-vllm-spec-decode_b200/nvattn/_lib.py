"""ctypes binding of libnvattn.so (the C ABI in include/nvattn.h).

The library is built in-tree by nano-vllm-spec-decode_b200/build.py.  There is no fallback: if the library is
missing or fails to load, importing any op raises, so a GPU run can never silently take another path.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libnvattn.so")

# (name, restype, argtypes) for every entry point of include/nvattn.h
_P, _I32, _I64, _F, _SZ = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
SIGNATURES = {
    "nva_version": (ctypes.c_int, []),
    "nva_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "nva_last_cuda_error": (ctypes.c_char_p, []),
    "nva_store_kvcache": (ctypes.c_int, [_P, _I64, _P, _I64, _P, _P, _I64, _P, _I32, _I32, _I32, _I32, _P]),
    "nva_paged_decode": (ctypes.c_int, [_P, _I64, _P, _P, _I32, _I32, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32,
                                        _F, _P, _I64, _P, _SZ, _P]),
    "nva_paged_decode_workspace_bytes": (ctypes.c_size_t, [_I32, _I32, _I32, _I32, _I32]),
    "nva_varlen_attention": (ctypes.c_int, [_P, _I64, _P, _I64, _P, _I64, _P, _P, _I32, _I32, _P, _P, _I32, _I32,
                                            _I32, _I32, _I32, _P, _I32, _I32, _I32, _I32, _F, _P, _I64, _P, _SZ,
                                            _P]),
    "nva_varlen_workspace_bytes": (ctypes.c_size_t, [_I32, _I32, _I32, _I32, _I32]),
    "nva_greedy_accept": (ctypes.c_int, [_P, _I64, _P, _I64, _P, _I32, _I32, _I32, _P, _P, _P]),
    "nva_qk_norm_rope_store": (ctypes.c_int, [_P, _I64, _I32, _I32, _I32, _I32, _P, _P, _I32, _P, _P, _F, _P, _I64,
                                              _P, _I64, _P, _P, _I64, _P, _P]),
    "nva_shard_argmax": (ctypes.c_int, [_P, _I64, _I32, _I32, _I64, _I32, _P, _P]),
    "nva_shard_accept": (ctypes.c_int, [_P, _I32, _I32, _I32, _P, _I64, _P, _I32, _P, _P, _P]),
    "nva_paged_decode_noalloc": (ctypes.c_int, [_P, _I64, _P, _P, _I32, _I32, _P, _P, _I32, _I32, _I32, _I32, _I32,
                                                _I32, _F, _P, _I64, _P]),
    "nva_get_device_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32)]),
    "nva_clear_device_error": (ctypes.c_int, []),
}

_lib = None


class NvattnError(RuntimeError):
    """A libnvattn entry point returned a non-zero nva_status."""


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"libnvattn.so not built ({LIB_PATH}); run nano-vllm-spec-decode_b200/build.py")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        lib = load()
        msg = lib.nva_status_string(status).decode()
        cuda = lib.nva_last_cuda_error().decode()
        raise NvattnError(f"{what}: {msg}" + (f" ({cuda})" if status == 5 and cuda else ""))


def device_error() -> int:
    """Bits of the device error word (synchronises the device)."""
    v = ctypes.c_uint32(0)
    check(load().nva_get_device_error(ctypes.byref(v)), "nva_get_device_error")
    return v.value


def clear_device_error() -> None:
    check(load().nva_clear_device_error(), "nva_clear_device_error")
