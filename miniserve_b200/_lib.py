"""ctypes binding of libmssample.so (the C ABI in include/mssample.h).

There is no fallback: if the library is missing or no CUDA device is
present, every sampling call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmssample.so")

MS_OK = 0
MS_E_TOO_LARGE = -5
MS_DTYPE_F32 = 0
MS_DTYPE_BF16 = 1
MS_ROW_OK = 0
MS_ROW_ALL_MASKED = 1
MS_ROW_BAD_TEMPERATURE = 2
MS_ROW_NONFINITE = 4
MS_ROW_UNSUPPORTED = 8
MS_ROW_PEER_TIMEOUT = 16

_lock = threading.Lock()
_lib = None

_P = ctypes.c_void_p
_I64 = ctypes.c_int64

# name -> (restype, argtypes); every function include/mssample.h declares
SIGNATURES = {
    "ms_sample": (ctypes.c_int, [_P, ctypes.c_int, _I64, _I64, _I64, _P, _P, _P, _P, _P, _I64,
                                 _P, _P, _P, _P]),
    "ms_sample_generic": (ctypes.c_int, [_P, ctypes.c_int, _I64, _I64, _I64, _P, _P, _P, _P, _P,
                                         _I64, _P, _P, _P, _P]),
    "ms_shard_candidates": (ctypes.c_int, [_P, ctypes.c_int, _I64, _I64, _I64, _I64, _I64, _P, _P, _P,
                                           _I64, ctypes.c_int32, _P, _P]),
    "ms_nucleus_hist_words": (_I64, []),
    "ms_nucleus_record_words": (_I64, []),
    "ms_nucleus_cut_words": (_I64, []),
    "ms_nucleus_segments": (_I64, []),
    "ms_nucleus_hist": (ctypes.c_int, [_P, ctypes.c_int, _I64, _I64, _P, _I64, _P, _I64, _I64, _I64, _P,
                                       ctypes.c_int32, ctypes.c_int32, _P, _P, _P, _P]),
    "ms_nucleus_bracket": (ctypes.c_int, [_P, _P, _I64, _I64, _P, _P, _P]),
    "ms_nucleus_classify": (ctypes.c_int, [_P, ctypes.c_int, _I64, _I64, _I64, _P, _I64, _P, _I64, _I64, _P,
                                           ctypes.c_int32, ctypes.c_int32, _P, _P, _P, _P, _P]),
    "ms_nucleus_cut": (ctypes.c_int, [_P, ctypes.c_int32, _P, _P, _P, _I64, _I64, _P, ctypes.c_int32, _P, _P, _P,
                                      _P, _P]),
    "ms_nucleus_draw": (ctypes.c_int, [_P, ctypes.c_int, _I64, _I64, _I64, _P, _I64, _P, _I64, _I64, _P,
                                       ctypes.c_int32, ctypes.c_int32, _P, _P, _P, _P, ctypes.c_int32, _P, _P]),
    "ms_build_json_mask_noalloc": (ctypes.c_int, [_P, _I64, _P, _P, _I64, _P, _I64, _P, _P]),
    "ms_mask_from_logits": (ctypes.c_int, [_P, ctypes.c_int, _I64, _I64, _I64, _P, _I64, _P]),
    "ms_shard_record_words": (_I64, [ctypes.c_int32]),
    "ms_shard_merge": (ctypes.c_int, [_P, ctypes.c_int32, _I64, ctypes.c_int32, _I64, _P, _P, _P, _P,
                                      _P, _P, _P, _P]),
    "ms_exchange_words": (_I64, [_I64, ctypes.c_int32, ctypes.c_int32]),
    "ms_exchange_records_offset": (_I64, [_I64, ctypes.c_int32, ctypes.c_int32, ctypes.c_uint32]),
    "ms_shard_exchange": (ctypes.c_int, [_P, ctypes.c_int, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P,
                                         _I64, ctypes.c_int32, _P, _P, ctypes.c_int32, ctypes.c_int32, _I64,
                                         ctypes.c_int32, ctypes.c_uint32, _P]),
    "ms_exchange_merge": (ctypes.c_int, [_P, _P, ctypes.c_int32, ctypes.c_int32, _I64, _I64, ctypes.c_int32,
                                         ctypes.c_int32, _I64, _P, _P, _P, _P, ctypes.c_uint32, _I64, _P, _P, _P,
                                         _P]),
    "ms_exchange_results": (ctypes.c_int, [_P, ctypes.c_int32, _I64, _I64, ctypes.c_int32, ctypes.c_uint32, _I64,
                                           _P, _P, _P, _P]),
    "ms_device_alloc": (ctypes.c_int, [_I64, ctypes.POINTER(ctypes.c_void_p)]),
    "ms_device_free": (ctypes.c_int, [_P]),
    "ms_ipc_handle": (ctypes.c_int, [_P, ctypes.c_char_p]),
    "ms_ipc_open": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
    "ms_ipc_close": (ctypes.c_int, [_P]),
    "ms_json_state_words": (_I64, []),
    "ms_json_init": (ctypes.c_int, [_P, _P, _I64, _P, _P]),
    "ms_json_advance": (ctypes.c_int, [_P, _I64, _P, _P, _I64, _P, _P]),
    "ms_build_json_mask": (ctypes.c_int, [_P, _I64, _P, _P, _I64, _P, _I64, _P, _P]),
    "ms_json_pack_vocab": (ctypes.c_int, [_P, _P, _I64, _P, _P, _P]),
    "ms_build_json_mask_packed": (ctypes.c_int, [_P, _I64, _P, _P, _P, _P, _I64, _P, _I64, _P, _P]),
    "ms_json_pack_vocab_ordered": (ctypes.c_int, [_P, _P, _I64, _P, _P, _P, _P]),
    "ms_build_json_mask_ordered": (ctypes.c_int, [_P, _I64, _P, _P, _P, _P, _P, _I64, _P, _I64, _P, _P]),
    "ms_error_string": (ctypes.c_char_p, [ctypes.c_int]),
    "ms_last_cuda_error": (ctypes.c_int, []),
    "ms_version": (ctypes.c_int, []),
}


class SamplerLibraryError(RuntimeError):
    pass


def lib():
    """Load libmssample.so once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise SamplerLibraryError(
                    f"{LIB_PATH} is missing: build it with `python -m miniserve_b200.build` "
                    "(there is no CPU fallback)")
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc != MS_OK:
        L = lib()
        msg = L.ms_error_string(rc).decode()
        if rc == -3:
            msg += f" (cudaError {L.ms_last_cuda_error()})"
        raise SamplerLibraryError(f"{what} failed: {msg}")
