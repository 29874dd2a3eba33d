"""ctypes binding of libyanchor_b200.so (the C ABI of include/yanchor_b200.h).

The library is loaded from this package directory.  There is no fallback:
if the shared object is missing or fails to load, every operator raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, 'libyanchor_b200.so')

YB_F32, YB_F16, YB_BF16 = 0, 1, 2
YB_OK, YB_ERR_ARGUMENT, YB_ERR_UNSUPPORTED, YB_ERR_CUDA, YB_ERR_WORKSPACE = 0, 1, 2, 3, 4

GDN_QK_L2NORM = 1
GDN_GATE_IN_KERNEL = 2
GDN_BETA_SIGMOID = 4
GDN_TRANSPOSE_STATE = 8
GDN_STATE_F16 = 16
GDN_STATE_BF16 = 32

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float
_U32 = ctypes.c_uint32

# name -> (restype, argtypes); must match include/yanchor_b200.h
SIGNATURES = {
    'yb_last_error': (ctypes.c_char_p, []),
    'yb_abi_version': (_I, []),
    'yb_device_error': (_I, [_I]),
    'yb_gdn_recurrent_fwd': (_I, [_P, _P, _P, _I64, _I64, _I64, _P, _P, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _F,
                                  _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _F, _I, _I, _I, _U32, _P]),
    'yb_gdn_chunk_workspace_bytes': (_I64, [_I64, _I64, _I64, _I64, _I64, _I64, _I64, _I]),
    'yb_gdn_chunk_fwd': (_I, [_P, _P, _P, _I64, _I64, _I64, _P, _P, _I64, _I64, _P, _P, _P, _P, _P, _P, _I64, _I64,
                              _I64, _I64, _I64, _I64, _I64, _F, _I, _I, _I, _U32, _P, _I64, _P]),
    'yb_gdn_gates': (_I, [_P, _P, _I64, _I64, _P, _P, _P, _P, _I64, _I64, _I, _P]),
    'yb_mem_decode_read': (_I, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I, _P]),
    'yb_mem_decode_commit': (_I, [_P, _P, _P, _P, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64,
                                  _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I, _P]),
    'yb_mem_decode_step': (_I, [_P, _P, _P, _P, _P, _P, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64,
                                _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I, _P]),
    'yb_mem_indexed_read': (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I, _P]),
    'yb_mem_indexed_read_timeline': (_I, [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                                          _I64, _I64, _I64, _P, _P, _P, _I, _P]),
    'yb_gdn_decode_fused': (_I, [_P, _I64, _P, _I64, _P, _P, _I64, _P, _I64, _I64, _P, _P, _I64, _P, _I, _P, _P, _P,
                                 _F, _P, _I64, _I64, _I64, _I64, _I64, _I64, _F, _I, _U32, _P]),
    'yb_swa_ring_write': (_I, [_P, _P, _I64, _I64, _P, _P, _P, _I64, _I64, _P, _I64, _P, _I, _I64, _I64, _I64, _I64,
                               _I, _P]),
    'yb_swa_decode_workspace_bytes': (_I64, [_I64, _I64, _I64, _I64, _I64]),
    'yb_swa_decode_attention': (_I, [_P, _P, _P, _I64, _I64, _P, _I64, _P, _I64, _I64, _I64, _I64, _I64, _I, _P, _I64,
                                     _P]),
    'yb_conv1d_update': (_I, [_P, _I64, _P, _I64, _I64, _I64, _I64, _P, _P, _P, _I64, _I64, _I64, _I64, _I, _I,
                              _P]),
    'yb_conv1d_fwd': (_I, [_P, _I64, _I64, _P, _P, _I64, _I64, _I64, _I64, _P, _P, _P, _I64, _I64, _I64, _I64, _I64,
                           _I64, _I,
                           _I, _P]),
    'yb_mem_select_topk': (_I, [_P, _P, _I, _P, _I64, _I64, _I64, _P, _P, _P, _P]),
    'yb_mem_exclusive_prefix_topk': (_I, [_P, _P, _I, _P, _I64, _I64, _I64, _I64, _I64, _P, _P, _I, _P, _P, _P, _P,
                                          _P]),
    'yb_mem_prefill_timeline': (_I, [_P, _P, _P, _P, _P, _I64, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64,
                                     _P, _P, _P, _P, _P, _P]),
    'yb_mem_prefill_table': (_I, [_P, _P, _I64, _I64, _I64, _I64, _I64, _I, _I, _P, _P, _P, _P]),
    'yb_mem_prefill_read_references': (_I, [_P, _P, _I64, _I64, _I64, _I64, _I64, _I, _P, _P]),
    'yb_mem_prefill_state': (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _P, _P, _I64, _P, _P, _I64,
                                  _P, _I64, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I, _P]),
    'yb_sample_workspace_bytes': (_I64, [_I64, _I64, _I64]),
    'yb_sample_greedy': (_I, [_P, _I64, _I64, _I64, _I, _P, _P, _I64, _P]),
    'yb_sample_greedy_noalloc': (_I, [_P, _I64, _I64, _I64, _I, _P, _P]),
    'yb_sample_top_k_top_p_counter': (_I, [_P, _I64, _I64, _I64, _I, _P, _P, _I64, _I64, _I64, _F, _I64, _F, _P, _P,
                                           _I64, _P]),
    'yb_presence_penalty': (_I, [_P, _P, _I64, _F, _I, _P]),
    'yb_swa_prefill_attention': (_I, [_P, _P, _P, _P, _I64, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I,
                                      _P]),
    'yb_decode_state_update': (_I, [_P, _I64, _P, _I, _I64, _I64, _I64, _P, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _P,
                                    _P, _I64, _P, _I64, _I64, _I64, _P, _I, _P]),
}

_lock = threading.Lock()
_lib = None


class YanchorError(RuntimeError):
    """A kernel entry point returned an error status."""


def lib():
    """The loaded library (loaded once).  Raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(f'{LIB_PATH} is missing: build it with `python -m yanchor_b200.build`')
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(rc: int, op: str) -> None:
    if rc == YB_OK:
        return
    msg = lib().yb_last_error().decode(errors='replace')
    if rc == YB_ERR_ARGUMENT:
        raise ValueError(f'{op}: {msg}')
    if rc == YB_ERR_UNSUPPORTED:
        raise NotImplementedError(f'{op}: {msg}')
    raise YanchorError(f'{op}: {msg} (status {rc})')
