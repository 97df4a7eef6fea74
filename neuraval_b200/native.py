"""ctypes binding of libnavsampler.so (the C ABI in include/navsampler.h).

This is the Python view of the drop-in boundary: the same entry points a C#
P/Invoke table (Neuraval.Cuda/Native/CudaNative.cs style) binds. There is no
CPU fallback: if the library is missing, loading it raises.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libnavsampler.so")

NCB_OK = 0
NCB_ERROR_NO_DEVICE = 1
NCB_ERROR_INIT_FAILED = 2
NCB_ERROR_ALLOC_FAILED = 3
NCB_ERROR_COPY_FAILED = 4
NCB_ERROR_LAUNCH_FAILED = 5
NCB_ERROR_NOT_INITIALIZED = 6
NCB_ERROR_INVALID_ARGUMENT = 7
NCB_ERROR_CAPACITY = 8

FLAG_DRAW_BOUNDARY = 0x1
FLAG_CUTOFF_BOUNDARY = 0x2
FLAG_TIE_AT_DRAW = 0x4
FLAG_NONFINITE = 0x8
FLAG_EXP_SLOW = 0x10
FLAG_BAD_HISTORY = 0x20
FLAG_TIES_OVERFLOW = 0x40
FLAG_PEER_TIMEOUT = 0x80
# rows whose token may legitimately differ from the reference's
PARITY_EXEMPT = FLAG_DRAW_BOUNDARY | FLAG_CUTOFF_BOUNDARY | FLAG_TIE_AT_DRAW

INT_MAX = 2**31 - 1


class NcbSamplerParams(ctypes.Structure):
    _fields_ = [
        ("greedy", ctypes.c_int32),
        ("temperature", ctypes.c_float),
        ("top_p", ctypes.c_float),
        ("top_k", ctypes.c_int32),
        ("repetition_penalty", ctypes.c_float),
        ("frequency_penalty", ctypes.c_float),
        ("presence_penalty", ctypes.c_float),
    ]


# name -> (restype, argtypes)
_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
SIGNATURES = {
    "ncb_sampler_params_validate": (_I, [ctypes.POINTER(NcbSamplerParams)]),
    "ncb_sampler_create": (_I, [_I, _I, _I, _I, ctypes.POINTER(_P)]),
    "ncb_sampler_destroy": (_I, [_P]),
    "ncb_sample_rows_device": (_I, [_P, _P, _I, _I, _P, _P, _P, ctypes.POINTER(NcbSamplerParams),
                                    _P, _P, _P, _P]),
    "ncb_sample_rows": (_I, [_P, _P, _I, _I, _P, _P, _P, ctypes.POINTER(NcbSamplerParams),
                             _P, _P, _P]),
    "ncb_sample_rows_noalloc_device": (_I, [_P, _I, _I, _P, _P, _P,
                                            ctypes.POINTER(NcbSamplerParams), _P, _P, _P, _P]),
    "ncb_vocab_shard_record_bytes": (_I, []),
    "ncb_vocab_shard_candidates_device": (_I, [_P, _P, _I, _I, _I, _I, _I, _P, _P,
                                               ctypes.POINTER(NcbSamplerParams), _P, _P]),
    "ncb_vocab_shard_merge_device": (_I, [_P, _P, _I, _I, _I, _P,
                                          ctypes.POINTER(NcbSamplerParams), _P, _P, _P]),
    "ncb_logits_repetition_penalty_device": (_I, [_P, _P, _I, _I, _P, _P, _F, _P]),
    "ncb_logits_frequency_presence_penalty_device": (_I, [_P, _P, _I, _I, _P, _P, _F, _F, _P]),
    "ncb_logits_temperature_device": (_I, [_P, _P, _I, _I, _F, _P]),
    "ncb_logits_filter_top_k_device": (_I, [_P, _P, _I, _I, _I, _P]),
    "ncb_logits_filter_top_p_device": (_I, [_P, _P, _I, _I, _F, _P, _P]),
    "ncb_peer_handle_bytes": (_I, []),
    "ncb_vocab_shard_peer_setup": (_I, [_P, _I, _I, _P]),
    "ncb_vocab_shard_peer_connect": (_I, [_P, _P]),
    "ncb_vocab_shard_push_peer_device": (_I, [_P, _P, _I, _I, _I, _I, _I, _P, _P,
                                              ctypes.POINTER(NcbSamplerParams), _P]),
    "ncb_vocab_shard_merge_peer_device": (_I, [_P, _I, _I, _P, ctypes.POINTER(NcbSamplerParams),
                                               _P, _P, _P]),
    "ncb_row_gather_setup": (_I, [_P, _I, _I, _I, _P]),
    "ncb_row_gather_connect": (_I, [_P, _P]),
    "ncb_sample_rows_gather_device": (_I, [_P, _P, _I, _I, _I, _P, _P, _P,
                                           ctypes.POINTER(NcbSamplerParams), _P, _P, _P]),
    "ncb_softmax_rows_device": (_I, [_P, _P, _I, _I, _P]),
    "ncb_logits_repetition_penalty": (_I, [_P, _P, _I, _I, _P, _P, _F]),
    "ncb_logits_frequency_presence_penalty": (_I, [_P, _P, _I, _I, _P, _P, _F, _F]),
    "ncb_logits_temperature": (_I, [_P, _P, _I, _I, _F]),
    "ncb_logits_filter_top_k": (_I, [_P, _P, _I, _I, _I]),
    "ncb_logits_filter_top_p": (_I, [_P, _P, _I, _I, _F, _P]),
    "ncb_sampler_full_sort_rows": (_I, [_P, ctypes.POINTER(ctypes.c_uint64)]),
    "ncb_fast_exp_max_steps": (_I, [_F, _F, ctypes.POINTER(ctypes.c_uint32)]),
    "ncb_sampler_last_status": (_I, []),
    "ncb_sampler_status_message": (ctypes.c_char_p, [_I]),
}

_lib = None


class NcbError(RuntimeError):
    """CudaException analogue (Neuraval.Cuda/CudaException.cs): status + message."""

    def __init__(self, status: int, where: str = ""):
        self.status = status
        msg = load().ncb_sampler_status_message(status).decode()
        super().__init__(f"{where}: status {status} ({msg})" if where else msg)


def load():
    """Load the in-tree library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} not built; run `python -m neuraval_b200.build`")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(status: int, where: str = "") -> None:
    if status != NCB_OK:
        raise NcbError(status, where)


def make_params(greedy=False, temperature=1.0, top_p=1.0, top_k=INT_MAX, repetition_penalty=1.0,
                frequency_penalty=0.0, presence_penalty=0.0) -> NcbSamplerParams:
    return NcbSamplerParams(int(bool(greedy)), float(temperature), float(top_p), int(top_k),
                            float(repetition_penalty), float(frequency_penalty),
                            float(presence_penalty))
