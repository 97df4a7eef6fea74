"""ctypes front end of the C oracle (oracle/sampler_oracle.c).

TEST INFRASTRUCTURE ONLY: the oracle the CUDA kernels are tested against and the timed CPU
stand-in for the reference's C# TokenSampler. The product package never
imports this module.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libsampler_oracle.so")

EXP_GLIBC = 0
EXP_CR = 1

FLAG_DRAW_BOUNDARY = 0x1
FLAG_CUTOFF_BOUNDARY = 0x2
FLAG_TIE_AT_DRAW = 0x4
FLAG_NONFINITE = 0x8
FLAG_EXP_SLOW = 0x10


class OracleParams(ctypes.Structure):
    _fields_ = [
        ("greedy", ctypes.c_int32),
        ("temperature", ctypes.c_float),
        ("top_p", ctypes.c_float),
        ("top_k", ctypes.c_int32),
        ("repetition_penalty", ctypes.c_float),
        ("frequency_penalty", ctypes.c_float),
        ("presence_penalty", ctypes.c_float),
    ]


def build() -> str:
    """Compile the oracle shared library with its Makefile (strict fp32 flags)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        fp = ctypes.POINTER(ctypes.c_float)
        ip = ctypes.POINTER(ctypes.c_int32)
        lp = ctypes.POINTER(ctypes.c_int64)
        up = ctypes.POINTER(ctypes.c_uint32)
        L.oracle_expf_cr.argtypes = [ctypes.c_float, ctypes.POINTER(ctypes.c_int)]
        L.oracle_expf_cr.restype = ctypes.c_float
        L.oracle_expf_dd.argtypes = [ctypes.c_float]
        L.oracle_expf_dd.restype = ctypes.c_float
        L.oracle_sample_row.argtypes = [fp, ctypes.c_int32, ip, ctypes.c_int32,
                                        ctypes.POINTER(OracleParams), ctypes.c_float,
                                        ctypes.c_int, up, fp]
        L.oracle_sample_row.restype = ctypes.c_int32
        L.oracle_sample_rows.argtypes = [fp, ctypes.c_int32, ctypes.c_int32, ip, lp, fp,
                                         ctypes.POINTER(OracleParams), ctypes.c_int,
                                         ctypes.c_int, ip, up, fp]
        L.oracle_sample_rows.restype = ctypes.c_int
        L.oracle_apply_repetition_penalty.argtypes = [fp, ctypes.c_int32, ip, ctypes.c_int32,
                                                      ctypes.c_float]
        L.oracle_apply_frequency_presence_penalty.argtypes = [fp, ctypes.c_int32, ip,
                                                              ctypes.c_int32, ctypes.c_float,
                                                              ctypes.c_float]
        L.oracle_apply_temperature.argtypes = [fp, ctypes.c_int32, ctypes.c_float]
        L.oracle_filter_top_k.argtypes = [fp, ctypes.c_int32, ctypes.c_int32]
        L.oracle_filter_top_p.argtypes = [fp, ctypes.c_int32, ctypes.c_float, up]
        for f in ("oracle_apply_repetition_penalty", "oracle_apply_frequency_presence_penalty",
                  "oracle_apply_temperature", "oracle_filter_top_k", "oracle_filter_top_p"):
            getattr(L, f).restype = ctypes.c_int
        _lib = L
    return _lib


def _ptr(a, ct):
    return a.ctypes.data_as(ctypes.POINTER(ct)) if a is not None else None


def make_params(greedy=False, temperature=1.0, top_p=1.0, top_k=2**31 - 1,
                repetition_penalty=1.0, frequency_penalty=0.0, presence_penalty=0.0):
    return OracleParams(int(bool(greedy)), float(temperature), float(top_p), int(top_k),
                        float(repetition_penalty), float(frequency_penalty),
                        float(presence_penalty))


def expf_cr(x: float):
    slow = ctypes.c_int(0)
    r = lib().oracle_expf_cr(ctypes.c_float(x), ctypes.byref(slow))
    return r, bool(slow.value)


def expf_dd(x: float) -> float:
    return lib().oracle_expf_dd(ctypes.c_float(x))


def sample_row(logits, history, params: OracleParams, u=0.0, exp_mode=EXP_CR,
               want_probs=False):
    """TokenSampler.SampleNext on one row -> (token, flags, probs|None)."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    hist = np.ascontiguousarray(history, dtype=np.int32)
    flags = np.zeros(1, dtype=np.uint32)
    probs = np.zeros(logits.size, dtype=np.float32) if want_probs else None
    tok = lib().oracle_sample_row(_ptr(logits, ctypes.c_float), logits.size,
                                  _ptr(hist, ctypes.c_int32) if hist.size else None,
                                  hist.size, ctypes.byref(params), ctypes.c_float(u),
                                  exp_mode, _ptr(flags, ctypes.c_uint32),
                                  _ptr(probs, ctypes.c_float))
    return int(tok), int(flags[0]), probs


def sample_rows(logits, hist_ids, hist_offsets, uniforms, params: OracleParams,
                exp_mode=EXP_CR, threads=1, want_probs=False):
    """Batched oracle over [B,V] with CSR histories -> (tokens, flags, probs|None)."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    B, V = logits.shape
    hist = np.ascontiguousarray(hist_ids, dtype=np.int32)
    off = np.ascontiguousarray(hist_offsets, dtype=np.int64)
    uni = np.ascontiguousarray(uniforms, dtype=np.float32)
    tokens = np.zeros(B, dtype=np.int32)
    flags = np.zeros(B, dtype=np.uint32)
    probs = np.zeros((B, V), dtype=np.float32) if want_probs else None
    st = lib().oracle_sample_rows(_ptr(logits, ctypes.c_float), B, V,
                                  _ptr(hist, ctypes.c_int32) if hist.size else None,
                                  _ptr(off, ctypes.c_int64), _ptr(uni, ctypes.c_float),
                                  ctypes.byref(params), exp_mode, int(threads),
                                  _ptr(tokens, ctypes.c_int32), _ptr(flags, ctypes.c_uint32),
                                  _ptr(probs, ctypes.c_float))
    if st != 0:
        raise ValueError(f"oracle_sample_rows status {st}")
    return tokens, flags, probs


def apply_repetition_penalty(logits, history, penalty):
    a = np.array(logits, dtype=np.float32)
    h = np.ascontiguousarray(history, dtype=np.int32)
    st = lib().oracle_apply_repetition_penalty(_ptr(a, ctypes.c_float), a.size,
                                               _ptr(h, ctypes.c_int32) if h.size else None,
                                               h.size, ctypes.c_float(penalty))
    return st, a


def apply_frequency_presence_penalty(logits, history, frequency, presence):
    a = np.array(logits, dtype=np.float32)
    h = np.ascontiguousarray(history, dtype=np.int32)
    st = lib().oracle_apply_frequency_presence_penalty(
        _ptr(a, ctypes.c_float), a.size, _ptr(h, ctypes.c_int32) if h.size else None,
        h.size, ctypes.c_float(frequency), ctypes.c_float(presence))
    return st, a


def apply_temperature(logits, temperature):
    a = np.array(logits, dtype=np.float32)
    st = lib().oracle_apply_temperature(_ptr(a, ctypes.c_float), a.size,
                                        ctypes.c_float(temperature))
    return st, a


def filter_top_k(logits, top_k):
    a = np.array(logits, dtype=np.float32)
    st = lib().oracle_filter_top_k(_ptr(a, ctypes.c_float), a.size, int(top_k))
    return st, a


def filter_top_p(probs, top_p):
    a = np.array(probs, dtype=np.float32)
    tie = np.zeros(1, dtype=np.uint32)
    st = lib().oracle_filter_top_p(_ptr(a, ctypes.c_float), a.size, ctypes.c_float(top_p),
                                   _ptr(tie, ctypes.c_uint32))
    return st, a, int(tie[0])
