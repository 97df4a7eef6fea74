"""Handle-owning front end over the C ABI: one CudaTokenSampler per device.

Mirrors the host class a Neuraval.Cuda caller would hold (CudaBuffer-style
ownership, Neuraval.Cuda/CudaBuffer.cs:5-82): the handle owns device scratch,
the caller owns every input and output buffer. Device-pointer methods take
torch CUDA tensors (torch is only the allocator and stream provider here);
host methods take numpy arrays.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import native
from .native import NcbSamplerParams, check, load, make_params


def _ptr(t):
    if t is None:
        return None
    if isinstance(t, np.ndarray):
        return t.ctypes.data_as(ctypes.c_void_p)
    return ctypes.c_void_p(t.data_ptr())


def _stream_ptr(stream):
    if stream is None:
        return None
    return ctypes.c_void_p(stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream))


class CudaTokenSampler:
    """Batched TokenSampler.SampleNext / LogitsProcessor on one GPU."""

    def __init__(self, device: int = 0, max_rows: int = 1, max_vocab: int = 32000,
                 max_history: int = 4096):
        self._lib = load()
        h = ctypes.c_void_p()
        check(self._lib.ncb_sampler_create(device, max_rows, max_vocab, max_history,
                                           ctypes.byref(h)), "ncb_sampler_create")
        self._h = h
        self.device = device
        self.max_rows, self.max_vocab, self.max_history = max_rows, max_vocab, max_history

    def close(self) -> None:
        if getattr(self, "_h", None) is not None and self._h.value:
            check(self._lib.ncb_sampler_destroy(self._h), "ncb_sampler_destroy")
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- sampling -------------------------------------------------------
    def sample_rows_device(self, logits, hist_ids, hist_offsets, uniforms,
                           params: NcbSamplerParams, tokens, flags=None, probs=None,
                           stream=None) -> None:
        """Asynchronous: all tensors on this sampler's device."""
        rows, vocab = int(logits.shape[0]), int(logits.shape[1])
        st = self._lib.ncb_sample_rows_device(
            self._h, _ptr(logits), rows, vocab, _ptr(hist_ids), _ptr(hist_offsets),
            _ptr(uniforms), ctypes.byref(params), _ptr(tokens), _ptr(flags), _ptr(probs),
            _stream_ptr(stream))
        check(st, "ncb_sample_rows_device")

    def sample_rows(self, logits: np.ndarray, hist_ids: np.ndarray, hist_offsets: np.ndarray,
                    uniforms: np.ndarray, params: NcbSamplerParams, want_probs: bool = False):
        """Host arrays in and out (copies, samples, synchronises)."""
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        rows, vocab = logits.shape
        hist = np.ascontiguousarray(hist_ids, dtype=np.int32)
        offs = np.ascontiguousarray(hist_offsets, dtype=np.int32)
        uni = np.ascontiguousarray(uniforms, dtype=np.float32)
        tokens = np.zeros(rows, dtype=np.int32)
        flags = np.zeros(rows, dtype=np.uint32)
        probs = np.zeros((rows, vocab), dtype=np.float32) if want_probs else None
        st = self._lib.ncb_sample_rows(self._h, _ptr(logits), rows, vocab,
                                       _ptr(hist) if hist.size else None, _ptr(offs), _ptr(uni),
                                       ctypes.byref(params), _ptr(tokens), _ptr(flags),
                                       _ptr(probs))
        check(st, "ncb_sample_rows")
        return tokens, flags, probs

    # ---- vocabulary shards (device tensors) -------------------------------
    @property
    def shard_record_bytes(self) -> int:
        return int(self._lib.ncb_vocab_shard_record_bytes())

    def shard_candidates_device(self, logits_shard, vocab: int, col_begin: int, hist_ids,
                                hist_offsets, params: NcbSamplerParams, records,
                                stream=None) -> None:
        """Records of columns [col_begin, col_begin + width) of every row;
        `logits_shard` is [rows, width] (row stride from the tensor)."""
        rows, width = int(logits_shard.shape[0]), int(logits_shard.shape[1])
        ld = int(logits_shard.stride(0)) if rows > 1 else width
        check(self._lib.ncb_vocab_shard_candidates_device(
            self._h, _ptr(logits_shard), rows, int(vocab), int(col_begin), int(col_begin) + width,
            ld, _ptr(hist_ids), _ptr(hist_offsets), ctypes.byref(params), _ptr(records),
            _stream_ptr(stream)), "ncb_vocab_shard_candidates_device")

    def shard_merge_device(self, records, shards: int, rows: int, vocab: int, uniforms,
                           params: NcbSamplerParams, tokens, flags=None, stream=None) -> None:
        """Tokens from the gathered records ([shards][rows], column order)."""
        check(self._lib.ncb_vocab_shard_merge_device(
            self._h, _ptr(records), int(shards), int(rows), int(vocab), _ptr(uniforms),
            ctypes.byref(params), _ptr(tokens), _ptr(flags), _stream_ptr(stream)),
            "ncb_vocab_shard_merge_device")

    # vocabulary shards exchanged through peer memory
    def peer_setup(self, shards: int, me: int) -> bytes:
        """Allocates this GPU's exchange area; returns its IPC handle."""
        n = int(self._lib.ncb_peer_handle_bytes())
        buf = ctypes.create_string_buffer(n)
        check(self._lib.ncb_vocab_shard_peer_setup(self._h, int(shards), int(me), buf),
              "ncb_vocab_shard_peer_setup")
        return buf.raw

    def peer_connect(self, handles: bytes) -> None:
        """`handles`: every shard's handle, concatenated in shard order."""
        buf = ctypes.create_string_buffer(handles, len(handles))
        check(self._lib.ncb_vocab_shard_peer_connect(self._h, buf), "ncb_vocab_shard_peer_connect")

    def shard_push_peer_device(self, logits_shard, vocab: int, col_begin: int, hist_ids,
                               hist_offsets, params: NcbSamplerParams, stream=None) -> None:
        rows, width = int(logits_shard.shape[0]), int(logits_shard.shape[1])
        ld = int(logits_shard.stride(0)) if rows > 1 else width
        check(self._lib.ncb_vocab_shard_push_peer_device(
            self._h, _ptr(logits_shard), rows, int(vocab), int(col_begin), int(col_begin) + width,
            ld, _ptr(hist_ids), _ptr(hist_offsets), ctypes.byref(params), _stream_ptr(stream)),
            "ncb_vocab_shard_push_peer_device")

    def shard_merge_peer_device(self, rows: int, vocab: int, uniforms, params: NcbSamplerParams,
                                tokens, flags=None, stream=None) -> None:
        check(self._lib.ncb_vocab_shard_merge_peer_device(
            self._h, int(rows), int(vocab), _ptr(uniforms), ctypes.byref(params), _ptr(tokens),
            _ptr(flags), _stream_ptr(stream)), "ncb_vocab_shard_merge_peer_device")

    # rows split over GPUs, gathered through peer memory
    def row_gather_setup(self, ranks: int, me: int, rows_total: int) -> bytes:
        """Allocates this GPU's gather area; returns its IPC handle."""
        n = int(self._lib.ncb_peer_handle_bytes())
        buf = ctypes.create_string_buffer(n)
        check(self._lib.ncb_row_gather_setup(self._h, int(ranks), int(me), int(rows_total), buf),
              "ncb_row_gather_setup")
        self._rg_rows_total = int(rows_total)
        return buf.raw

    def row_gather_connect(self, handles: bytes) -> None:
        """`handles`: every rank's handle, concatenated in rank order."""
        buf = ctypes.create_string_buffer(handles, len(handles))
        check(self._lib.ncb_row_gather_connect(self._h, buf), "ncb_row_gather_connect")

    def sample_rows_gather_device(self, logits, row_begin: int, hist_ids, hist_offsets, uniforms,
                                  params: NcbSamplerParams, tokens_all, flags_all=None,
                                  stream=None) -> None:
        """This GPU's rows [row_begin, row_begin + rows); every row's token and
        flags into tokens_all / flags_all (rows_total each)."""
        rows, vocab = int(logits.shape[0]), int(logits.shape[1])
        total = getattr(self, "_rg_rows_total", 0)
        for name, t in (("tokens_all", tokens_all), ("flags_all", flags_all)):
            if t is not None and (t.numel() < total or t.element_size() != 4
                                  or not t.is_contiguous()):
                raise ValueError(f"{name} must be {total} contiguous 32-bit words")
        check(self._lib.ncb_sample_rows_gather_device(
            self._h, _ptr(logits), rows, vocab, int(row_begin), _ptr(hist_ids),
            _ptr(hist_offsets), _ptr(uniforms), ctypes.byref(params), _ptr(tokens_all),
            _ptr(flags_all), _stream_ptr(stream)), "ncb_sample_rows_gather_device")

    # ---- LogitsProcessor (in place, device tensors) ----------------------
    def repetition_penalty_(self, logits, hist_ids, hist_offsets, penalty, stream=None):
        check(self._lib.ncb_logits_repetition_penalty_device(
            self._h, _ptr(logits), int(logits.shape[0]), int(logits.shape[1]), _ptr(hist_ids),
            _ptr(hist_offsets), ctypes.c_float(penalty), _stream_ptr(stream)),
            "repetition_penalty")

    def frequency_presence_penalty_(self, logits, hist_ids, hist_offsets, frequency, presence,
                                    stream=None):
        check(self._lib.ncb_logits_frequency_presence_penalty_device(
            self._h, _ptr(logits), int(logits.shape[0]), int(logits.shape[1]), _ptr(hist_ids),
            _ptr(hist_offsets), ctypes.c_float(frequency), ctypes.c_float(presence),
            _stream_ptr(stream)), "frequency_presence_penalty")

    def temperature_(self, logits, temperature, stream=None):
        check(self._lib.ncb_logits_temperature_device(
            self._h, _ptr(logits), int(logits.shape[0]), int(logits.shape[1]),
            ctypes.c_float(temperature), _stream_ptr(stream)), "temperature")

    def filter_top_k_(self, logits, top_k, stream=None):
        check(self._lib.ncb_logits_filter_top_k_device(
            self._h, _ptr(logits), int(logits.shape[0]), int(logits.shape[1]), int(top_k),
            _stream_ptr(stream)), "filter_top_k")

    def filter_top_p_(self, probs, top_p, flags=None, stream=None):
        check(self._lib.ncb_logits_filter_top_p_device(
            self._h, _ptr(probs), int(probs.shape[0]), int(probs.shape[1]),
            ctypes.c_float(top_p), _ptr(flags), _stream_ptr(stream)), "filter_top_p")

    def full_sort_rows(self) -> int:
        """Rows this handle redid on the exact full-sort kernel (synchronises)."""
        n = ctypes.c_uint64(0)
        check(self._lib.ncb_sampler_full_sort_rows(self._h, ctypes.byref(n)), "full_sort_rows")
        return int(n.value)


def fast_exp_max_steps(x_lo: float, x_hi: float) -> int:
    """Largest float-step distance between the bucketed kernel's fast exp
    estimate and the correctly rounded exp over every float in [x_lo, x_hi]."""
    out = ctypes.c_uint32(0)
    check(native.load().ncb_fast_exp_max_steps(ctypes.c_float(x_lo), ctypes.c_float(x_hi),
                                               ctypes.byref(out)), "fast_exp_max_steps")
    return int(out.value)


__all__ = ["CudaTokenSampler", "NcbSamplerParams", "make_params", "native", "fast_exp_max_steps"]
