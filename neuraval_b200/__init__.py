"""neuraval_b200: sm_100a decode-time logits processing and token sampling.

A from-scratch B200 implementation of Neuraval's TokenSampler / LogitsProcessor
path (Neuraval/Generation/TokenSampler.cs, LogitsProcessor.cs) behind a C ABI
(include/navsampler.h, libnavsampler.so).
"""
from .native import (FLAG_BAD_HISTORY, FLAG_CUTOFF_BOUNDARY, FLAG_DRAW_BOUNDARY, FLAG_EXP_SLOW,
                     FLAG_NONFINITE, FLAG_TIE_AT_DRAW, INT_MAX, PARITY_EXEMPT, NcbError,
                     NcbSamplerParams, make_params)

__all__ = ["NcbError", "NcbSamplerParams", "make_params", "INT_MAX", "PARITY_EXEMPT",
           "FLAG_DRAW_BOUNDARY", "FLAG_CUTOFF_BOUNDARY", "FLAG_TIE_AT_DRAW", "FLAG_NONFINITE",
           "FLAG_EXP_SLOW", "FLAG_BAD_HISTORY"]
