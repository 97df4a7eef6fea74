"""A second, independent restatement of the reference sampler in plain Python
(numpy float32 scalars, one operation at a time), used only to cross-check the C
oracle on small rows. Follows Neuraval/Generation/TokenSampler.cs:32-143 and
LogitsProcessor.cs:8-114 literally, including the min-heap of capacity K.
"""
from __future__ import annotations

import ctypes
import heapq

import numpy as np

f32 = np.float32
_libm = ctypes.CDLL("libm.so.6")
_libm.expf.argtypes = [ctypes.c_float]
_libm.expf.restype = ctypes.c_float


def expf(x):
    return f32(_libm.expf(float(x)))


def _adjust(v, tid, repeated, penalty, counts, freq, pres):
    v = f32(v)
    if repeated is not None and tid in repeated:
        v = f32(v / f32(penalty)) if v > f32(0) else f32(v * f32(penalty))
    c = counts.get(tid, 0) if counts is not None else 0
    if c > 0:
        v = f32(v - f32(f32(c) * f32(freq)))
        v = f32(v - f32(pres))
    return v


def sample_next(logits, history, p, u, exp=expf):
    logits = [f32(x) for x in logits]
    V = len(logits)
    pen = f32(p.get("repetition_penalty", 1.0))
    freq = f32(p.get("frequency_penalty", 0.0))
    pres = f32(p.get("presence_penalty", 0.0))
    repeated = set(history) if (pen != f32(1) and len(history) > 0) else None
    counts = None
    if (freq != 0 or pres != 0) and len(history) > 0:
        counts = {}
        for t in history:
            counts[t] = counts.get(t, 0) + 1
    if p.get("greedy", False):
        best, bestv = 0, _adjust(logits[0], 0, repeated, pen, counts, freq, pres)
        for i in range(1, V):
            v = _adjust(logits[i], i, repeated, pen, counts, freq, pres)
            if v > bestv:
                best, bestv = i, v
        return best
    K = min(int(p.get("top_k", 2**31 - 1)), V)
    scale = f32(f32(1.0) / f32(p["temperature"]))
    heap = []
    for i in range(V):
        v = f32(_adjust(logits[i], i, repeated, pen, counts, freq, pres) * scale)
        if len(heap) < K:
            heapq.heappush(heap, v)
        elif v > heap[0]:
            heapq.heapreplace(heap, v)
    thr = heap[0]
    cands = []
    for i in range(V):
        v = f32(_adjust(logits[i], i, repeated, pen, counts, freq, pres) * scale)
        if v >= thr:
            cands.append((i, f32(v + f32(0.0))))
    # descending by value; equal values keep ascending id (stable sort)
    cands.sort(key=lambda c: -float(c[1]))
    mx = cands[0][1]
    w = [exp(f32(c[1] - mx)) for c in cands]
    total = f32(0)
    for x in w:
        total = f32(total + x)
    cutoff = len(cands)
    top_p = f32(p.get("top_p", 1.0))
    if top_p < f32(1):
        target = f32(total * top_p)
        cum = f32(0)
        for i, x in enumerate(w):
            cum = f32(cum + x)
            if cum >= target:
                cutoff = i + 1
                break
    retained = f32(0)
    for i in range(cutoff):
        retained = f32(retained + w[i])
    sample = f32(f32(u) * retained)
    cum = f32(0)
    for i in range(cutoff):
        cum = f32(cum + w[i])
        if sample <= cum or i == cutoff - 1:
            return cands[i][0]
    return cands[-1][0]
