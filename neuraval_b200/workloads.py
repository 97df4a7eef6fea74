"""Seeded synthetic decode-time batches with the shapes and value distributions
of the five sampling workloads the library is measured on (no dataset involved).

Each generator returns a dict with
  logits  [B, V] float32,  hist_ids  int32 (CSR),  hist_offsets  int32 [B+1],
  uniforms  float32 [B] in [0, 1),  params  (keyword arguments of make_params).
"""
from __future__ import annotations

import numpy as np

INT_MAX = 2**31 - 1


def _uniform_history(rng, B, H, V):
    ids = rng.integers(0, V, size=(B, H), dtype=np.int64).astype(np.int32)
    return ids.reshape(-1), (np.arange(B + 1, dtype=np.int64) * H).astype(np.int32)


def _uniforms(rng, B):
    # (float)random.NextDouble(): a double in [0,1) rounded to float (may round to 1.0f
    # only for doubles within 2^-25 of 1; kept < 1 here)
    u = rng.random(B, dtype=np.float64).astype(np.float32)
    return np.minimum(u, np.float32(1.0) - np.float32(2**-24)).astype(np.float32)


def zipf_rank_offsets(V: int, span_nats: float, s: float = 1.0) -> np.ndarray:
    """Log-mass of a Zipf(s) law over ranks 0..V-1, scaled to span `span_nats`."""
    r = np.arange(V, dtype=np.float64)
    lo = -s * np.log1p(r)
    return (lo * (span_nats / (s * np.log(V)))).astype(np.float32)


def peaked_head(B=1, V=32000, H=64, seed=1, greedy=False):
    """Single-row latency case: N(0,3^2) with 8 ids raised by +8; 64-id history;
    repetition 1.1, T 0.8, top-k 40, top-p 0.9 (or greedy)."""
    rng = np.random.default_rng(seed)
    logits = (rng.standard_normal((B, V), dtype=np.float32) * np.float32(3.0))
    for b in range(B):
        idx = rng.choice(V, 8, replace=False)
        logits[b, idx] += np.float32(8.0)
    hist, off = _uniform_history(rng, B, H, V)
    params = dict(greedy=greedy, temperature=0.8, top_p=0.9, top_k=40, repetition_penalty=1.1)
    return dict(name="peaked_head_1x32000", logits=logits, hist_ids=hist, hist_offsets=off,
                uniforms=_uniforms(rng, B), params=params)


def zipf_history_nucleus(B=32, V=32000, H=512, seed=2):
    """N(0,2^2) logits; 512-id Zipf(1.1) histories over a seeded vocab permutation;
    frequency 0.5, presence 0.3, T 1.0, top-p 0.95, no top-k (full-vocab nucleus)."""
    rng = np.random.default_rng(seed)
    logits = rng.standard_normal((B, V), dtype=np.float32) * np.float32(2.0)
    perm = rng.permutation(V).astype(np.int32)
    pmf = np.power(np.arange(1, V + 1, dtype=np.float64), -1.1)
    cdf = np.cumsum(pmf)
    cdf /= cdf[-1]
    ranks = np.searchsorted(cdf, rng.random(B * H), side="right")
    ranks = np.minimum(ranks, V - 1)
    hist = perm[ranks].astype(np.int32)
    off = (np.arange(B + 1, dtype=np.int64) * H).astype(np.int32)
    params = dict(temperature=1.0, top_p=0.95, top_k=INT_MAX, frequency_penalty=0.5,
                  presence_penalty=0.3)
    return dict(name="zipf_history_nucleus_32x32000", logits=logits, hist_ids=hist,
                hist_offsets=off, uniforms=_uniforms(rng, B), params=params)


def zipf_ranked(B=256, V=128256, H=1024, seed=3, repetition_penalty=1.15, temperature=0.7,
                top_k=50, top_p=0.9, name="zipf_ranked_topk_256x128256"):
    """N(0,2.5^2) noise plus a Zipf(1.0)-shaped rank offset spanning 12 nats placed
    through a per-row permutation; 1024-id uniform history; repetition 1.15,
    T 0.7, top-k 50, top-p 0.9. This is the headline workload."""
    rng = np.random.default_rng(seed)
    logits = rng.standard_normal((B, V), dtype=np.float32) * np.float32(2.5)
    offs = zipf_rank_offsets(V, 12.0)
    perms = rng.permuted(np.tile(np.arange(V, dtype=np.int32), (B, 1)), axis=1)
    rows = np.arange(B)[:, None]
    logits[rows, perms] += offs[None, :]
    hist, off = _uniform_history(rng, B, H, V)
    params = dict(temperature=temperature, top_p=top_p, top_k=top_k,
                  repetition_penalty=repetition_penalty)
    return dict(name=name, logits=logits, hist_ids=hist, hist_offsets=off,
                uniforms=_uniforms(rng, B), params=params)


def high_entropy_nucleus(B=1024, V=151936, H=256, seed=4):
    """N(0,0.5^2) logits (nucleus spans most of the vocab); T 1.2, top-p 0.99,
    no top-k, presence 0.2 over a 256-id uniform history."""
    rng = np.random.default_rng(seed)
    logits = rng.standard_normal((B, V), dtype=np.float32) * np.float32(0.5)
    hist, off = _uniform_history(rng, B, H, V)
    params = dict(temperature=1.2, top_p=0.99, top_k=INT_MAX, presence_penalty=0.2)
    return dict(name="high_entropy_nucleus_1024x151936", logits=logits, hist_ids=hist,
                hist_offsets=off, uniforms=_uniforms(rng, B), params=params)


def vocab_sharded(B=128, V=262144, H=2048, seed=5):
    """The zipf_ranked generator at V=262144 with a 2048-id history; repetition 1.1,
    T 0.8, top-k 64, top-p 0.9 (split into contiguous vocab shards across GPUs)."""
    return zipf_ranked(B=B, V=V, H=H, seed=seed, repetition_penalty=1.1, temperature=0.8,
                       top_k=64, top_p=0.9, name="vocab_sharded_128x262144")


WORKLOADS = {
    "peaked_head": peaked_head,
    "zipf_history_nucleus": zipf_history_nucleus,
    "zipf_ranked": zipf_ranked,
    "high_entropy_nucleus": high_entropy_nucleus,
    "vocab_sharded": vocab_sharded,
}


def bytes_per_row(V: int, H: int) -> int:
    """Algorithmic HBM bytes per sampled row: logits 4V, history 4H, u 4, token 4."""
    return 4 * V + 4 * H + 8
