"""The chunked top-k kernels (topk_chunk_kernel + topk_chunk_finish_kernel):
every top-k <= 64 call on wide rows without a probability output.

Bar: tokens and flags equal the oracle's bit for bit with the correctly rounded
exp, the same as the one-CTA-per-row kernel's (NAVSAMPLER_CHUNKED=0), and,
against libm expf, equal on every row without a boundary or tie flag. Rows the
finish cannot prove (a warp holding more than 8 of the row's top K, too many
ties, fewer than K finite values) are redone by the exact full-vocabulary
kernel; the tests count them.
"""
import numpy as np
import pytest

from neuraval_b200 import native, workloads
from tests.gpu_util import assert_exact, parity_report, run_gpu, run_oracle

pytestmark = pytest.mark.gpu


def _check(s, oracle, wl, label, offset=0, max_redone=None):
    before = s.full_sort_rows()
    gt, gf, _ = run_gpu(s, wl, offset=offset)
    redone = s.full_sort_rows() - before
    ot, of, _ = run_oracle(oracle, wl, oracle.EXP_CR)
    assert_exact(gt, gf, ot, of, label)
    lt, lf, _ = run_oracle(oracle, wl, oracle.EXP_GLIBC)
    rep = parity_report(gt, gf, lt, lf)
    assert rep["differ_unflagged"] == 0, (label, rep)
    if max_redone is not None:
        assert redone <= max_redone, (label, redone)
    return gt, gf, redone


@pytest.fixture(scope="module")
def sampler(navlib):
    from neuraval_b200.sampler import CudaTokenSampler
    s = CudaTokenSampler(device=0, max_rows=256, max_vocab=262144, max_history=2048)
    yield s
    s.close()


@pytest.fixture(scope="module")
def row_sampler(navlib):
    """A handle on the one-CTA-per-row kernel, for side-by-side checks."""
    import os
    from neuraval_b200.sampler import CudaTokenSampler
    os.environ["NAVSAMPLER_CHUNKED"] = "0"  # read when the handle is created
    try:
        s = CudaTokenSampler(device=0, max_rows=256, max_vocab=262144, max_history=2048)
    finally:
        del os.environ["NAVSAMPLER_CHUNKED"]
    yield s
    s.close()


def test_headline_batch_twice(sampler, row_sampler, oracle):
    wl = workloads.zipf_ranked()
    for call in range(2):  # the kept-value scratch is reused
        gt, gf, redone = _check(sampler, oracle, wl, f"zipf_ranked call {call}", max_redone=0)
    rt, rf, _ = run_gpu(row_sampler, wl)
    assert np.array_equal(gt, rt) and np.array_equal(gf, rf)


@pytest.mark.parametrize("B,V,K", [(1, 32000, 40), (3, 8192, 8), (5, 8195, 10),
                                   (7, 40003, 50), (16, 262144, 64), (2, 131075, 64)])
def test_shapes(sampler, oracle, B, V, K):
    wl = workloads.zipf_ranked(B=B, V=V, H=300, seed=B * 31 + V % 97, top_k=K)
    _check(sampler, oracle, wl, f"B={B} V={V} K={K}")
    _check(sampler, oracle, wl, f"B={B} V={V} K={K} unaligned", offset=1)


def test_peaked_head_rows(sampler, oracle):
    wl = workloads.peaked_head(B=64, seed=5)
    _check(sampler, oracle, wl, "peaked_head x64")


def test_vocab_sharded_batch(sampler, oracle):
    wl = workloads.vocab_sharded()
    _check(sampler, oracle, wl, "vocab_sharded 128x262144", max_redone=0)


def test_counts_penalties(sampler, oracle):
    wl = workloads.zipf_history_nucleus(B=24, V=65536, H=700, seed=8)
    wl["params"] = dict(temperature=0.9, top_k=48, top_p=0.85, repetition_penalty=1.2,
                        frequency_penalty=0.4, presence_penalty=0.2)
    _check(sampler, oracle, wl, "frequency/presence")


@pytest.mark.parametrize("mantissa_bits", [7, 3, 1])
def test_quantised_logits(sampler, oracle, mantissa_bits):
    """bf16-like and coarser logits: ties at the K-th value, at warps' cutoffs
    and at the draw."""
    wl = workloads.zipf_ranked(B=48, V=50000, H=256, seed=31)
    m, e = np.frexp(wl["logits"])
    q = np.float32(2.0 ** (mantissa_bits + 1))
    wl["logits"] = np.ldexp(np.round(m * q) / q, e).astype(np.float32)
    _check(sampler, oracle, wl, f"quantised {mantissa_bits}")


def test_edge_rows(sampler, oracle):
    rng = np.random.default_rng(11)
    V = 40000
    rows = []
    r = rng.standard_normal(V).astype(np.float32) * 2
    rows.append(r)
    r = r.copy(); r[12345] = np.nan; rows.append(r)                      # NaN: -1, nonfinite
    r = rows[0].copy(); r[V - 1] = np.inf; rows.append(r)                # +inf: -1, nonfinite
    r = rows[0].copy(); r[777] = 3.0e38; r[778] = 3.0e38; rows.append(r)  # finite, x1/T overflows
    rows.append(np.zeros(V, np.float32))                                 # all equal: fix-up
    r = np.full(V, -np.inf, np.float32); r[rng.choice(V, 20, replace=False)] = 1.0
    rows.append(r)                                                       # fewer than K finite
    rows.append(np.full(V, -np.inf, np.float32))                         # no finite value
    r = np.where(rng.random(V) < 0.7, -np.inf, rng.standard_normal(V)).astype(np.float32)
    rows.append(r)                                                       # masked columns
    r = rng.standard_normal(V).astype(np.float32)
    r[1000:1064] += 20.0                                                 # top K in one warp's range
    rows.append(r)
    r = rng.standard_normal(V).astype(np.float32)
    r[0:3] = 9.0; r[-3:] = 9.5                                           # head and tail scalars
    rows.append(r)
    r = rng.standard_normal(V).astype(np.float32); r[5] = -0.0; r[6] = 0.0
    rows.append(r)
    logits = np.stack(rows)
    B = logits.shape[0]
    Hs = rng.integers(0, 60, B)
    hist = np.concatenate([rng.integers(-5, V + 5, h) for h in Hs]).astype(np.int32)
    hist[:3] = [777, 12345, V - 1]
    offs = np.concatenate([[0], np.cumsum(Hs)]).astype(np.int32)
    wl = dict(name="edge", logits=logits, hist_ids=hist, hist_offsets=offs,
              uniforms=rng.random(B).astype(np.float32),
              params=dict(temperature=0.7, top_p=0.8, top_k=50, repetition_penalty=1.3))
    for off in (0, 1, 3):
        gt, gf, _ = _check(sampler, oracle, wl, f"edge rows offset {off}", offset=off)
        assert gt[1] == -1 and gf[1] & native.FLAG_NONFINITE
        assert gt[2] == -1 and gf[2] & native.FLAG_NONFINITE
        assert gt[6] == -1 and gf[6] & native.FLAG_NONFINITE


def test_raising_penalty_and_probs_take_the_row_kernel(sampler, oracle):
    """Penalties that can raise a value (repetition < 1) and calls that want the
    probabilities keep the one-CTA-per-row kernel; results stay exact."""
    wl = workloads.zipf_ranked(B=6, V=50000, H=256, seed=3, repetition_penalty=0.8)
    _check(sampler, oracle, wl, "repetition < 1")
    wl = workloads.zipf_ranked(B=6, V=50000, H=256, seed=4)
    gt, gf, gp = run_gpu(sampler, wl, want_probs=True)
    ot, of, op = run_oracle(oracle, wl, oracle.EXP_CR, want_probs=True)
    assert_exact(gt, gf, ot, of, "with probabilities")
    assert np.array_equal(gp, op)


def test_vocab_shards_through_the_chunked_kernels(sampler, row_sampler, oracle):
    """Shards of 40000 columns (two per 80000-column row) take the chunked
    stream and finish kernels, the finish writing each row's shard record; rows
    it cannot prove (top K in one warp's range, all values equal, fewer than K
    finite values) are redone by the one-CTA-per-row shard kernel. The merged
    tokens and flags equal those of the one-CTA-per-row shard kernel on every
    row, and the oracle's on every row whose ties did not overflow a record."""
    from tests.test_vocab_shard_gpu import run_sharded
    rng = np.random.default_rng(29)
    V = 80000
    rows = []
    base = rng.standard_normal(V).astype(np.float32) * 2
    rows.append(base)
    r = base.copy(); r[12345] = np.nan; rows.append(r)
    r = base.copy(); r[V - 1] = np.inf; rows.append(r)
    rows.append(np.zeros(V, np.float32))
    r = np.full(V, -np.inf, np.float32); r[rng.choice(V, 20, replace=False)] = 1.0
    rows.append(r)
    r = np.where(rng.random(V) < 0.7, -np.inf, rng.standard_normal(V)).astype(np.float32)
    rows.append(r)
    for lo in (1000, 41000, 39990):  # top K inside one warp's range of either shard, or across
        r = rng.standard_normal(V).astype(np.float32)
        r[lo:lo + 64] += 20.0
        rows.append(r)
    r = rng.standard_normal(V).astype(np.float32)
    r[0:3] = 9.0; r[-3:] = 9.5; r[39998:40002] = 9.2
    rows.append(r)
    logits = np.stack(rows)
    B = logits.shape[0]
    Hs = rng.integers(0, 60, B)
    hist = np.concatenate([rng.integers(-5, V + 5, h) for h in Hs]).astype(np.int32)
    hist[:3] = [777, 12345, V - 1]
    offs = np.concatenate([[0], np.cumsum(Hs)]).astype(np.int32)
    for params in (dict(temperature=0.7, top_p=0.8, top_k=50, repetition_penalty=1.3),
                   dict(temperature=1.1, top_p=0.95, top_k=64, frequency_penalty=0.4,
                        presence_penalty=0.2)):
        wl = dict(name="shard edge", logits=logits, hist_ids=hist, hist_offsets=offs,
                  uniforms=rng.random(B).astype(np.float32), params=params)
        ct, cf = run_sharded(sampler, wl, 2)
        rt, rf = run_sharded(row_sampler, wl, 2)
        assert np.array_equal(ct, rt) and np.array_equal(cf, rf), (params, ct, rt, cf, rf)
        ot, of, _ = run_oracle(oracle, wl, oracle.EXP_CR)
        ok = (cf & native.FLAG_TIES_OVERFLOW) == 0
        assert_exact(ct[ok], cf[ok], ot[ok], of[ok], "shard edge")
        assert ok[[0, 1, 2, 5, 6, 7, 8, 9]].all()  # rows whose ties cannot overflow a record
        assert ct[1] == -1 and ct[2] == -1  # NaN / +inf: -1 with NCB_FLAG_NONFINITE


@pytest.mark.parametrize("at", [200, 70000, 127900])
def test_clustered_top_k_rescans_instead_of_fix_up(sampler, oracle, at):
    """Every row's 64 largest values inside one 1024-value group (as common
    tokens with nearby ids can be): the finish cannot prove the K-th value from
    the kept values, reads the row again, and still samples every row itself
    (no row reaches the full-vocabulary fix-up); tokens equal the oracle's."""
    rng = np.random.default_rng(31 + at)
    B, V = 64, 128256
    logits = rng.standard_normal((B, V), dtype=np.float32) * 2.0
    logits[:, at:at + 64] += rng.uniform(6.0, 12.0, (B, 64)).astype(np.float32)
    H = 128
    hist = rng.integers(0, V, B * H).astype(np.int32)
    hist[::7] = at + rng.integers(0, 64, hist[::7].size)  # penalised ids inside the cluster
    wl = dict(name=f"clustered at {at}", logits=logits, hist_ids=hist,
              hist_offsets=(np.arange(B + 1) * H).astype(np.int32),
              uniforms=rng.random(B).astype(np.float32),
              params=dict(temperature=0.9, top_p=0.9, top_k=50, repetition_penalty=1.2))
    _check(sampler, oracle, wl, wl["name"], max_redone=0)
