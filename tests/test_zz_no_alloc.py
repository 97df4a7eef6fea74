"""The allocation-free entry point (ncb_sample_rows_noalloc_device).

It exists for callers that cannot allocate device memory when they sample (a
process whose device memory is all owned by its own pool or another allocator,
or a loop that cannot afford cudaMalloc's device synchronisation); its scratch is
a fixed device array inside the library. These tests call it through the C ABI
and require the same tokens, flags and probabilities as the handle-based entry
point, on two calls in a row (the array keeps the previous call's contents).
This file is collected last so a failure here never hides the other tests.
"""
import ctypes

import numpy as np
import pytest

from neuraval_b200 import native, workloads

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _run_noalloc(lib, dev, params, want_probs):
    import torch
    logits, hist, offs, u = dev
    B, V = logits.shape
    tokens = torch.full((B,), -7, dtype=torch.int32, device="cuda")
    flags = torch.zeros(B, dtype=torch.int32, device="cuda")
    probs = torch.full((B, V), -1.0, dtype=torch.float32, device="cuda") if want_probs else None
    st = lib.ncb_sample_rows_noalloc_device(_ptr(logits), B, V, _ptr(hist), _ptr(offs), _ptr(u),
                                            ctypes.byref(params), _ptr(tokens), _ptr(flags),
                                            _ptr(probs), None)
    assert st == native.NCB_OK, st
    torch.cuda.synchronize()
    return (tokens.cpu().numpy(), flags.cpu().numpy().astype(np.uint32),
            probs.cpu().numpy() if want_probs else None)


@pytest.mark.parametrize("case", ["topk_split_rows", "topk_counts", "greedy"])
def test_noalloc_matches_handle_entry_point_twice(case, navlib):
    from neuraval_b200.sampler import CudaTokenSampler
    from tests.gpu_util import run_gpu, to_dev
    lib = navlib
    if case == "topk_split_rows":       # few rows: every row is split across CTAs
        wl = workloads.zipf_ranked(B=12, V=60000, H=200, seed=41)
    elif case == "topk_counts":
        wl = workloads.zipf_history_nucleus(B=40, V=32000, H=300, seed=42)
        wl["params"] = dict(wl["params"], top_k=40)
    else:
        wl = workloads.peaked_head(B=20, V=48000, seed=43, greedy=True)
    want_probs = case != "greedy"
    params = native.make_params(**wl["params"])
    with CudaTokenSampler(0, max_rows=64, max_vocab=65536, max_history=1024) as s:
        rt, rf, rp = run_gpu(s, wl, want_probs=want_probs)
    dev = to_dev(wl)
    for call in range(2):
        gt, gf, gp = _run_noalloc(lib, dev, params, want_probs)
        assert np.array_equal(gt, rt), (case, call, gt, rt)
        assert np.array_equal(gf, rf), (case, call)
        if want_probs:
            assert np.array_equal(gp, rp), (case, call)


def test_noalloc_rejects_what_it_does_not_serve(navlib):
    import torch
    lib = navlib
    t = torch.zeros((1, 16), dtype=torch.float32, device="cuda")
    offs = torch.zeros(2, dtype=torch.int32, device="cuda")
    u = torch.zeros(1, dtype=torch.float32, device="cuda")
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    # top-k above 64 on a row wide enough that top_k < vocab
    wide = torch.zeros((1, 1000), dtype=torch.float32, device="cuda")
    big = native.make_params(temperature=1.0, top_k=65)
    assert lib.ncb_sample_rows_noalloc_device(_ptr(wide), 1, 1000, None, _ptr(offs), _ptr(u),
                                              ctypes.byref(big), _ptr(tok), None, None,
                                              None) == native.NCB_ERROR_CAPACITY
    # top_k >= vocab: "no top-k", the full-vocabulary nucleus
    narrow = torch.zeros((1, 40), dtype=torch.float32, device="cuda")
    nok = native.make_params(temperature=1.0, top_k=50)
    assert lib.ncb_sample_rows_noalloc_device(_ptr(narrow), 1, 40, None, _ptr(offs), _ptr(u),
                                              ctypes.byref(nok), _ptr(tok), None, None,
                                              None) == native.NCB_ERROR_CAPACITY
    many = torch.zeros((2000, 16), dtype=torch.float32, device="cuda")
    offs2 = torch.zeros(2001, dtype=torch.int32, device="cuda")
    p = native.make_params(temperature=1.0, top_k=5)
    assert lib.ncb_sample_rows_noalloc_device(_ptr(many), 2000, 16, None, _ptr(offs2), _ptr(u),
                                              ctypes.byref(p), _ptr(tok), None, None,
                                              None) == native.NCB_ERROR_CAPACITY


def _compare_twice(lib, wl, sampler_kwargs, want_probs=True):
    from neuraval_b200.sampler import CudaTokenSampler
    from tests.gpu_util import run_gpu, to_dev
    params = native.make_params(**wl["params"])
    with CudaTokenSampler(0, **sampler_kwargs) as s:
        rt, rf, rp = run_gpu(s, wl, want_probs=want_probs)
    dev = to_dev(wl)
    for call in range(2):
        gt, gf, gp = _run_noalloc(lib, dev, params, want_probs)
        assert np.array_equal(gt, rt), (call, np.nonzero(gt != rt)[0][:8])
        assert np.array_equal(gf, rf), call
        if want_probs:
            assert np.array_equal(gp, rp), call
    return rt, rf


def test_noalloc_single_wide_row_top64(navlib):
    """One 300000-column row with top-k 64: the row is split into column
    segments whose candidate lists must all fit the merge (K x segments)."""
    wl = workloads.zipf_ranked(B=1, V=300000, H=500, seed=44, top_k=64)
    rt, rf = _compare_twice(navlib, wl, dict(max_rows=1, max_vocab=300000, max_history=1024))
    assert rt[0] >= 0 and (rf[0] & native.FLAG_TIES_OVERFLOW) == 0


def test_noalloc_600_rows(navlib):
    """More rows than the segment budget allows to split: one CTA per row."""
    wl = workloads.zipf_ranked(B=600, V=8192, H=64, seed=45)
    _compare_twice(navlib, wl, dict(max_rows=600, max_vocab=8192, max_history=64),
                   want_probs=False)


def test_noalloc_tied_row_overflows(navlib):
    """A row whose every value equals the k-th value overflows the candidate
    buffers: the handle path resolves it with its full-vocabulary scratch, the
    allocation-free path returns -1 with NCB_FLAG_TIES_OVERFLOW. The other rows
    of the batch are unaffected."""
    from neuraval_b200.sampler import CudaTokenSampler
    from tests.gpu_util import run_gpu, to_dev
    wl = workloads.zipf_ranked(B=4, V=20000, H=32, seed=46, top_k=40)
    wl["logits"][2, :] = np.float32(1.5)
    params = native.make_params(**wl["params"])
    with CudaTokenSampler(0, max_rows=4, max_vocab=20000, max_history=64) as s:
        rt, rf, _ = run_gpu(s, wl)
    assert rt[2] >= 0
    dev = to_dev(wl)
    for call in range(2):
        gt, gf, _ = _run_noalloc(navlib, dev, params, False)
        assert gt[2] == -1 and (gf[2] & native.FLAG_TIES_OVERFLOW) != 0, (call, gt, gf)
        keep = np.array([0, 1, 3])
        assert np.array_equal(gt[keep], rt[keep]) and np.array_equal(gf[keep], rf[keep]), call


def test_noalloc_long_history_with_counts(navlib):
    """Frequency counting over more history ids than the allocation-free path
    counts (4096): that row returns -1 with NCB_FLAG_BAD_HISTORY; the handle path
    created for 8192 ids samples it; other rows agree."""
    from neuraval_b200.sampler import CudaTokenSampler
    from tests.gpu_util import run_gpu, to_dev
    rng = np.random.default_rng(47)
    B, V = 3, 16000
    lens = np.array([100, 5000, 200])
    wl = workloads.zipf_ranked(B=B, V=V, H=1, seed=47, top_k=20)
    wl["hist_ids"] = rng.integers(0, V, size=int(lens.sum()), dtype=np.int64).astype(np.int32)
    wl["hist_offsets"] = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    wl["params"] = dict(wl["params"], frequency_penalty=0.4, presence_penalty=0.1)
    params = native.make_params(**wl["params"])
    with CudaTokenSampler(0, max_rows=B, max_vocab=V, max_history=8192) as s:
        rt, rf, _ = run_gpu(s, wl)
    assert rt[1] >= 0 and (rf[1] & native.FLAG_BAD_HISTORY) == 0
    dev = to_dev(wl)
    for call in range(2):
        gt, gf, _ = _run_noalloc(navlib, dev, params, False)
        assert gt[1] == -1 and (gf[1] & native.FLAG_BAD_HISTORY) != 0, (call, gt, gf)
        keep = np.array([0, 2])
        assert np.array_equal(gt[keep], rt[keep]) and np.array_equal(gf[keep], rf[keep]), call
