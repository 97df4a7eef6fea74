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
    big = native.make_params(temperature=1.0, top_k=500)   # top-k above 64
    assert lib.ncb_sample_rows_noalloc_device(_ptr(t), 1, 16, None, _ptr(offs), _ptr(u),
                                              ctypes.byref(big), _ptr(tok), None, None,
                                              None) == native.NCB_ERROR_CAPACITY
    many = torch.zeros((2000, 16), dtype=torch.float32, device="cuda")
    offs2 = torch.zeros(2001, dtype=torch.int32, device="cuda")
    p = native.make_params(temperature=1.0, top_k=5)
    assert lib.ncb_sample_rows_noalloc_device(_ptr(many), 2000, 16, None, _ptr(offs2), _ptr(u),
                                              ctypes.byref(p), _ptr(tok), None, None,
                                              None) == native.NCB_ERROR_CAPACITY
