"""GPU LogitsProcessor kernels against the oracle and the reference's KATs."""
import json
import os

import numpy as np
import pytest

from tests.test_oracle import check_processor_expectation

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
KATS = json.load(open(os.path.join(HERE, "golden", "reference_kats.json")))


def _dev(x, dtype=None):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _gpu_op(s, op, logits, hist, arg):
    import torch
    from neuraval_b200 import native
    x = _dev(np.asarray([logits], dtype=np.float32))
    h = _dev(np.asarray(hist if len(hist) else [0], dtype=np.int32))
    offs = _dev(np.asarray([0, len(hist)], dtype=np.int32))
    try:
        if op == "repetition_penalty":
            s.repetition_penalty_(x, h, offs, arg)
        elif op == "temperature":
            s.temperature_(x, arg)
        elif op == "filter_top_k":
            s.filter_top_k_(x, arg)
        else:
            s.filter_top_p_(x, arg)
    except native.NcbError as e:
        return e.status, None
    torch.cuda.synchronize()
    return 0, x.cpu().numpy()[0]


@pytest.mark.parametrize("case", KATS["processor"], ids=lambda c: f"{c['op']}@{c['src'].rsplit(':', 1)[1]}")
def test_processor_kats_on_gpu(gpu_sampler, case):
    st, out = _gpu_op(gpu_sampler, case["op"], case["logits"], case.get("history", []), case["arg"])
    check_processor_expectation(case, st, out)


def _batch(rng, B, V, H):
    x = (rng.standard_normal((B, V)) * 2).astype(np.float32)
    x[0] = np.round(x[0])  # ties
    x[1, ::3] = -0.0
    Hs = rng.integers(0, H, B)
    hist = np.concatenate([rng.integers(-3, V + 3, h) for h in Hs]).astype(np.int32)
    offs = np.concatenate([[0], np.cumsum(Hs)]).astype(np.int32)
    return x, hist, offs


@pytest.mark.parametrize("V", [7, 1000, 32001])
def test_penalties_and_temperature_match_oracle(gpu_sampler, oracle, V):
    import torch
    rng = np.random.default_rng(V)
    x, hist, offs = _batch(rng, 16, V, 300)
    for op, arg in (("rep", 1.3), ("rep", 0.7), ("fp", (0.5, 0.3)), ("temp", 0.7), ("temp", 1.9)):
        d = _dev(x)
        if op == "rep":
            gpu_sampler.repetition_penalty_(d, _dev(hist), _dev(offs), arg)
        elif op == "fp":
            gpu_sampler.frequency_presence_penalty_(d, _dev(hist), _dev(offs), *arg)
        else:
            gpu_sampler.temperature_(d, arg)
        torch.cuda.synchronize()
        got = d.cpu().numpy()
        for r in range(x.shape[0]):
            hr = hist[offs[r]:offs[r + 1]]
            if op == "rep":
                _, want = oracle.apply_repetition_penalty(x[r], hr, arg)
            elif op == "fp":
                _, want = oracle.apply_frequency_presence_penalty(x[r], hr, *arg)
            else:
                _, want = oracle.apply_temperature(x[r], arg)
            assert np.array_equal(got[r], want), (op, arg, r)


@pytest.mark.parametrize("V", [5, 1000, 40000])
def test_filter_top_k_matches_oracle(gpu_sampler, oracle, V):
    import torch
    rng = np.random.default_rng(V + 1)
    x, _, _ = _batch(rng, 8, V, 2)
    for k in (1, 2, min(50, V - 1), V - 1, V, V + 5):
        d = _dev(x)
        gpu_sampler.filter_top_k_(d, k)
        torch.cuda.synchronize()
        got = d.cpu().numpy()
        for r in range(x.shape[0]):
            _, want = oracle.filter_top_k(x[r], k)
            assert np.array_equal(got[r], want), (k, r)


@pytest.mark.parametrize("V", [4, 1000, 151936])
def test_filter_top_p_matches_oracle(gpu_sampler, oracle, V):
    import torch
    rng = np.random.default_rng(V + 2)
    z = (rng.standard_normal((6, V)) * np.array([[0.3], [1.0], [2.0], [4.0], [0.0], [1.5]])).astype(np.float64)
    p = np.exp(z - z.max(axis=1, keepdims=True))
    p = (p / p.sum(axis=1, keepdims=True)).astype(np.float32)
    p[5] = np.round(p[5] * 2000) / 2000  # ties
    for top_p in (0.05, 0.5, 0.9, 0.99, 1.0):
        d = _dev(p)
        fl = _dev(np.zeros(p.shape[0], np.int32))
        gpu_sampler.filter_top_p_(d, top_p, fl)
        torch.cuda.synchronize()
        got = d.cpu().numpy()
        gfl = fl.cpu().numpy()
        for r in range(p.shape[0]):
            _, want, tie = oracle.filter_top_p(p[r], top_p)
            assert bool(gfl[r] & 0x4) == bool(tie), (top_p, r)
            assert np.array_equal(got[r], want), (top_p, r)


def test_host_array_entry_points_match_device_ones(gpu_sampler):
    """ncb_logits_* on host arrays give the bits of the device entry points."""
    import ctypes
    import torch
    from neuraval_b200 import native
    lib = native.load()
    h = gpu_sampler._h
    rng = np.random.default_rng(91)
    B, V = 5, 7001
    x = (rng.standard_normal((B, V)) * 3).astype(np.float32)
    hist = rng.integers(-5, V + 5, size=40).astype(np.int32)
    offs = np.array([0, 8, 8, 20, 31, 40], np.int32)
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    T = lambda t: ctypes.c_void_p(t.data_ptr())

    def both(host_call, dev_call):
        a = x.copy()
        assert host_call(a) == 0
        d = torch.from_numpy(x).cuda()
        assert dev_call(d) == 0
        torch.cuda.synchronize()
        assert np.array_equal(a, d.cpu().numpy())

    dh, do = torch.from_numpy(hist).cuda(), torch.from_numpy(offs).cuda()
    both(lambda a: lib.ncb_logits_repetition_penalty(h, P(a), B, V, P(hist), P(offs), 1.3),
         lambda d: lib.ncb_logits_repetition_penalty_device(h, T(d), B, V, T(dh), T(do), 1.3, None))
    both(lambda a: lib.ncb_logits_frequency_presence_penalty(h, P(a), B, V, P(hist), P(offs),
                                                             0.4, 0.2),
         lambda d: lib.ncb_logits_frequency_presence_penalty_device(h, T(d), B, V, T(dh), T(do),
                                                                    0.4, 0.2, None))
    both(lambda a: lib.ncb_logits_temperature(h, P(a), B, V, 0.7),
         lambda d: lib.ncb_logits_temperature_device(h, T(d), B, V, 0.7, None))
    both(lambda a: lib.ncb_logits_filter_top_k(h, P(a), B, V, 37),
         lambda d: lib.ncb_logits_filter_top_k_device(h, T(d), B, V, 37, None))
    p = np.exp(x - x.max(axis=1, keepdims=True))
    x = (p / p.sum(axis=1, keepdims=True)).astype(np.float32)
    both(lambda a: lib.ncb_logits_filter_top_p(h, P(a), B, V, 0.9, None),
         lambda d: lib.ncb_logits_filter_top_p_device(h, T(d), B, V, 0.9, None, None))
    assert lib.ncb_logits_temperature(h, P(x.copy()), B, V, 0.0) == native.NCB_ERROR_INVALID_ARGUMENT
