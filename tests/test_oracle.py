"""CPU tests of the oracle: the reference's own known-answer cases, an
independent Python restatement, the correctly rounded exp, and the generators."""
import ctypes
import json
import os
from decimal import Decimal, getcontext

import numpy as np
import pytest

from tests import pyref

HERE = os.path.dirname(os.path.abspath(__file__))
KATS = json.load(open(os.path.join(HERE, "golden", "reference_kats.json")))


@pytest.mark.parametrize("case", KATS["sampler"], ids=lambda c: c["name"])
@pytest.mark.parametrize("mode", [0, 1])
def test_sampler_kats(oracle, case, mode):
    p = oracle.make_params(**case["params"])
    for u in case["uniforms"]:
        tok, flags, _ = oracle.sample_row(case["logits"], case["history"], p, u=u, exp_mode=mode)
        assert tok == case["expect"], (case["src"], u)


def _run_processor(oracle, case):
    op, x, arg = case["op"], case["logits"], case["arg"]
    if op == "repetition_penalty":
        return oracle.apply_repetition_penalty(x, case["history"], arg)
    if op == "temperature":
        return oracle.apply_temperature(x, arg)
    if op == "filter_top_k":
        return oracle.filter_top_k(x, arg)
    st, out, _ = oracle.filter_top_p(x, arg)
    return st, out


def check_processor_expectation(case, st, out):
    exp = case["expect"]
    if exp == "invalid":
        assert st == 7, case["src"]
        return
    assert st == 0, case["src"]
    if exp == "nucleus_2_renormalised":
        # LogitsProcessorTests.cs:132-139
        assert out[2] == 0 and out[3] == 0 and out[0] > 0 and out[1] > 0
        assert abs(float(out.sum()) - 1.0) < 5e-6
        return
    want = np.array([-np.inf if e == "-inf" else e for e in exp], dtype=np.float32)
    assert np.array_equal(out, want), (case["src"], out, want)


@pytest.mark.parametrize("case", KATS["processor"], ids=lambda c: f"{c['op']}@{c['src'].rsplit(':', 1)[1]}")
def test_processor_kats(oracle, case):
    st, out = _run_processor(oracle, case)
    check_processor_expectation(case, st, out)


def _random_row(rng, V):
    kind = rng.integers(0, 4)
    if kind == 0:
        x = rng.standard_normal(V).astype(np.float32) * 3
    elif kind == 1:  # many ties
        x = np.round(rng.standard_normal(V) * 2).astype(np.float32)
    elif kind == 2:  # zeros, negative zeros, -inf
        x = rng.choice(np.array([0.0, -0.0, 1.0, -1.0, -np.inf, 2.5], dtype=np.float32), V)
        x[rng.integers(0, V)] = 3.0
    else:
        x = (rng.standard_normal(V) * 0.01).astype(np.float32)
    H = int(rng.integers(0, 12))
    hist = rng.integers(-3, V + 3, H).astype(np.int32)
    return x, hist


def test_oracle_matches_python_restatement(oracle):
    rng = np.random.default_rng(7)
    n = 0
    for V in (1, 2, 3, 5, 17, 64, 257):
        for _ in range(25):
            x, hist = _random_row(rng, V)
            p = dict(greedy=bool(rng.integers(0, 5) == 0),
                     temperature=float(rng.choice([0.3, 0.7, 1.0, 1.7])),
                     top_p=float(rng.choice([0.2, 0.9, 0.95, 1.0])),
                     top_k=int(rng.choice([1, 2, 5, 40, 2**31 - 1])),
                     repetition_penalty=float(rng.choice([1.0, 1.1, 2.0, 0.5])),
                     frequency_penalty=float(rng.choice([0.0, 0.5])),
                     presence_penalty=float(rng.choice([0.0, 0.3])))
            u = float(np.float32(rng.random()))
            want = pyref.sample_next(x, [int(t) for t in hist], p, u)
            got, flags, _ = oracle.sample_row(x, hist, oracle.make_params(**p), u=u,
                                              exp_mode=oracle.EXP_GLIBC)
            if flags & oracle.FLAG_NONFINITE:
                continue
            assert got == want, (V, p, u, x, hist)
            n += 1
    assert n > 150


def test_expf_cr_matches_high_precision():
    from oracle import pyoracle
    getcontext().prec = 60
    rng = np.random.default_rng(11)
    xs = np.concatenate([-rng.exponential(3.0, 1500), rng.uniform(-103, 0, 500)]).astype(np.float32)
    for x in xs:
        e = Decimal(float(x)).exp()
        f = np.float32(float(e))
        best = min([f, np.nextafter(f, np.float32(np.inf)), np.nextafter(f, np.float32(0))],
                   key=lambda c: abs(Decimal(float(c)) - e))
        r, _ = pyoracle.expf_cr(float(x))
        assert np.float32(r) == best, float(x)
        assert np.float32(pyoracle.expf_dd(float(x))) == best, float(x)


def test_glibc_expf_rarely_misrounds(oracle):
    """MathF.Exp (libm expf) and the correctly rounded exp differ in well under 1%
    of arguments; the parity tests count the rows this could affect."""
    libm = ctypes.CDLL("libm.so.6")
    libm.expf.argtypes = [ctypes.c_float]
    libm.expf.restype = ctypes.c_float
    xs = -np.random.default_rng(3).exponential(2.0, 20000).astype(np.float32)
    diff = sum(np.float32(libm.expf(float(x))) != np.float32(oracle.expf_cr(float(x))[0]) for x in xs)
    assert diff < 0.005 * len(xs)


def test_params_validation_matches_generation_options(navlib):
    from neuraval_b200 import native
    base = KATS["options_base"]
    assert navlib.ncb_sampler_params_validate(native.make_params(**base)) == 0
    for case in KATS["options"]:
        p = dict(base)
        p[case["field"]] = case["value"]
        st = navlib.ncb_sampler_params_validate(native.make_params(**p))
        assert st == native.NCB_ERROR_INVALID_ARGUMENT, case["src"]
    p = dict(base, frequency_penalty=float("nan"))
    assert navlib.ncb_sampler_params_validate(native.make_params(**p)) == 7
    assert navlib.ncb_sampler_params_validate(None) == 7


def test_workloads_are_seeded_and_shaped():
    from neuraval_b200 import workloads as w
    a = w.peaked_head()
    b = w.peaked_head()
    assert np.array_equal(a["logits"], b["logits"]) and np.array_equal(a["uniforms"], b["uniforms"])
    assert a["logits"].shape == (1, 32000) and a["hist_offsets"][-1] == 64
    c = w.zipf_history_nucleus(B=4)
    assert c["logits"].shape == (4, 32000) and c["hist_offsets"][-1] == 4 * 512
    assert c["hist_ids"].min() >= 0 and c["hist_ids"].max() < 32000
    d = w.zipf_ranked(B=2, V=4096, H=16)
    assert d["logits"].dtype == np.float32 and (d["uniforms"] < 1).all()
    assert w.bytes_per_row(128256, 1024) == 517128
