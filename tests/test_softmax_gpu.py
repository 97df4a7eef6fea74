"""Row softmax (ncb_softmax_rows_device) against the reference's own kernel
(ncb_cuda_softmax_rows_device, navcuda.cu:616-700, compiled from its source
into oracle/_ref): every output bit equal, NaN where the reference gives NaN.
Also against a float64 softmax within 1e-5 relative: the reference's own fp32
arithmetic (expf within 2 ulp, 501-term fp32 partial sums over 128256 columns)
is up to ~4e-6 relative from the exact value."""
import ctypes

import numpy as np
import pytest

from neuraval_b200 import native
from oracle import refcuda

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _ours(x, inplace=False):
    import torch
    d = torch.from_numpy(x).cuda()
    out = d if inplace else torch.empty_like(d)
    assert native.load().ncb_softmax_rows_device(_p(d), _p(out), x.shape[0], x.shape[1], None) == 0
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _reference(x):
    import torch
    lib = refcuda.load()
    assert lib.ncb_cuda_init(0) == 1
    d = torch.from_numpy(x).cuda()
    out = torch.empty_like(d)
    lib.ncb_cuda_softmax_rows_device(_p(d), _p(out), x.shape[0], x.shape[1])
    torch.cuda.synchronize()
    assert lib.ncb_cuda_last_status() == 0
    return out.cpu().numpy()


def _cases():
    rng = np.random.default_rng(17)
    yield "17x23", rng.standard_normal((17, 23), dtype=np.float32)
    yield "1x1", np.array([[3.5]], np.float32)
    yield "3x255", (rng.standard_normal((3, 255)) * 4).astype(np.float32)
    yield "5x256", (rng.standard_normal((5, 256)) * 4).astype(np.float32)
    yield "4x257", (rng.standard_normal((4, 257)) * 4).astype(np.float32)
    yield "6x4099", (rng.standard_normal((6, 4099)) * 8).astype(np.float32)
    yield "64x32000", (rng.standard_normal((64, 32000)) * 3).astype(np.float32)
    x = (rng.standard_normal((8, 5000)) * 5).astype(np.float32)
    x[0, :100] = -np.inf
    x[1, :] = -np.inf          # all -inf: 0/0 in both
    x[2, 7] = np.nan
    x[3, 11] = np.inf
    x[4, :] = 0.0
    x[4, 3] = -0.0
    x[5, ::2] = 88.0           # large equal maxima
    yield "special", x
    # rows of 8192+ columns take the cluster kernel (one cluster of CTAs per row)
    yield "3x8195", (rng.standard_normal((3, 8195)) * 4).astype(np.float32)
    yield "2x40003", (rng.standard_normal((2, 40003)) * 6).astype(np.float32)
    w = (rng.standard_normal((8, 9000)) * 5).astype(np.float32)
    w[0, :300] = -np.inf
    w[1, :] = -np.inf
    w[2, 4097] = np.nan
    w[3, 8999] = np.inf
    w[4, :] = 0.0
    w[4, 257] = -0.0
    w[5, 1::3] = 88.0
    w[6, 8191] = 1e30         # one huge maximum in the last piece
    yield "special_wide", w
    yield "1x393216", (rng.standard_normal((1, 393216)) * 3).astype(np.float32)
    yield "1x393217", (rng.standard_normal((1, 393217)) * 3).astype(np.float32)


@pytest.mark.parametrize("name,x", list(_cases()), ids=[c[0] for c in _cases()])
def test_softmax_bits_equal_reference_kernel(name, x):
    if not refcuda.available():
        pytest.skip("oracle/_ref/libnavcuda.so not built (needs the reference source tree)")
    got, ref = _ours(x), _reference(x)
    bad = np.argwhere(~((got == ref) | (np.isnan(got) & np.isnan(ref))))
    assert bad.size == 0, (name, bad[:5], got[tuple(bad[0])], ref[tuple(bad[0])])


def test_softmax_full_logits_batch():
    from neuraval_b200 import workloads
    x = workloads.zipf_ranked(B=256, V=128256, H=1, seed=5)["logits"]
    got = _ours(x)
    if refcuda.available():
        ref = _reference(x)
        assert np.array_equal(got, ref)
    e = np.exp(x.astype(np.float64) - x.max(axis=1, keepdims=True))
    want = e / e.sum(axis=1, keepdims=True)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-30)


def test_softmax_in_place_and_errors():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((9, 3001), dtype=np.float32)
    assert np.array_equal(_ours(x, inplace=True), _ours(x))
    x = rng.standard_normal((5, 20001), dtype=np.float32)  # the cluster kernel
    assert np.array_equal(_ours(x, inplace=True), _ours(x))
    lib = native.load()
    assert lib.ncb_softmax_rows_device(None, None, 0, 4, None) == native.NCB_ERROR_INVALID_ARGUMENT
    assert lib.ncb_softmax_rows_device(None, None, 2, 0, None) == native.NCB_ERROR_INVALID_ARGUMENT
