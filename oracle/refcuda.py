"""The reference's own CUDA library, Neuraval.Cuda.Native (navcuda.cu), compiled
from its source for sm_100a by `make -C oracle ref` into oracle/_ref/.

Test infrastructure only: what the row-softmax tests compare against (the reference's
ncb_cuda_softmax_rows_device, navcuda.cu:616-700). The compiled library travels
with the repository copy; building it needs the reference source tree, whose
root the NEURAVAL_REFERENCE environment variable names (no default).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_ref", "libnavcuda.so")
SRC_REL = os.path.join("Neuraval.Cuda.Native", "src", "navcuda.cu")

_lib = None


def source() -> str | None:
    """The reference's navcuda.cu under NEURAVAL_REFERENCE, or None."""
    root = os.environ.get("NEURAVAL_REFERENCE")
    if not root:
        return None
    src = os.path.join(root, SRC_REL)
    return src if os.path.exists(src) else None


def build() -> bool:
    """Compiles the reference library when its source is present; True when it exists."""
    src = source()
    if src is not None:
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF_SRC={src}"], check=True)
    return os.path.exists(LIB)


def available() -> bool:
    return os.path.exists(LIB)


def load():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(LIB)
        lib.ncb_cuda_init.restype = ctypes.c_int
        lib.ncb_cuda_init.argtypes = [ctypes.c_int]
        lib.ncb_cuda_softmax_rows_device.restype = None
        lib.ncb_cuda_softmax_rows_device.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                                     ctypes.c_int]
        lib.ncb_cuda_last_status.restype = ctypes.c_int
        lib.ncb_cuda_last_status.argtypes = []
        _lib = lib
    return _lib
