"""The reference's own CUDA library, Neuraval.Cuda.Native (navcuda.cu), compiled
from its source for sm_100a by `make -C oracle ref` into oracle/_ref/.

Test infrastructure only: what the row-softmax tests compare against (the reference's
ncb_cuda_softmax_rows_device, navcuda.cu:616-700). The compiled library travels
with the repository copy; building it needs the reference source tree.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_ref", "libnavcuda.so")
SRC = "/root/reference/Neuraval.Cuda.Native/src/navcuda.cu"

_lib = None


def build() -> bool:
    """Compiles the reference library when its source is present; True when it exists."""
    if os.path.exists(SRC):
        subprocess.run(["make", "-s", "-C", HERE, "ref"], check=True)
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
