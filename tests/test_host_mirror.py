"""The C++ host mirror (neuraval_b200/host/neuraval_generation.hpp) compiled with
g++ against libnavsampler and run on the reference's own test cases
(tests/cpp/host_mirror_tests.cpp), including a TextGenerator decode loop over a
toy model (host logits and device-resident logits)."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def _build(tmp_path):
    from neuraval_b200 import build
    lib = build.build()
    inc = tmp_path / "kats.inc"
    subprocess.run([sys.executable, os.path.join(ROOT, "tests", "cpp", "gen_kats.py"),
                    os.path.join(ROOT, "tests", "golden", "reference_kats.json"), str(inc)],
                   check=True)
    exe = tmp_path / "host_mirror_tests"
    libdir = os.path.dirname(lib)
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Wextra",
                    "-I", os.path.join(ROOT, "include"),
                    "-I", os.path.join(ROOT, "neuraval_b200", "host"), "-I", str(tmp_path),
                    "-I", os.path.join(CUDA, "include"),
                    os.path.join(ROOT, "tests", "cpp", "host_mirror_tests.cpp"),
                    "-L", libdir, "-lnavsampler", f"-Wl,-rpath,{libdir}",
                    "-L", os.path.join(CUDA, "lib64"), "-lcudart", f"-Wl,-rpath,{os.path.join(CUDA, 'lib64')}",
                    "-o", str(exe)],
                   check=True)
    return exe


def test_host_mirror_options_without_gpu(tmp_path):
    exe = _build(tmp_path)
    r = subprocess.run([str(exe), "--options-only"], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr


@pytest.mark.gpu
def test_host_mirror_reference_tests_on_gpu(tmp_path):
    exe = _build(tmp_path)
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    print(r.stdout)
