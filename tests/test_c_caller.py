"""The reference C ABI used from plain C: the headers compile as C (the way an
FFI binding such as cgo includes them), a C program links against
libfp8imma.so and the CUDA runtime only, and (on a GPU) its outputs for three
reference variants equal the CPU oracle bit for bit."""
import os
import subprocess
import tempfile

import numpy as np
import pytest

from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "cuda-fp8-ampere_b200")
SRC = os.path.join(ROOT, "tests", "c_caller", "fp8imma_c_caller.c")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def _build(out_dir):
    exe = os.path.join(out_dir, "fp8imma_c_caller")
    cmd = ["gcc", "-std=c11", "-O2", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), "-I",
           os.path.join(CUDA, "include"), SRC, "-L", PKG, "-lfp8imma", "-L", os.path.join(CUDA, "lib64"), "-lcudart",
           "-Wl,-rpath," + PKG, "-o", exe]
    subprocess.run(cmd, check=True, capture_output=True)
    return exe


def test_headers_are_c_and_the_caller_links():
    tu = '#include "fp8imma/imma_fp8.h"\n#include "fp8imma/fp8imma_ext.h"\nint main(void) { return 0; }\n'
    subprocess.run(["gcc", "-std=c11", "-fsyntax-only", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                    "-I", os.path.join(CUDA, "include"), "-x", "c", "-"], input=tu.encode(), check=True,
                   capture_output=True)
    with tempfile.TemporaryDirectory() as d:
        assert os.path.exists(_build(d))


def _lcg_inputs(M, N, K):
    s = 12345

    def nxt():
        nonlocal s
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        return s

    A = np.empty(M * K, np.uint16)
    for i in range(M * K):
        r = nxt()
        A[i] = ((r >> 31) << 15) | ((12 + (r >> 8) % 5) << 10) | (r & 0x3FF)
    B = np.array([nxt() >> 24 for _ in range(N * K)], np.uint8)
    S = np.array([0x3800 + (nxt() >> 22) for _ in range(N)], np.uint16)
    return A.reshape(M, K), B.reshape(N, K), S


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(16, 200, 512), (1, 96, 1024), (48, 64, 256)])
def test_c_caller_matches_oracle(cuda, M, N, K):
    with tempfile.TemporaryDirectory() as d:
        exe = _build(d)
        out = os.path.join(d, "out.bin")
        r = subprocess.run([exe, str(M), str(N), str(K), out], capture_output=True)
        assert r.returncode == 0, (r.returncode, r.stderr)
        got = np.fromfile(out, np.uint16).reshape(3, N, M)
    A, B, S = _lcg_inputs(M, N, K)
    for i, (variant, kchunk) in enumerate([("v4_f16", 32), ("v3_f16", 32), ("v4_f16", 64)]):
        _, D_o, _ = O.imma_fp8(variant, kchunk, A, B, S, 0.125, 8.0)
        assert np.array_equal(got[i], D_o), variant
