"""Build the fp8imma B200 native libraries in-tree.

* ``libfp8imma.so`` — the CUDA kernels + C ABI (nvcc, sm_100a only), placed in
  this directory so it travels with the source tree;
* ``fp8imma_ext`` and ``fp8wgt_ext`` — the PyTorch extension modules (C++,
  compiled against torch's headers and linked to libfp8imma.so), placed in
  this directory under the reference's module names.

Run ``python cuda-fp8-ampere_b200/build.py`` (or call ``build_all()``).
Nothing is compiled at import time on the GPU box: the built files travel
with the repository.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libfp8imma.so")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-DFP8IMMA_NVTX", "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
              "--expt-relaxed-constexpr", "-I" + INCLUDE, "-I" + CSRC]

CU_SOURCES = ["api.cu", "gemv_splitk.cu", "decode.cu", "generic.cu", "fp8wgt.cu", "host_util.cu", "gemm_tc.cu", "noalloc.cu", "peer.cu", "quantize.cu"]


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("command failed: %s\n%s\n%s" % (" ".join(cmd), r.stdout, r.stderr))
    if os.environ.get("FP8IMMA_BUILD_VERBOSE"):
        sys.stderr.write(r.stdout + r.stderr)


def _newer(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return False
    t = os.path.getmtime(out)
    return all(os.path.getmtime(d) <= t for d in deps)


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs += [os.path.join(INCLUDE, "fp8imma", f) for f in os.listdir(os.path.join(INCLUDE, "fp8imma"))]
    return hs


def build_lib(force: bool = False, extra_flags: list[str] | None = None) -> str:
    """Compile every .cu for sm_100a and link libfp8imma.so."""
    os.makedirs(OBJ, exist_ok=True)
    hdrs = _headers()
    # objects built with other flags (or another nvcc) are stale whatever their age
    stamp = os.path.join(OBJ, "flags.txt")
    flags = " ".join([NVCC] + ARCH + NVCC_FLAGS + (extra_flags or []))
    if not os.path.exists(stamp) or open(stamp).read() != flags:
        force = True
    objs, jobs = [], []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ, src.replace(".cu", ".o"))
        objs.append(o)
        if force or not _newer(o, [s] + hdrs):
            jobs.append([NVCC] + ARCH + NVCC_FLAGS + (extra_flags or []) + ["-c", s, "-o", o])
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        list(ex.map(_run, jobs))
    relink = force or bool(jobs) or not _newer(LIB, objs)
    if relink:
        _run([NVCC] + ARCH + ["-shared", "-Xcompiler", "-fPIC", "-o", LIB] + objs + ["-lcudart"])
    with open(stamp, "w") as f:
        f.write(flags)
    sys.stderr.write("libfp8imma.so: %d of %d sources compiled, %s\n"
                     % (len(jobs), len(CU_SOURCES), "relinked" if relink else "up to date"))
    return LIB


def _torch_ext(name: str, sources: list[str], force: bool = False) -> str:
    import torch
    from torch.utils import cpp_extension as ce

    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    out = os.path.join(HERE, name + suffix)
    srcs = [os.path.join(HERE, "torch_ext", s) for s in sources]
    if not force and _newer(out, srcs + [LIB, os.path.join(INCLUDE, "fp8imma", "imma_fp8.h")]):
        return out
    inc = ce.include_paths() + [os.path.join(CUDA_HOME, "include"), INCLUDE, sysconfig.get_paths()["include"]]
    libdirs = ce.library_paths() + [HERE]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O3", "-shared", "-fPIC", "-std=c++17", "-DTORCH_EXTENSION_NAME=" + name,
           "-DTORCH_API_INCLUDE_EXTENSION_H", "-D_GLIBCXX_USE_CXX11_ABI=%d" % abi]
    cmd += ["-I" + p for p in inc] + srcs + ["-o", out]
    cmd += ["-L" + p for p in libdirs]
    cmd += ["-lfp8imma", "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda", "-ltorch_cuda",
            "-L" + os.path.join(CUDA_HOME, "lib64"), "-lcudart"]
    cmd += ["-Wl,-rpath,$ORIGIN"] + ["-Wl,-rpath," + p for p in ce.library_paths()]
    _run(cmd)
    return out


def build_all(force: bool = False) -> None:
    build_lib(force=force)
    with cf.ThreadPoolExecutor(max_workers=2) as ex:
        futs = [ex.submit(_torch_ext, "fp8imma_ext", ["fp8imma_ext.cpp"], force),
                ex.submit(_torch_ext, "fp8wgt_ext", ["fp8wgt_ext.cpp"], force)]
        for f in futs:
            f.result()


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
    print("built", LIB)
