"""Generate golden vectors from the reference library itself.

Runs on a CUDA machine: loads oracle/_ref/libfp8imma_ref.so (the reference
fp8imma sources compiled for sm_100a by `make -C oracle ref`), calls its C ABI
on small seeded inputs and writes tests/golden/ref_<case>.npz with the inputs
and the reference output. tests/test_oracle.py checks the CPU oracle against
these files without a GPU.

    python tests/golden/make_ref_golden.py [outdir]
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "cuda-fp8-ampere_b200"))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from test_gpu_parity import REF_FUNCS, np_inputs, to_dev  # noqa: E402
from test_gpu_vs_reference_lib import run_ref  # noqa: E402
import reflib  # noqa: E402

CASES = [
    ("v4_f16", 16, 64, 128, "normal", "uniform", 32),
    ("v4_f16", 20, 80, 256, "special", "all", 64),
    ("v4_bf16", 8, 48, 512, "normal", "all", 32),
    ("v3_f16", 33, 64, 64, "normal", "uniform", 64),
    ("v3_bf16", 5, 32, 96, "special", "uniform", 32),
    ("v2", 16, 32, 128, "normal", "all", 32),
    ("v2_i8lut", 16, 32, 128, "normal", "uniform", 32),
    ("v4_f16", 1, 256, 512, "normal", "uniform", 32),
]


def main(outdir):
    os.makedirs(outdir, exist_ok=True)
    torch.cuda.set_device(0)
    reflib.lib().fp8imma_init_fp8_e4m3_lut()
    for i, (variant, M, N, K, sm, codes, kc) in enumerate(CASES):
        A, B, s = np_inputs(variant, M, N, K, seed=100 + i, scale_mode=sm, codes=codes)
        dA, dB, ds = to_dev(A, B, s, variant)
        ainv = None if variant.startswith("v2") else 6.0
        D = run_ref(REF_FUNCS[variant], kc, dA, dB, ds, M, N, K, 0.125, ainv)
        torch.cuda.synchronize()
        Dn = D.cpu().view(torch.int16).numpy().view(np.uint16)
        np.savez_compressed(os.path.join(outdir, "ref_%02d_%s_%dx%dx%d.npz" % (i, variant, M, N, K)),
                            variant=variant, kchunk=kc, A=A, B=B, scales=s, gs=np.float32(0.125),
                            ainv=np.float32(ainv if ainv is not None else 1.0), D=Dn)
    print("wrote", len(CASES), "golden files to", outdir)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else HERE)
