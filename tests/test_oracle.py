"""CPU tests of the oracle (test infrastructure) against the reference's own
known answers: its host-built E4M3 table, and outputs of the reference library
itself (tests/golden/ref_*.npz, produced by tests/golden/make_ref_golden.py on
a B200 from the reference sources compiled for sm_100a)."""
import glob
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_lut_matches_reference_host_table():
    gold = np.array([int(l.split()[1], 16) for l in open(os.path.join(GOLDEN, "lut_e4m3_ref.txt"))], np.uint16)
    assert gold.shape == (256,)
    assert (O.lut_e4m3_ref() == gold).all()


def test_lut_exponent15_semantics():
    lut = O.lut_e4m3_ref()
    assert lut[0x78] == 0x7C00 and lut[0xF8] == 0xFC00       # +-Inf
    for b in list(range(0x79, 0x80)) + list(range(0xF9, 0x100)):
        assert (lut[b] & 0x7C00) == 0x7C00 and (lut[b] & 0x3FF) != 0  # NaN
    assert lut[0x77] == np.float16(240.0).view(np.uint16)
    assert lut[0x01] == np.float16(2.0 ** -9).view(np.uint16)


def test_lut_e5m2_is_high_byte():
    lut = O.lut_e5m2()
    for b in range(256):
        assert lut[b] == b << 8


def test_f32_to_f16_matches_numpy():
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(20000) * 10.0 ** rng.integers(-9, 6, 20000)).astype(np.float32)
    x = np.concatenate([x, np.array([65504, 65519.99, 65520, 2 ** -25, 2 ** -24, 3 * 2 ** -26, -0.0, np.inf, -np.inf], np.float32)])
    with np.errstate(over="ignore"):
        ref = x.astype(np.float16).view(np.uint16)
    mine = np.array([O.f32_to_f16_bits(v) for v in x], np.uint16)
    assert (mine == ref).all()


@pytest.mark.parametrize("v,q", [(0.5, 0), (1.5, 2), (2.5, 2), (-0.5, 0), (-1.5, -2), (126.5, 126), (127.5, 127),
                                  (200.0, 127), (-128.5, -128), (-300.0, -128), (float("inf"), 127),
                                  (float("-inf"), -128), (float("nan"), 0), (0.49951171875, 0)])
def test_cvt_rni_sat_s8(v, q):
    bits = int(np.float16(v).view(np.uint16))
    assert O.cvt_rni_sat_s8_f16(bits) == q


def test_hmul_is_fp16_rounded_product():
    rng = np.random.default_rng(1)
    a = rng.standard_normal(5000).astype(np.float16)
    b = (rng.standard_normal(5000) * 100).astype(np.float16)
    ref = (a.astype(np.float32) * b.astype(np.float32)).astype(np.float16).view(np.uint16)
    mine = np.array([O.hmul_bits(int(x), int(y)) for x, y in zip(a.view(np.uint16), b.view(np.uint16))], np.uint16)
    assert (mine == ref).all()


def test_inv_scale_rule():
    # |s| <= 1e-8 -> 0 ; fp16 Inf for tiny-but-larger scales
    assert O.inv_scale_bits(0) == 0
    assert O.inv_scale_bits(int(np.float16(2.0).view(np.uint16))) == int(np.float16(0.5).view(np.uint16))
    assert O.inv_scale_bits(int(np.float16(6e-8).view(np.uint16))) == 0x7C00
    nan_bits = 0x7E00
    assert O.inv_scale_bits(nan_bits) == 0


def test_encoders_match_torch():
    import torch

    rng = np.random.default_rng(2)
    v = (rng.standard_normal(50000) * 100).astype(np.float32)
    v = np.clip(v, -448, 448)
    t = torch.from_numpy(v).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert (O.e4m3fn_encode(v) == t).all()
    v5 = (rng.standard_normal(50000) * 1000).astype(np.float32)
    t5 = torch.from_numpy(v5).to(torch.float8_e5m2).view(torch.uint8).numpy()
    assert (O.e5m2_encode(v5) == t5).all()


def test_k_tail_group_semantics():
    # v4 reads activations in groups of 8: a partial trailing group is zero
    rng = np.random.default_rng(3)
    M, N, K = 3, 5, 20
    A = (rng.standard_normal((M, K))).astype(np.float16).view(np.uint16)
    B = rng.integers(0, 0x70, (N, K), dtype=np.uint8)
    s = np.full(N, np.float16(1.0)).view(np.uint16)
    _, _, acc8 = O.imma_fp8("v4_f16", 32, A, B, s, 1.0, 8.0)
    _, _, acc16 = O.imma_fp8("v3_f16", 32, A, B, s, 1.0, 8.0)
    Aq = O.quant_a(A, O.f32_to_f16_bits(8.0), group=1)
    Bq = O.transcode_b(B, s)
    assert (acc8 == O.gemm_s8(Aq, Bq, keff=16)).all()
    assert (acc16 == O.gemm_s8(Aq, Bq, keff=16)).all()
    _, _, acc8b = O.imma_fp8("v4_f16", 32, A[:, :16].copy(), B[:, :16].copy(), s, 1.0, 8.0)
    assert (acc8 == acc8b).all()


def test_invalid_kchunk():
    A = np.zeros((16, 16), np.uint16)
    B = np.zeros((16, 16), np.uint8)
    s = np.zeros(16, np.uint16)
    err, _, _ = O.imma_fp8("v4_f16", 48, A, B, s, 1.0, 1.0)
    assert err == 1


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "ref_*.npz"))) or [None])
def test_oracle_matches_reference_library_outputs(path):
    """Golden vectors: outputs of the reference library (WMMA, sm_100a build)."""
    if path is None:
        pytest.skip("no reference-library golden vectors generated yet")
    z = np.load(path)
    variant = str(z["variant"])
    kc = int(z["kchunk"])
    A = z["A"]
    err, D, _ = O.imma_fp8(variant, kc, A, z["B"], z["scales"], float(z["gs"]), float(z["ainv"]))
    assert err == 0
    from helpers import bits_equal

    eq = bits_equal(D, z["D"])
    assert eq.all(), "%s: %d mismatches" % (os.path.basename(path), (~eq).sum())
