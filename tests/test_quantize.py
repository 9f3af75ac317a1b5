"""Weight quantiser (fp8imma_quantize_weights): the CPU restatement is pinned
against torch's own float8 conversions on the recipe the benchmarks use
(workloads.make_weights), and the GPU kernel must equal the restatement bit
for bit (bytes, fp32 column scales, fp16 int8-step scales) in every format."""
import numpy as np
import pytest
import torch

from oracle import oracle as O


def _weights(N, K, seed, scale=0.02):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((N, K)) * scale).astype(np.float32)
    W[0] = 0.0                       # an all-zero column
    W[1, :] = 0.0
    W[1, 3] = 7.5                    # a single-spike column
    W[2] *= 1e-6                     # a tiny-scale column
    return W


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_oracle_matches_torch_float8_recipe(fmt):
    W = _weights(64, 300, seed=1)
    B, sigma, step = O.quantize_weights(W, fmt)
    w = torch.from_numpy(W)
    fmax = 448.0 if fmt == "e4m3" else 57344.0
    absmax = w.abs().amax(dim=1).clamp_min(1e-30)
    sig = absmax / fmax
    x = (w / sig[:, None]).clamp(-fmax, fmax)
    q = x.to(torch.float8_e4m3fn if fmt == "e4m3" else torch.float8_e5m2)
    assert np.array_equal(sigma, sig.numpy())
    assert np.array_equal(B, q.view(torch.uint8).numpy())
    st = (q.float().abs().amax(dim=1) / 127.0).to(torch.float16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(step, st)


def test_oracle_reference_range_has_no_exponent_15_codes():
    W = _weights(32, 256, seed=2)
    B, sigma, _ = O.quantize_weights(W, "e4m3_ref")
    assert ((B & 0x78) != 0x78).all()
    assert (np.abs(O.e4m3fn_decode(B)) <= 240.0).all()


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["e4m3", "e5m2", "e4m3_ref"])
@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("N,K", [(96, 1000), (7, 4096), (300, 33)])
def test_gpu_quantiser_bitexact(cuda, fmt, dtype, N, K):
    import fp8imma_b200 as F

    W = _weights(N, K, seed=N + K)
    tw = torch.from_numpy(W).to(getattr(torch, dtype))
    Wq = tw.float().numpy()  # the values the kernel sees
    B_o, s_o, st_o = O.quantize_weights(Wq, fmt)
    B, s, st = F.ext().quantize_weights(tw.cuda(), fmt)
    torch.cuda.synchronize()
    assert np.array_equal(B.cpu().numpy(), B_o)
    assert np.array_equal(s.cpu().numpy(), s_o)
    assert np.array_equal(st.cpu().numpy().view(np.uint16), st_o)


@pytest.mark.gpu
def test_gpu_quantiser_feeds_the_gemm(cuda):
    """Quantised weights + step scales through the reference API equal the
    oracle GEMM on the same bytes."""
    import fp8imma_b200 as F
    from helpers import bits_equal, to_np_bits

    rng = np.random.default_rng(5)
    W = (rng.standard_normal((256, 512)) * 0.02).astype(np.float32)
    B, _, st = F.ext().quantize_weights(torch.from_numpy(W).cuda(), "e4m3_ref")
    A = (rng.standard_normal((16, 512))).astype(np.float16)
    D = F.ext().imma_fp8_v4_act(torch.from_numpy(A).cuda(), B, st.view(torch.float16), 0.25, 4.0, 32)
    torch.cuda.synchronize()
    _, D_o, _ = O.imma_fp8("v4_f16", 32, A.view(np.uint16), B.cpu().numpy(), st.cpu().numpy().view(np.uint16),
                           0.25, 4.0)
    assert bits_equal(to_np_bits(D), D_o).all()


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_oracle_decoders_match_torch_on_all_codes(fmt):
    codes = np.arange(256, dtype=np.uint8)
    t = torch.from_numpy(codes).view(torch.float8_e4m3fn if fmt == "e4m3" else torch.float8_e5m2).float().numpy()
    o = O.e4m3fn_decode(codes) if fmt == "e4m3" else O.e5m2_decode(codes)
    nan = np.isnan(t)
    assert (np.isnan(o) == nan).all()
    assert np.array_equal(o[~nan], t[~nan])
    # encode(decode(b)) == b for every finite code (satfinite encoders map +-Inf to the largest finite)
    fin = np.isfinite(o)
    enc = O.e4m3fn_encode(o[fin]) if fmt == "e4m3" else O.e5m2_encode(o[fin])
    assert np.array_equal(enc, codes[fin])
