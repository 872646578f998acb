"""Tensor-core building blocks of the batched prefill, through the C ABI:
the activation quantiser (bit-exact against oracle/prefill.c) and the
block-scaled FP8 digit GEMM (tcgen05; against the oracle's double-precision
restatement, and against the unquantised fp32 product within the BASELINE
chain tolerance).

Tolerances: quantiser bytes and scales bit-exact; GEMM vs its own restated
arithmetic within 1e-5 of max |Y| (fp32 accumulation order only); GEMM with
3 digits vs the unquantised activations within 2e-3 (the BASELINE bound for
chain outputs; the digits' representation error is <= 2^-13).
"""
import numpy as np
import pytest

from oracle import pyoracle as po
from tests._lib import ds4f_cuda

pytestmark = pytest.mark.gpu
dc = ds4f_cuda()
GEMM_TOL = 1e-5
CHAIN_TOL = 2e-3


@pytest.fixture(scope="module", autouse=True)
def gpu():
    dc.init()
    yield


def _acts(N, Cc, seed):
    x = po.fill_f32(N * Cc, po.key(seed, 0, 4, 0, 0), 1.0).reshape(N, Cc)
    if N >= 4:
        x[1, :128] = 0.0                       # all-zero block: scale 1, digits 0
        x[2, :] *= 1e-30                       # tiny (subnormal E4M3 digits)
        x[3, 5] = -0.0
        x[3, 7] = 3.0e4                        # one large element per block
    return x


@pytest.mark.parametrize("nd", [1, 2, 3])
def test_quant_digits_bit_exact(nd):
    import torch
    N, Cc = 37, 512
    x = _acts(N, Cc, 3)
    q_ref, s_ref = po.quant_f8_digits(x, nd)
    xg = torch.from_numpy(x).cuda()
    q = torch.empty((nd, N, Cc), dtype=torch.uint8, device="cuda")
    s = torch.empty((N, Cc // 128), dtype=torch.float32, device="cuda")
    dc.quant_f8_digits_dev(xg, q, s, nd)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))
    assert np.array_equal(q.cpu().numpy(), q_ref)


@pytest.mark.parametrize("R,Cc,N", [(128, 128, 1), (256, 512, 100), (512, 2048, 64), (2048, 512, 130)])
def test_f8_gemm_matches_restated_arithmetic(R, Cc, N):
    import torch
    W, sW = po.quant_fp8(R, Cc, po.key(11, 0, 3, 0, 0), 0.02)
    x = _acts(N, Cc, 12)
    q, sx = po.quant_f8_digits(x, 3)
    want = po.f8_gemm_digits(W, sW, q, sx)
    Y = torch.zeros((N, R), dtype=torch.float32, device="cuda")
    dc.f8_gemm_dev(torch.from_numpy(W).cuda(), torch.from_numpy(sW).cuda(), torch.from_numpy(q).cuda(),
                   torch.from_numpy(sx).cuda(), Y)
    got = Y.cpu().numpy().astype(np.float64)
    err = np.abs(got - want).max() / np.abs(want).max()
    assert err < GEMM_TOL, err
    # against the unquantised activations (the reference's fp32 x)
    Wd = np.array([po.lib().orc_f8_value(int(b)) for b in range(256)], np.float64)[W]
    Wd *= np.repeat(np.repeat(sW.astype(np.float64), 128, 0), 128, 1)
    exact = x.astype(np.float64) @ Wd.T
    err2 = np.abs(got - exact).max() / np.abs(exact).max()
    assert err2 < CHAIN_TOL, err2


def test_f8_gemm_single_digit_is_coarse_but_consistent():
    import torch
    R, Cc, N = 256, 256, 48
    W, sW = po.quant_fp8(R, Cc, po.key(13, 0, 3, 0, 0), 0.02)
    x = _acts(N, Cc, 14)
    q, sx = po.quant_f8_digits(x, 1)
    want = po.f8_gemm_digits(W, sW, q, sx)
    Y = torch.zeros((N, R), dtype=torch.float32, device="cuda")
    dc.f8_gemm_dev(torch.from_numpy(W).cuda(), torch.from_numpy(sW).cuda(), torch.from_numpy(q).cuda(),
                   torch.from_numpy(sx).cuda(), Y)
    got = Y.cpu().numpy().astype(np.float64)
    assert np.abs(got - want).max() / np.abs(want).max() < GEMM_TOL


def test_f8_gemm_rejects_bad_shapes():
    import torch
    W = torch.zeros((100, 128), dtype=torch.uint8, device="cuda")
    sW = torch.zeros((1, 1), dtype=torch.float32, device="cuda")
    q = torch.zeros((3, 4, 128), dtype=torch.uint8, device="cuda")
    sx = torch.zeros((4, 1), dtype=torch.float32, device="cuda")
    Y = torch.zeros((4, 100), dtype=torch.float32, device="cuda")
    with pytest.raises(dc.GpuError, match="multiples of 128"):
        dc.f8_gemm_dev(W, sW, q, sx, Y)
