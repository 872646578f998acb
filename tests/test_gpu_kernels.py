"""Dequant-matvec and decode kernels vs the oracle and the reference's own
outputs (tests/golden/ref_vectors.npz), through the C ABI.

Tolerances: dequantised values bit-exact; single matvecs within 1e-4 of
max |y| (fp32 reassociation only; observed ~1e-6); the BASELINE bound for
expert-chain outputs is 2e-3 (test_gpu_moe.py).
"""
import ctypes as C
import os

import numpy as np
import pytest

from oracle import pyoracle as po
from tests._lib import ds4f_cuda

pytestmark = pytest.mark.gpu
dc = ds4f_cuda()
GOLD = os.path.join(os.path.dirname(__file__), "golden", "ref_vectors.npz")
MV_TOL = 1e-4


@pytest.fixture(scope="module", autouse=True)
def gpu():
    dc.init()
    yield


@pytest.fixture(scope="module")
def g():
    return np.load(GOLD)


def relerr(a, b):
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30))


def bits_eq(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    same = a.view(np.uint32) == b.view(np.uint32)
    return bool(np.all(same | (np.isnan(a) & np.isnan(b))))


def xvec(n, seed=1):
    return po.fill_f32(n, po.key(seed, 0, 4, 0, 0), 1.0)


@pytest.mark.parametrize("R,Cc", [(512, 2048), (2048, 512), (128, 128), (256, 4096)])
def test_f8_matvec_fp32_scales(R, Cc):
    W, s = po.quant_fp8(R, Cc, po.key(7, 0, 3, R, Cc), 0.02)
    x = xvec(Cc)
    y = dc.f8_matvec(W, dc.SCALE_F32, s, R // 128, Cc // 128, x)
    ref = po.f8_matvec(W, po.SCALE_F32, s, R // 128, Cc // 128, x)
    assert relerr(y, ref) < MV_TOL


@pytest.mark.parametrize("name", ["a", "b", "c"])
def test_f8_matvec_vs_reference_output(g, name):
    """E8M0 block scales and edge-heavy bytes (subnormals, every e=15 byte):
    against the reference's own ds4f_f8_matvec output. Shape c (130 x 200)
    takes the any-shape path."""
    r, c, sr, sc = (int(v) for v in g[f"f8mv_{name}_shape"])
    y = dc.f8_matvec(g[f"f8mv_{name}_W"], dc.SCALE_E8M0, g[f"f8mv_{name}_S"], sr, sc,
                     g[f"f8mv_{name}_x"])
    assert relerr(y, g[f"f8mv_{name}_y"]) < MV_TOL


def test_mxfp4_matvec_vs_reference_output(g):
    r, c = (int(v) for v in g["mxmv_shape"])
    y = dc.mxfp4_matvec(g["mxmv_V"], g["mxmv_S"], r, c, g["mxmv_x"])
    assert relerr(y, g["mxmv_y"]) < MV_TOL


@pytest.mark.parametrize("R,Cc,bsize", [(512, 2048, 32), (2048, 512, 32), (40, 96, 16),
                                        (7, 40, 16)])
def test_mxfp4_matvec_fixture(R, Cc, bsize):
    if bsize == 32:
        v, s = po.quant_mxfp4(R, Cc, po.key(9, 0, 3, R, Cc), 0.02)
    else:
        rng = np.random.default_rng(R)
        v = rng.integers(0, 256, R * Cc // 2, dtype=np.uint16).astype(np.uint8)
        s = rng.integers(118, 130, (R * Cc + bsize - 1) // bsize, dtype=np.uint16).astype(np.uint8)
    x = xvec(Cc)
    y = dc.mxfp4_matvec(v, s, R, Cc, x, bsize)
    assert relerr(y, po.mxfp4_matvec(v, s, R, Cc, x, bsize)) < MV_TOL


def test_bf16_matvec_vs_reference_output(g):
    assert relerr(dc.bf16_matvec(g["bfmv_W"], g["bfmv_x"]), g["bfmv_y"]) < MV_TOL
    assert relerr(dc.bf16_matvec(g["bfmv_W"], g["bfmv_x"], g["bfmv_bias"]),
                  g["bfmv_yb"]) < MV_TOL


def test_bf16_router_shape():
    W = po.fill_bf16(256 * 2048, po.key(0, 0, 1, 0, 0), 0.02).reshape(256, 2048)
    x = xvec(2048)
    assert relerr(dc.bf16_matvec(W, x), po.bf16_matvec(W, x)) < MV_TOL


def test_mlx4_matvec_vs_reference_output(g):
    y = dc.mlx4_matvec(g["mlx_V"], g["mlx_S"], g["mlx_B"], 16, 256, g["mlx_x"])
    assert relerr(y, g["mlx_y"]) < MV_TOL
    y0 = dc.mlx4_matvec(g["mlx_V"], g["mlx_S"], None, 16, 256, g["mlx_x"])
    assert relerr(y0, g["mlx_y0"]) < MV_TOL


def test_mlx4_batch_arena_by_id():
    """gpu.h:39-52: weights are cached per stable id; a second call with the
    same ids reuses the first upload even if the host pointer changed."""
    rng = np.random.default_rng(3)
    R, Cc, nj = 64, 512, 4
    vals = [rng.integers(0, 2**32, R * Cc // 8, dtype=np.uint64).astype(np.uint32) for _ in range(nj)]
    sc = [((rng.random(R * Cc // 64) * 0.02 + 0.001).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16) for _ in range(nj)]
    bi = [((rng.standard_normal(R * Cc // 64) * 0.02).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16) for _ in range(nj)]
    xs = [xvec(Cc, 10 + j) for j in range(nj)]
    ys = [np.zeros(R, np.float32) for _ in range(nj)]
    ids = [C.c_void_p(0x1000 + 16 * j) for j in range(nj)]

    def arr(lst):
        return (C.c_void_p * nj)(*[a.ctypes.data for a in lst])

    L = dc.lib()
    dc.check(L.ds4f_gpu_mlx4_batch(arr(vals), arr(sc), arr(bi), arr(xs), arr(ys),
                                   (C.c_void_p * nj)(*ids), R, Cc, nj))
    for j in range(nj):
        assert relerr(ys[j], po.mlx4_matvec(vals[j], sc[j], bi[j], R, Cc, xs[j])) < MV_TOL
    first = [y.copy() for y in ys]
    vals2 = [np.zeros_like(v) for v in vals]          # same ids, new bytes: cached
    dc.check(L.ds4f_gpu_mlx4_batch(arr(vals2), arr(sc), arr(bi), arr(xs), arr(ys),
                                   (C.c_void_p * nj)(*ids), R, Cc, nj))
    for j in range(nj):
        assert np.array_equal(first[j], ys[j])


def test_f8_decode_bit_exact_all_bytes():
    W = np.arange(256 * 4, dtype=np.uint32).astype(np.uint8).reshape(8, 128)
    for kind, S in ((dc.SCALE_E8M0, np.array([0, 1, 126, 127, 128, 200, 254, 255], np.uint8)),
                    (dc.SCALE_F32, np.array([1.0, 2.5e-4, 3e-39, 1e30, -0.5, 7.0, 1.0, 0.1],
                                            np.float32))):
        out = dc.f8_decode_rows(W, kind, S, 8, 1, 0, 8)
        ref = np.zeros((8, 128), np.float32)
        po.lib().orc_f8_decode_rows(po.ptr(W), kind, po.ptr(S), 8, 128, 8, 1, 0, 8, po.ptr(ref))
        assert bits_eq(out, ref)
        part = dc.f8_decode_rows(W, kind, S, 8, 1, 3, 6)
        assert bits_eq(part, ref[3:6])


def test_f8_decode_vs_reference_rows(g):
    for name in ("a", "b", "c"):
        r, c, sr, sc = (int(v) for v in g[f"f8mv_{name}_shape"])
        out = dc.f8_decode_rows(g[f"f8mv_{name}_W"], dc.SCALE_E8M0, g[f"f8mv_{name}_S"], sr, sc,
                                0, r)
        for k, row in enumerate((0, r // 2, r - 1)):
            assert bits_eq(out[row], g[f"f8mv_{name}_rows"][k])


def test_mxfp4_decode_bit_exact(g):
    out = dc.mxfp4_decode(g["mxdec_vals"], g["mxdec_scales"], 512, 32)
    assert bits_eq(out, g["mxdec_out"])
    rng = np.random.default_rng(11)
    v = rng.integers(0, 256, 4096, dtype=np.uint16).astype(np.uint8)
    s = rng.integers(0, 256, 8192 // 16, dtype=np.uint16).astype(np.uint8)
    ref = np.zeros(8192, np.float32)
    po.lib().orc_mxfp4_decode(po.ptr(v), po.ptr(s), 8192, 16, po.ptr(ref))
    assert bits_eq(dc.mxfp4_decode(v, s, 8192, 16), ref)


@pytest.mark.parametrize("fmt", [dc.FMT_FP8, dc.FMT_MXFP4])
def test_gpu_generator_matches_cpu_generator(fmt):
    H, M, E = 1024, 256, 3
    m = dc.Model(fmt, 2, H, M, E, 2)
    m.synth(5)
    lay = po.Layer(fmt, H, M, E, seed=5, layer=1)
    tr = m.get_trunk(1)
    for a, b in zip(tr, (lay.norm, lay.router, lay.sh_gate, lay.sh_up, lay.sh_down, lay.sh_gw)):
        assert np.array_equal(a.reshape(-1), b.reshape(-1))
    for x in range(E):
        assert np.array_equal(m.get_expert(1, x), lay.experts[x])
    m.close()


def test_mv_plan_config1_microbench():
    """Config 1: 8 experts x (gate, up, down) FP8 + MXFP4 as device jobs in
    one launch each, against the oracle per job."""
    import torch
    jobs_f8, jobs_mx, refs, keep = [], [], [], []
    for e in range(8):
        for t, (R, Cc) in enumerate(((512, 2048), (512, 2048), (2048, 512))):
            k = po.key(1, 0, 3, e, t)
            x = xvec(Cc, 100 + e)
            W, s = po.quant_fp8(R, Cc, k, 0.02)
            v, sm = po.quant_mxfp4(R, Cc, k, 0.02)
            tW, ts, tv, tsm, tx = (torch.from_numpy(a).cuda() for a in (W, s, v, sm, x))
            ty8 = torch.zeros(R, device="cuda")
            tym = torch.zeros(R, device="cuda")
            keep += [tW, ts, tv, tsm, tx, ty8, tym]
            jobs_f8.append(dc.Ds4fMvJob(tW.data_ptr(), ts.data_ptr(), tx.data_ptr(),
                                        ty8.data_ptr(), R, Cc, R // 128, Cc // 128,
                                        dc.FMT_FP8, dc.SCALE_F32, 32, 1))
            jobs_mx.append(dc.Ds4fMvJob(tv.data_ptr(), tsm.data_ptr(), tx.data_ptr(),
                                        tym.data_ptr(), R, Cc, 1, 1, dc.FMT_MXFP4, 0, 32, 0))
            refs.append((po.f8_matvec(W, po.SCALE_F32, s, R // 128, Cc // 128, x),
                         po.mxfp4_matvec(v, sm, R, Cc, x), ty8, tym))
    for jobs in (jobs_f8, jobs_mx):
        p = dc.MvPlan(jobs)
        p.run(C.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    for r8, rm, ty8, tym in refs:
        assert relerr(ty8.cpu().numpy(), r8) < MV_TOL
        assert relerr(tym.cpu().numpy(), rm) < MV_TOL


def test_mv_plan_stream_kernel_shapes_and_formats():
    """Job lists through the TMA stream kernel (expert-shaped jobs) and the
    job kernel (the rest) in one plan, run twice: FP8 with E8M0 block scales
    and raw bytes (e=15 canonicalised in-kernel), FP8 with fp32 scales, MXFP4,
    BF16 with and without bias; odd row counts; 64 MB of FP8 rows so that
    every CTA's ring of copy slots wraps its phase; a 96-column job that the
    stream kernel does not take."""
    import torch
    rng = np.random.default_rng(5)
    jobs, checks, keep = [], [], []

    def dev(a):
        t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
        keep.append(t)
        return t

    def add(fmt, W, s, x, R, Cc, SR, SC, kind, canon, ref):
        tW, tx = dev(W), dev(x)
        ts = dev(s) if s is not None else None
        ty = torch.zeros(R, device="cuda")
        keep.append(ty)
        jobs.append(dc.Ds4fMvJob(tW.data_ptr(), ts.data_ptr() if ts is not None else 0, tx.data_ptr(),
                                 ty.data_ptr(), R, Cc, SR, SC, fmt, kind, 32, canon))
        checks.append((ty, ref))

    for (R, Cc) in ((100, 2048), (300, 512), (2048, 128), (640, 384)):
        W = rng.integers(0, 256, (R, Cc), dtype=np.uint8)            # e=15 bytes included
        SR, SC = max(1, R // 128), Cc // 128
        s8 = rng.integers(110, 125, (SR, SC), dtype=np.uint8)
        x = xvec(Cc, R)
        add(dc.FMT_FP8, W, s8, x, R, Cc, SR, SC, dc.SCALE_E8M0, 1,
            po.f8_matvec(W, po.SCALE_E8M0, s8, SR, SC, x))
    for (R, Cc) in ((4096, 2048),) * 8:                                 # 64 MB
        k = po.key(2, 0, 3, len(jobs), 0)
        W, s = po.quant_fp8(R, Cc, k, 0.02)
        x = xvec(Cc, len(jobs) + 7)
        add(dc.FMT_FP8, W, s, x, R, Cc, R // 128, Cc // 128, dc.SCALE_F32, 0,
            po.f8_matvec(W, po.SCALE_F32, s, R // 128, Cc // 128, x))
    for (R, Cc) in ((333, 1024), (2048, 512)):
        v, sm = po.quant_mxfp4(R, Cc, po.key(3, 0, 3, R, 0), 0.02)
        x = xvec(Cc, 11)
        add(dc.FMT_MXFP4, v, sm, x, R, Cc, 1, 1, 0, 0, po.mxfp4_matvec(v, sm, R, Cc, x))
    for (R, Cc, bias) in ((256, 2048, False), (2048, 512, True), (77, 256, True)):
        W = (rng.standard_normal((R, Cc), dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)
        b = rng.standard_normal(R).astype(np.float32) if bias else None
        x = xvec(Cc, 13)
        add(3, W, b, x, R, Cc, 1, 1, 0, 0, po.bf16_matvec(W, x, b))
    W = rng.integers(0, 120, (64, 96), dtype=np.uint8)                   # job kernel, not streamed
    x = xvec(96, 17)
    add(dc.FMT_FP8, W, None, x, 64, 96, 1, 1, dc.SCALE_F32, 0, po.f8_matvec(W, po.SCALE_F32, None, 1, 1, x))
    p = dc.MvPlan(jobs)
    sp = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(2):
        for ty, _ in checks:
            ty.fill_(float("nan"))
        p.run(sp)
        torch.cuda.synchronize()
        for i, (ty, ref) in enumerate(checks):
            assert relerr(ty.cpu().numpy(), ref) < MV_TOL, i
    del p


def test_bad_arguments_fail_loudly():
    with pytest.raises(dc.GpuError, match="bsize"):
        dc.mxfp4_matvec(np.zeros(8, np.uint8), np.zeros(1, np.uint8), 1, 16, np.zeros(16, np.float32), 8)
    with pytest.raises(dc.GpuError):
        dc.Model(dc.FMT_FP8, 1, 3000, 512, 256, 8)
