"""The output head (ds4f_gpu_head_*, the step after the MoE path): logits
against the oracle's matvec for the reference head's FP8 (E8M0 blocks), BF16
and MLX4 forms (src/head.c:243-299), and the greedy pick bit-exact against
the reference rule (ds4f_argmax, src/head.c:303-309; oracle po.argmax)
including ties, NaN and infinities."""
import ctypes as C

import numpy as np
import pytest

from oracle import pyoracle as po
from tests._lib import ds4f_cuda

pytestmark = pytest.mark.gpu
dc = ds4f_cuda()
MV_TOL = 1e-4


@pytest.fixture(scope="module", autouse=True)
def gpu():
    dc.init()
    yield


def relerr(a, b):
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30))


def bf16(a):
    return (np.asarray(a, np.float32).view(np.uint32) >> 16).astype(np.uint16)


@pytest.mark.parametrize("V", [50_021, 248_320])
def test_bf16_head(V):
    H = 2048
    rng = np.random.default_rng(V)
    W = bf16(rng.standard_normal((V, H)) * 0.02)
    x = rng.standard_normal(H).astype(np.float32)
    hd = dc.Head(dc.HEAD_BF16, W, V=V, H=H)
    y, best = hd.logits(x)
    ref = po.bf16_matvec(W, x)
    assert relerr(y, ref) < MV_TOL
    assert best == po.argmax(y)                 # the pick of the logits it returned
    _, best2 = hd.logits(x, want_logits=False)
    assert best2 == best
    # the device-pointer call on torch's stream: same logits, same pick
    import torch
    tx = torch.from_numpy(x).cuda()
    ty = torch.zeros(V, device="cuda")
    tb = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    hd.logits_dev(tx, ty, tb, C.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert np.array_equal(ty.cpu().numpy(), y) and int(tb.item()) == best
    hd.close()


def test_f8_head_e8m0_blocks():
    V, H = 4096 + 96, 2048
    rng = np.random.default_rng(1)
    W = rng.integers(0, 256, (V, H), dtype=np.uint8)          # every byte, e=15 included
    SR, SC = (V + 127) // 128, H // 128
    S = rng.integers(110, 125, (SR, SC), dtype=np.uint8)      # E8M0 2^-17 .. 2^-3
    x = rng.standard_normal(H).astype(np.float32)
    hd = dc.Head(dc.HEAD_F8, W, S, V=V, H=H, SR=SR, SC=SC)
    y, best = hd.logits(x)
    ref = po.f8_matvec(W, dc.SCALE_E8M0, S, SR, SC, x)
    assert relerr(y, ref) < MV_TOL
    assert best == po.argmax(y)
    hd.close()


def test_mlx4_head():
    V, H = 8192, 2048
    rng = np.random.default_rng(2)
    vals = rng.integers(0, 2**32, V * H // 8, dtype=np.uint64).astype(np.uint32)
    sc = bf16(rng.random(V * H // 64) * 0.02 + 0.001)
    bi = bf16(rng.standard_normal(V * H // 64) * 0.02)
    x = rng.standard_normal(H).astype(np.float32)
    hd = dc.Head(dc.HEAD_MLX4, vals, sc, bi, V=V, H=H)
    y, best = hd.logits(x)
    assert relerr(y, po.mlx4_matvec(vals, sc, bi, V, H, x)) < MV_TOL
    assert best == po.argmax(y)
    hd.close()


def test_unbuilt_head_dtypes_refused():
    with pytest.raises(dc.GpuError, match="not built"):
        dc.Head(0, np.zeros((4, 8), np.float32), V=4, H=8)


def _pick(arr):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(arr, np.float32)).cuda()
    out = torch.full((1,), -5, dtype=torch.int32, device="cuda")
    dc.argmax_dev(t, out)
    torch.cuda.synchronize()
    return int(out.item())


def test_argmax_rule_edge_cases():
    n = 248_320
    rng = np.random.default_rng(4)
    base = rng.standard_normal(n).astype(np.float32)
    cases = {}
    a = base.copy(); a[[5, 100_000, n - 1]] = 9.0; cases["tie: lowest index"] = a
    a = base.copy(); a[n - 1] = 9.0; cases["max at the end"] = a
    a = base.copy(); a[0] = np.nan; a[77] = 9.0; cases["NaN at 0 wins"] = a
    a = base.copy(); a[3] = np.nan; a[1:3] = 9.0; cases["NaN skipped"] = a
    a = base.copy(); a[::2] = np.nan; cases["half NaN"] = a
    cases["all equal"] = np.ones(n, np.float32)
    cases["all -inf"] = np.full(n, -np.inf, np.float32)
    a = np.full(n, -np.inf, np.float32); a[123_456] = np.inf; a[200_000] = np.inf; cases["+inf twice"] = a
    a = np.zeros(n, np.float32); a[0] = -0.0; a[10] = 0.0; cases["signed zeros tie"] = a
    a = np.full(n, np.nan, np.float32); cases["all NaN"] = a
    a = base.copy(); a[0] = -np.inf; a[1:] = np.nan; cases["-inf then NaN"] = a
    cases["one element"] = np.array([3.0], np.float32)
    cases["short"] = base[:1000].copy()
    for name, arr in cases.items():
        assert _pick(arr) == po.argmax(arr.tolist()), name
