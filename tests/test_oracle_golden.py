"""Pin the CPU oracle to the reference (no GPU).

1. Known-answer vectors of the reference's own gate test
   (tests/test_kernels.c:57-76, :79-137, :258-276), restated here.
2. tests/golden/ref_vectors.npz: outputs of the reference's own kernels,
   compiled in place (tests/golden/make_golden.py). Bit-exact.
3. When oracle/_ref is built, fresh seeded inputs against it directly.
"""
import ctypes as C
import math
import os

import numpy as np
import pytest

from oracle import pyoracle as po

GOLD = os.path.join(os.path.dirname(__file__), "golden", "ref_vectors.npz")


@pytest.fixture(scope="module")
def g():
    return np.load(GOLD)


@pytest.fixture(scope="module")
def L():
    return po.lib()


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


# ---- 1. the reference's known-answer tests ---------------------------

def test_e8m0_known(L):          # tests/test_kernels.c:57-60
    assert L.orc_e8m0_value(0) == math.ldexp(1.0, -127)
    assert L.orc_e8m0_value(127) == 1.0
    assert L.orc_e8m0_value(130) == 8.0
    assert math.isinf(L.orc_e8m0_value(255))


def test_mxfp4_decode_known(L):  # tests/test_kernels.c:63-76
    vals = np.array([0x07 | (0x03 << 4), 0x08], np.uint8)
    scales = np.array([127], np.uint8)
    out = np.zeros(4, np.float32)
    L.orc_mxfp4_decode(po.ptr(vals), po.ptr(scales), 4, 16, po.ptr(out))
    assert list(out) == [6.0, 1.5, 0.0, 0.0]


def _ref_test_encode(xs, bsize):
    """Encoder of tests/test_kernels.c:19-54 (nearest magnitude, strict <)."""
    mags = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    n = len(xs)
    nb = (n + bsize - 1) // bsize
    vals = np.zeros((n + 1) // 2, np.uint8)
    scales = np.zeros(nb, np.uint8)
    for bi in range(nb):
        blk = xs[bi * bsize:(bi + 1) * bsize]
        m = float(np.max(np.abs(blk))) if len(blk) else 0.0
        k = math.ceil(math.log2(m / 6.0)) if m > 0 else -127
        k = max(-127, min(127, k))
        scales[bi] = (k + 127) & 0xFF
        s = np.float32(math.ldexp(1.0, int(scales[bi]) - 127))
        for j, x in enumerate(blk):
            q = np.float32(x) / s if s else np.float32(0)
            a = abs(float(q))
            best, bd = 0, a
            for i in range(1, 8):
                d = abs(a - mags[i])
                if d < bd:
                    bd, best = d, i
            nib = (8 if q < 0 else 0) | best
            i = bi * bsize + j
            vals[i // 2] |= nib if i % 2 == 0 else nib << 4
    return vals, scales


def test_mxfp4_roundtrip(L):     # tests/test_kernels.c:79-101
    for bsize in (16, 32):
        n = 100
        xs = np.array([((i * 37 + 11) % 200 - 100) * 0.03 for i in range(n)],
                      np.float32)
        vals, scales = _ref_test_encode(xs, bsize)
        back = np.zeros(n, np.float32)
        L.orc_mxfp4_decode(po.ptr(vals), po.ptr(scales), n, bsize,
                           po.ptr(back))
        mags = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
        for i in range(n):
            nib = (vals[i // 2] >> (4 if i & 1 else 0)) & 0xF
            want = np.float32(mags[nib & 7]) * np.float32(
                math.ldexp(1.0, int(scales[i // bsize]) - 127))
            if nib & 8:
                want = -want
            assert back[i] == want


def test_mxfp4_matvec_vs_naive(L):   # tests/test_kernels.c:104-137
    R, Cc, bsize = 7, 40, 16
    W = np.array([((i * 13 + 5) % 240 - 120) * 0.02 for i in range(R * Cc)],
                 np.float32)
    x = np.array([((c * 7) % 9 - 4) * 0.1 for c in range(Cc)], np.float32)
    vals, scales = _ref_test_encode(W, bsize)
    scr = np.zeros(R * Cc, np.float32)
    L.orc_mxfp4_decode(po.ptr(vals), po.ptr(scales), R * Cc, bsize, po.ptr(scr))
    want = np.zeros(R, np.float32)
    for r in range(R):
        acc = np.float32(0)
        for c in range(Cc):
            acc = np.float32(acc + np.float32(scr[r * Cc + c] * x[c]))
        want[r] = acc
    got = po.mxfp4_matvec(vals, scales, R, Cc, x, bsize)
    assert np.array_equal(bits(got), bits(want))


def test_f8_known_bytes(L):      # tests/test_kernels.c:258-276
    W = np.array([0x38, 0xB8, 0x3C, 0xBC, 0x00, 0x38, 0xB8, 0x3C],
                 np.uint8).reshape(2, 4)
    S = np.array([127, 130], np.uint8)
    x = np.array([1, 2, 3, 4], np.float32)
    y = po.f8_matvec(W, po.SCALE_E8M0, S, 1, 2, x)
    assert list(y) == [-13.0, 26.0]
    # the same with fp32 block scales (the BASELINE scale format)
    y2 = po.f8_matvec(W, po.SCALE_F32, np.array([1.0, 8.0], np.float32), 1, 2, x)
    assert list(y2) == [-13.0, 26.0]


def test_f8_edge_bytes_glibc_rand(L):   # tests/test_kernels.c:319-355
    """The reference's edge-byte test inputs, regenerated with glibc
    srand(7)/rand() exactly as the test does; scalar oracle vs the
    reference scalar (bit-exact) and AVX2 (1e-3) when _ref is built."""
    libc = C.CDLL("libc.so.6")
    libc.srand(7)
    W = np.zeros(16 * 64, np.uint8)
    for i in range(16 * 64):
        v = libc.rand() % 256
        if i % 5 == 0:
            v &= 0x87
        if i % 7 == 0:
            v |= 0x78
        W[i] = v
    sc = np.array([117 + libc.rand() % 8 for _ in range(32)], np.uint8)
    x = np.array([(libc.rand() % 200) / 100.0 - 1.0 for _ in range(64)],
                 np.float32)
    W = W.reshape(16, 64)
    for SR, SC in ((1, 1), (2, 4)):
        y = po.f8_matvec(W, po.SCALE_E8M0, sc, SR, SC, x)
        R = po.ref()
        if R is None:
            continue
        ys = np.zeros(16, np.float32)
        R.ds4f_kernels_set_simd(0)
        R.ds4f_f8_matvec(po.ptr(W), po.ptr(sc), 16, 64, SR, SC, po.ptr(x),
                         po.ptr(ys))
        assert np.array_equal(bits(y), bits(ys))
        R.ds4f_kernels_set_simd(1)
        yv = np.zeros(16, np.float32)
        R.ds4f_f8_matvec(po.ptr(W), po.ptr(sc), 16, 64, SR, SC, po.ptr(x),
                         po.ptr(yv))
        R.ds4f_kernels_set_simd(0)
        assert np.all(np.abs(yv - ys) <= 1e-3 * (1 + np.abs(ys)))


# ---- 2. committed golden vectors from the reference's own kernels ----

def test_golden_lut(L, g):
    ours = np.array([L.orc_f8_value(b) for b in range(256)], np.float32)
    assert np.array_equal(bits(ours), bits(g["f8_lut"]))
    # the e=15 rule: every e=15 byte is +-448 (src/kernels.c:234-235)
    for b in range(256):
        if (b >> 3) & 0xF == 0xF:
            assert abs(ours[b]) == 448.0
    e8 = np.array([L.orc_e8m0_value(b) for b in range(256)], np.float32)
    assert np.array_equal(bits(e8), bits(g["e8m0"]))


def test_golden_mxfp4_decode(L, g):
    out = np.zeros(512, np.float32)
    L.orc_mxfp4_decode(po.ptr(g["mxdec_vals"]), po.ptr(g["mxdec_scales"]),
                       512, 32, po.ptr(out))
    assert np.array_equal(bits(out), bits(g["mxdec_out"]))


@pytest.mark.parametrize("name", ["a", "b", "c"])
def test_golden_f8_matvec(L, g, name):
    r, c, sr, sc = (int(v) for v in g[f"f8mv_{name}_shape"])
    W, S, x = g[f"f8mv_{name}_W"], g[f"f8mv_{name}_S"], g[f"f8mv_{name}_x"]
    y = po.f8_matvec(W, po.SCALE_E8M0, S, sr, sc, x)
    assert np.array_equal(bits(y), bits(g[f"f8mv_{name}_y"]))
    # the timed AVX2 baseline computes the same within lane-order tolerance
    ys = g[f"f8mv_{name}_y_simd"]
    assert np.all(np.abs(ys - y) <= 1e-3 * (1 + np.abs(y)))
    rows = g[f"f8mv_{name}_rows"]
    for k, row in enumerate((0, r // 2, r - 1)):
        o = np.zeros((1, c), np.float32)
        L.orc_f8_decode_rows(po.ptr(W), po.SCALE_E8M0, po.ptr(S), r, c, sr,
                             sc, row, row + 1, po.ptr(o))
        assert np.array_equal(bits(o[0]), bits(rows[k]))


def test_golden_mxfp4_matvec(g):
    r, c = (int(v) for v in g["mxmv_shape"])
    y = po.mxfp4_matvec(g["mxmv_V"], g["mxmv_S"], r, c, g["mxmv_x"])
    assert np.array_equal(bits(y), bits(g["mxmv_y"]))


def test_golden_bf16_matvec(g):
    y = po.bf16_matvec(g["bfmv_W"], g["bfmv_x"])
    assert np.array_equal(bits(y), bits(g["bfmv_y"]))
    yb = po.bf16_matvec(g["bfmv_W"], g["bfmv_x"], g["bfmv_bias"])
    assert np.array_equal(bits(yb), bits(g["bfmv_yb"]))


def test_golden_mlx4_matvec(g):
    V, S, B, x = g["mlx_V"], g["mlx_S"], g["mlx_B"], g["mlx_x"]
    r, c = 16, 256
    y = po.mlx4_matvec(V, S, B, r, c, x)
    assert np.array_equal(bits(y), bits(g["mlx_y"]))
    y0 = po.mlx4_matvec(V, S, None, r, c, x)
    assert np.array_equal(bits(y0), bits(g["mlx_y0"]))


def test_golden_topk(g):
    sc = g["topk_scores"]
    for t in range(sc.shape[0]):
        idx, w = po.topk(np.ascontiguousarray(sc[t]), 8)
        assert np.array_equal(idx, g["topk_idx"][t])
        assert np.array_equal(bits(w), bits(g["topk_w"][t]))
    # tie rule: among equal scores the lower index comes first
    for t in range(sc.shape[0]):
        ids = g["topk_idx"][t]
        vals = sc[t][ids]
        for a in range(7):
            assert vals[a] > vals[a + 1] or (vals[a] == vals[a + 1]
                                             and ids[a] < ids[a + 1])
    assert 10 in g["topk_idx"][1][:3] and 200 in g["topk_idx"][1][:3]
    assert list(g["topk_idx"][3]) == list(range(8))


# ---- 3. live cross-check against the in-place reference build --------

def test_live_ref_random():
    R = po.ref()
    if R is None:
        pytest.skip("oracle/_ref not built (reference tree absent)")
    rng = np.random.default_rng(5)
    R.ds4f_kernels_set_simd(0)
    for trial in range(3):
        r, c = 128, 512
        W = rng.integers(0, 256, (r, c), dtype=np.uint16).astype(np.uint8)
        S = rng.integers(115, 130, 16, dtype=np.uint16).astype(np.uint8)
        x = rng.standard_normal(c).astype(np.float32)
        want = np.zeros(r, np.float32)
        R.ds4f_f8_matvec(po.ptr(W), po.ptr(S), r, c, 4, 4, po.ptr(x),
                         po.ptr(want))
        got = po.f8_matvec(W, po.SCALE_E8M0, S, 4, 4, x)
        assert np.array_equal(bits(got), bits(want))
        sc = rng.standard_normal(256).astype(np.float32)
        i1, w1 = po.topk(sc, 8)
        i2 = np.zeros(8, np.int32)
        w2 = np.zeros(8, np.float32)
        R.ds4f_topk(po.ptr(sc), 256, 8, po.ptr(i2), po.ptr(w2))
        assert np.array_equal(i1, i2) and np.array_equal(bits(w1), bits(w2))


# ---- fixture generator and composed-chain sanity ---------------------

def test_fixture_ln_and_gauss(L):
    for s in (1e-300, 1e-20, 0.001, 0.3, 0.5, 0.70710678, 0.9999999):
        assert abs(L.fx_ln(s) - math.log(s)) <= 4e-16 * abs(math.log(s)) + 1e-300
    k = po.key(0, 0, 4, 0, 0)
    a = po.fill_f32(200000, k, 1.0)
    assert abs(a.mean()) < 0.01 and abs(a.std() - 1.0) < 0.01
    assert np.array_equal(a[:10], po.fill_f32(10, k, 1.0))   # deterministic


def test_fixture_f8_encode_is_nearest_canonical(L):
    lut = np.array([L.orc_f8_value(b) for b in range(256)], np.float32)
    canon = [b for b in range(0x78)] + [0x7E]
    mags = lut[canon].astype(np.float64)
    rng = np.random.default_rng(1)
    for v in np.concatenate([rng.standard_normal(3000) * 100,
                             rng.standard_normal(500) * 0.01, mags,
                             (mags[1:] + mags[:-1]) / 2]).astype(np.float32):
        b = L.fx_f8_encode(float(v))
        assert (b & 0x7F) in canon
        d = np.abs(mags - abs(float(v)))
        assert abs(abs(lut[b]) - abs(float(v))) == d.min()
        assert (b >> 7) == (1 if v < 0 else 0)


def test_fixture_mxfp4_matches_reference_encoder(L):
    k = po.key(3, 1, 3, 5, 0)
    R, Cc = 4, 64
    vals, scales = po.quant_mxfp4(R, Cc, k, 0.02)
    xs = po.fill_f32(R * Cc, k, 0.02)
    v2, s2 = _ref_test_encode(xs, 32)
    assert np.array_equal(vals, v2) and np.array_equal(scales, s2)


def test_fixture_fp8_scales(L):
    k = po.key(0, 2, 3, 1, 0)
    v, s = po.quant_fp8(256, 256, k, 0.02)
    w = po.fill_f32(256 * 256, k, 0.02).reshape(256, 256)
    for br in range(2):
        for bc in range(2):
            blk = w[br * 128:(br + 1) * 128, bc * 128:(bc + 1) * 128]
            assert s[br, bc] == np.float32(np.abs(blk).max()) / np.float32(448)
    lut = np.array([L.orc_f8_value(b) for b in range(256)], np.float32)
    deq = lut[v] * np.repeat(np.repeat(s, 128, 0), 128, 1)
    # canonical magnitudes step from 240 straight to 448 (the reference
    # decodes every e=15 byte as 448), so the widest half-gap is 104 units
    assert np.max(np.abs(deq - w)) <= np.max(s) * 104.0001
    inner = np.abs(w) <= 240 * np.repeat(np.repeat(s, 128, 0), 128, 1)
    assert np.max(np.abs(deq - w)[inner]) <= np.max(s) * 8.0001
    assert not np.any(((v >> 3) & 0xF) == 0xF) or np.all(
        (v[((v >> 3) & 0xF) == 0xF] & 0x7F) == 0x7E)


@pytest.mark.parametrize("fmt", [po.FMT_FP8, po.FMT_MXFP4])
def test_chain_composition_vs_float64(fmt):
    """orc_moe_layer against an independent float64 numpy evaluation of
    the same decoded weights (tolerance: composition, not rounding)."""
    H, M, E, K = 256, 128, 16, 4
    lay = po.Layer(fmt, H, M, E, seed=11, layer=0)
    x = po.fill_f32(H, po.key(11, 0, 4, 0, 0), 1.0)
    st, idx, w, sc, acc = lay.moe(x, K)
    L = po.lib()

    def bf(a):
        return (a.astype(np.uint32) << 16).view(np.float32).astype(np.float64)

    xin = x.astype(np.float64)
    xin = xin / np.sqrt(np.mean(xin * xin) + 1e-6) * bf(lay.norm)
    scores = bf(lay.router) @ xin
    assert np.allclose(scores, sc, atol=1e-4)
    order = np.argsort(-sc, kind="stable")[:K]
    assert np.array_equal(order, idx)

    def deq(slot, t):
        R, Cc = (M, H) if t < 2 else (H, M)
        v = slot[lay.lay.rel_v[t]:]
        s = slot[lay.lay.rel_s[t]:]
        if fmt == po.FMT_FP8:
            out = np.zeros((R, Cc), np.float32)
            L.orc_f8_decode_rows(po.ptr(np.ascontiguousarray(v[:R * Cc])),
                                 po.SCALE_F32,
                                 po.ptr(np.ascontiguousarray(s[:R * Cc // 16384 * 4])),
                                 R, Cc, R // 128, Cc // 128, 0, R, po.ptr(out))
        else:
            out = np.zeros(R * Cc, np.float32)
            L.orc_mxfp4_decode(po.ptr(np.ascontiguousarray(v[:R * Cc // 2])),
                               po.ptr(np.ascontiguousarray(s[:R * Cc // 32])),
                               R * Cc, 32, po.ptr(out))
        return out.reshape(R, Cc).astype(np.float64)

    acc64 = np.zeros(H)
    for j in range(K):
        slot = lay.experts[idx[j]]
        g_, u_ = deq(slot, 0) @ xin, deq(slot, 1) @ xin
        c_ = g_ / (1 + np.exp(-g_)) * u_
        acc64 += w[j] * (deq(slot, 2) @ c_)
    g_, u_ = bf(lay.sh_gate) @ xin, bf(lay.sh_up) @ xin
    so = bf(lay.sh_down) @ (g_ / (1 + np.exp(-g_)) * u_)
    acc64 += so / (1 + np.exp(-(bf(lay.sh_gw) @ xin)))
    err = np.max(np.abs(acc64 - acc)) / np.max(np.abs(acc64))
    assert err < 1e-5
    assert abs(float(np.sum(w)) - 1.0) < 1e-6          # renormalised
    assert np.array_equal(st, (x + acc).astype(np.float32))


def test_batch_equals_per_token():
    H, M, E, K, B = 256, 128, 16, 4, 5
    lay = po.Layer(po.FMT_FP8, H, M, E, seed=3, layer=1)
    xs = po.fill_f32(B * H, po.key(3, 1, 4, 0, 0), 1.0).reshape(B, H)
    st, idx, w = lay.moe_batch(xs, K)
    for b in range(B):
        s1, i1, w1, _, _ = lay.moe(xs[b], K)
        assert np.array_equal(i1, idx[b])
        assert np.array_equal(bits(w1), bits(w[b]))
        assert np.array_equal(bits(s1), bits(st[b]))


# ---- the batched prefill's activation quantiser (oracle/prefill.c) --------

def test_prefill_digits_reconstruct_activations():
    x = po.fill_f32(8 * 256, po.key(21, 0, 4, 0, 0), 1.0).reshape(8, 256)
    x[0, :128] = 0.0
    q, s = po.quant_f8_digits(x, 3)
    val = np.array([po.lib().orc_f8_value(b) for b in range(256)], np.float64)
    rec = (val[q[0]] + val[q[1]] / 16 + val[q[2]] / 256) * np.repeat(s.astype(np.float64), 128, 1)
    amax = np.repeat(np.abs(x).reshape(8, 2, 128).max(2), 128, 1)
    err = np.abs(rec - x) / np.where(amax > 0, amax, 1)
    assert err.max() < 2.0 ** -12
    assert (q[:, 0, :128] == 0).all() and (s[0, 0] == 1.0)
    assert np.abs(val[q]).max() <= 240.0          # digits stay where both E4M3 tables agree
