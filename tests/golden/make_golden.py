"""Generate tests/golden/ref_vectors.npz from the reference's OWN kernels.

Run in a container that has the reference tree: it builds
oracle/_ref/libds4f_ref.so from the reference's src/kernels.c, simd.c,
moe.c, router.c and gpu_stub.c where they lie (oracle/Makefile), feeds it
seeded inputs, and stores inputs and outputs. The committed .npz then pins
the oracle restatement without the reference tree (tests/test_oracle_golden.py).

Every output is produced by the reference's scalar path
(ds4f_kernels_set_simd(0), src/kernels.c:16) unless the key says _simd.

    python tests/golden/make_golden.py
"""
import ctypes as C
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import pyoracle as po  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ref_vectors.npz")


def edge_f8(rng, n):
    """Random E4M3 bytes with forced subnormals (e=0) and e=15 bytes, as in
    the reference's own edge test (tests/test_kernels.c:325-331)."""
    w = rng.integers(0, 256, n, dtype=np.uint16).astype(np.uint8)
    i = np.arange(n)
    w[i % 5 == 0] &= 0x87
    w[i % 7 == 0] |= 0x78
    return w


def main():
    po.build()
    R = po.ref()
    if R is None:
        sys.exit("reference build missing: need the reference tree to build oracle/_ref")
    ptr = po.ptr
    rng = np.random.default_rng(20261201)
    g = {}

    g["f8_lut"] = np.array([R.ds4f_f8_value(b) for b in range(256)], np.float32)
    g["e8m0"] = np.array([R.ds4f_e8m0_value(b) for b in range(256)], np.float32)

    R.ds4f_kernels_set_simd(0)
    # MXFP4 decode of random bytes; scales include the subnormal (0) and
    # extreme (1, 254) cases.
    mv = rng.integers(0, 256, 256, dtype=np.uint16).astype(np.uint8)
    ms = np.array([0, 1, 64, 100, 120, 125, 126, 127, 128, 129, 130, 140,
                   160, 200, 254, 127], np.uint8)
    out = np.zeros(512, np.float32)
    R.ds4f_mxfp4_decode(ptr(mv), ptr(ms), 512, 32, ptr(out))
    g["mxdec_vals"], g["mxdec_scales"], g["mxdec_out"] = mv, ms, out

    # FP8 matvec with E8M0 block scales, edge-heavy bytes.
    for name, (r, c, sr, sc) in {"a": (48, 256, 3, 2),
                                 "b": (256, 256, 2, 2),
                                 "c": (130, 200, 1, 1)}.items():
        W = edge_f8(rng, r * c).reshape(r, c)
        S = rng.integers(117, 125, sr * sc, dtype=np.uint16).astype(np.uint8)
        x = rng.standard_normal(c).astype(np.float32)
        y = np.zeros(r, np.float32)
        R.ds4f_f8_matvec(ptr(W), ptr(S), r, c, sr, sc, ptr(x), ptr(y))
        g[f"f8mv_{name}_W"], g[f"f8mv_{name}_S"] = W, S
        g[f"f8mv_{name}_x"], g[f"f8mv_{name}_y"] = x, y
        g[f"f8mv_{name}_shape"] = np.array([r, c, sr, sc], np.int32)
        rows = []
        for row in (0, r // 2, r - 1):
            o = np.zeros(c, np.float32)
            R.ds4f_f8_decode_row(ptr(W), ptr(S), r, c, sr, sc, row, ptr(o))
            rows.append(o)
        g[f"f8mv_{name}_rows"] = np.stack(rows)
        R.ds4f_kernels_set_simd(1)
        ys = np.zeros(r, np.float32)
        R.ds4f_f8_matvec(ptr(W), ptr(S), r, c, sr, sc, ptr(x), ptr(ys))
        g[f"f8mv_{name}_y_simd"] = ys
        R.ds4f_kernels_set_simd(0)

    # MXFP4 matvec (scalar two-pass).
    r, c = 24, 256
    V = rng.integers(0, 256, r * c // 2, dtype=np.uint16).astype(np.uint8)
    S = rng.integers(118, 128, r * c // 32, dtype=np.uint16).astype(np.uint8)
    x = rng.standard_normal(c).astype(np.float32)
    y = np.zeros(r, np.float32)
    scr = np.zeros(r * c, np.float32)
    R.ds4f_mxfp4_matvec(ptr(V), ptr(S), r, c, 32, ptr(x), ptr(y), ptr(scr))
    g["mxmv_V"], g["mxmv_S"], g["mxmv_x"], g["mxmv_y"] = V, S, x, y
    g["mxmv_shape"] = np.array([r, c], np.int32)

    # bf16 matvec, without and with bias.
    r, c = 40, 320
    Wf = (rng.standard_normal(r * c) * 0.05).astype(np.float32)
    Wb = (Wf.view(np.uint32) >> 16).astype(np.uint16).reshape(r, c)
    x = rng.standard_normal(c).astype(np.float32)
    bias = rng.standard_normal(r).astype(np.float32)
    y = np.zeros(r, np.float32)
    yb = np.zeros(r, np.float32)
    R.ds4f_bf16_matvec(ptr(Wb), r, c, ptr(x), None, ptr(y))
    R.ds4f_bf16_matvec(ptr(Wb), r, c, ptr(x), ptr(bias), ptr(yb))
    g["bfmv_W"], g["bfmv_x"], g["bfmv_bias"] = Wb, x, bias
    g["bfmv_y"], g["bfmv_yb"] = y, yb

    # MLX-4bit matvec (scalar table path), with and without biases.
    r, c = 16, 256
    V = rng.integers(0, 2**32, r * c // 8, dtype=np.uint64).astype(np.uint32)
    Sf = (rng.random(r * c // 64) * 0.02 + 0.001).astype(np.float32)
    Bf = (rng.standard_normal(r * c // 64) * 0.05).astype(np.float32)
    Sb = (Sf.view(np.uint32) >> 16).astype(np.uint16)
    Bb = (Bf.view(np.uint32) >> 16).astype(np.uint16)
    x = rng.standard_normal(c).astype(np.float32)
    y = np.zeros(r, np.float32)
    y0 = np.zeros(r, np.float32)
    R.ds4f_mlx4_matvec(ptr(V), ptr(Sb), ptr(Bb), r, c, ptr(x), ptr(y))
    R.ds4f_mlx4_matvec(ptr(V), ptr(Sb), None, r, c, ptr(x), ptr(y0))
    g["mlx_V"], g["mlx_S"], g["mlx_B"], g["mlx_x"] = V, Sb, Bb, x
    g["mlx_y"], g["mlx_y0"] = y, y0

    # top-k with softmax (no renorm, as the reference), including ties.
    T, E, K = 24, 256, 8
    sc = rng.standard_normal((T, E)).astype(np.float32)
    sc[1, 10] = sc[1, 200] = sc[1].max()          # exact tie at the top
    sc[2, 30] = sc[2, 31] = np.sort(sc[2])[-8]    # tie at the k boundary
    sc[3, :] = 0.5                                 # all equal
    idx = np.zeros((T, K), np.int32)
    w = np.zeros((T, K), np.float32)
    for t in range(T):
        R.ds4f_topk(ptr(sc[t]), E, K, ptr(idx[t]), ptr(w[t]))
    g["topk_scores"], g["topk_idx"], g["topk_w"] = sc, idx, w

    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes, {len(g)} arrays)")


if __name__ == "__main__":
    main()
