"""ctypes binding of the C99 oracle and the CPU fixture generator.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline leg, as the checker. The product path never loads
it. `ref()` exposes the reference's own kernels compiled in place
(oracle/_ref/libds4f_ref.so), when that build exists.
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libds4f_oracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libds4f_ref.so")

FMT_MXFP4 = 0
FMT_FP8 = 2
SCALE_E8M0 = 0
SCALE_F32 = 1

_u8p = C.POINTER(C.c_uint8)
_u16p = C.POINTER(C.c_uint16)
_f32p = C.POINTER(C.c_float)
_i32p = C.POINTER(C.c_int)


class OrcExpertLayout(C.Structure):
    _fields_ = [("rel_v", C.c_int64 * 3), ("rel_s", C.c_int64 * 3),
                ("nbytes", C.c_int64)]


class OrcLayerW(C.Structure):
    _fields_ = [("norm", C.c_void_p), ("router", C.c_void_p),
                ("sh_gate", C.c_void_p), ("sh_up", C.c_void_p),
                ("sh_down", C.c_void_p), ("sh_gw", C.c_void_p),
                ("experts", C.c_void_p)]


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = C.CDLL(LIB)
        L.orc_e8m0_value.restype = C.c_float
        L.orc_e8m0_value.argtypes = [C.c_uint8]
        L.orc_f8_value.restype = C.c_float
        L.orc_f8_value.argtypes = [C.c_uint8]
        L.fx_mix64.restype = C.c_uint64
        L.fx_mix64.argtypes = [C.c_uint64]
        L.fx_tid.restype = C.c_uint64
        L.fx_tid.argtypes = [C.c_uint32] * 4
        L.fx_key.restype = C.c_uint64
        L.fx_key.argtypes = [C.c_uint64, C.c_uint64]
        L.fx_gauss.restype = C.c_double
        L.fx_gauss.argtypes = [C.c_uint64, C.c_uint64]
        L.fx_ln.restype = C.c_double
        L.fx_ln.argtypes = [C.c_double]
        L.fx_value.restype = C.c_float
        L.fx_value.argtypes = [C.c_uint64, C.c_uint64, C.c_double]
        L.fx_f8_encode.restype = C.c_uint8
        L.fx_f8_encode.argtypes = [C.c_float]
        L.fx_fill_f32.argtypes = [C.c_void_p, C.c_int64, C.c_uint64, C.c_double]
        L.fx_fill_bf16.argtypes = [C.c_void_p, C.c_int64, C.c_uint64, C.c_double]
        L.fx_quant_fp8.argtypes = [C.c_int, C.c_int, C.c_uint64, C.c_double,
                                   C.c_void_p, C.c_void_p]
        L.fx_quant_mxfp4.argtypes = [C.c_int, C.c_int, C.c_uint64, C.c_double,
                                     C.c_void_p, C.c_void_p]
        L.fx_expert.argtypes = [C.c_int, C.c_int, C.c_int, C.c_uint64,
                                C.c_uint32, C.c_uint32, C.c_double, C.c_void_p]
        L.fx_trunk.argtypes = [C.c_int, C.c_int, C.c_int, C.c_uint64,
                               C.c_uint32, C.c_double] + [C.c_void_p] * 6
        L.orc_mxfp4_decode.argtypes = [C.c_void_p, C.c_void_p, C.c_int64,
                                       C.c_int, C.c_void_p]
        L.orc_f8_decode_rows.argtypes = [C.c_void_p, C.c_int, C.c_void_p] + \
            [C.c_int] * 6 + [C.c_void_p]
        L.orc_f8_matvec.argtypes = [C.c_void_p, C.c_int, C.c_void_p] + \
            [C.c_int] * 4 + [C.c_void_p, C.c_void_p]
        L.orc_mxfp4_matvec.argtypes = [C.c_void_p, C.c_void_p, C.c_int,
                                       C.c_int, C.c_int, C.c_void_p,
                                       C.c_void_p, C.c_void_p]
        L.orc_bf16_matvec.argtypes = [C.c_void_p, C.c_int, C.c_int,
                                      C.c_void_p, C.c_void_p, C.c_void_p]
        L.orc_mlx4_matvec.argtypes = [C.c_void_p] * 3 + [C.c_int, C.c_int,
                                                         C.c_void_p, C.c_void_p]
        L.orc_rmsnorm.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        L.orc_topk.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                               C.c_void_p]
        L.orc_topk_renorm.argtypes = [C.c_int, C.c_void_p]
        L.orc_silu_mul.restype = C.c_float
        L.orc_silu_mul.argtypes = [C.c_float, C.c_float]
        L.orc_expert_layout.argtypes = [C.c_int, C.c_int, C.c_int,
                                        C.POINTER(OrcExpertLayout)]
        L.orc_expert_chain.argtypes = [C.c_int, C.c_void_p,
                                       C.POINTER(OrcExpertLayout), C.c_int,
                                       C.c_int, C.c_void_p, C.c_void_p]
        L.orc_moe_layer.argtypes = [C.c_int] * 6 + [
            C.POINTER(OrcLayerW), C.POINTER(OrcExpertLayout), C.c_void_p,
            C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
        L.orc_moe_batch.argtypes = [C.c_int] * 6 + [
            C.POINTER(OrcLayerW), C.POINTER(OrcExpertLayout), C.c_int,
            C.c_void_p, C.c_void_p, C.c_void_p]
        L.orc_quant_f8_digits.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int,
                                          C.c_void_p, C.c_void_p]
        L.orc_moe_batch_sel.argtypes = [C.c_int] * 4 + [
            C.POINTER(OrcLayerW), C.POINTER(OrcExpertLayout), C.c_int,
            C.c_void_p, C.c_void_p, C.c_void_p]
        L.orc_shared_add.argtypes = [C.POINTER(OrcLayerW), C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        L.orc_prefill_layer.argtypes = [C.c_int] * 4 + [
            C.POINTER(OrcLayerW), C.POINTER(OrcExpertLayout), C.c_int,
            C.c_void_p, C.c_void_p, C.c_void_p]
        L.orc_f8_gemm_digits.argtypes = [C.c_void_p] * 5 + [C.c_int] * 4
        _lib = L
    return _lib


def ref():
    """The reference's own kernels (compiled in place), or None."""
    global _ref
    if _ref is None and os.path.exists(REF_LIB):
        R = C.CDLL(REF_LIB)
        R.ds4f_e8m0_value.restype = C.c_float
        R.ds4f_e8m0_value.argtypes = [C.c_uint8]
        R.ds4f_f8_value.restype = C.c_float
        R.ds4f_f8_value.argtypes = [C.c_uint8]
        R.ds4f_kernels_set_simd.argtypes = [C.c_int]
        R.ds4f_mxfp4_decode.argtypes = [C.c_void_p, C.c_void_p, C.c_int,
                                        C.c_int, C.c_void_p]
        R.ds4f_mxfp4_matvec.argtypes = [C.c_void_p, C.c_void_p, C.c_int,
                                        C.c_int, C.c_int, C.c_void_p,
                                        C.c_void_p, C.c_void_p]
        R.ds4f_bf16_matvec.argtypes = [C.c_void_p, C.c_int, C.c_int,
                                       C.c_void_p, C.c_void_p, C.c_void_p]
        R.ds4f_f8_matvec.argtypes = [C.c_void_p, C.c_void_p] + \
            [C.c_int] * 4 + [C.c_void_p, C.c_void_p]
        R.ds4f_f8_decode_row.argtypes = [C.c_void_p, C.c_void_p] + \
            [C.c_int] * 5 + [C.c_void_p]
        R.ds4f_mlx4_matvec.argtypes = [C.c_void_p] * 3 + [C.c_int, C.c_int,
                                                          C.c_void_p, C.c_void_p]
        R.ds4f_topk.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                C.c_void_p]
        _ref = R
    return _ref


def argmax(logits):
    """ds4f_argmax (src/head.c:303-309): start from logits[0]; an index is
    taken only if its logit is strictly greater than the best so far."""
    best, bv = 0, logits[0]
    for i in range(1, len(logits)):
        if logits[i] > bv:
            bv, best = logits[i], i
    return best


def ptr(a):
    return a.ctypes.data_as(C.c_void_p) if a is not None else None


# ---- convenience wrappers (numpy in, numpy out) ----------------------

def expert_layout(fmt, H, M):
    lay = OrcExpertLayout()
    if lib().orc_expert_layout(fmt, H, M, C.byref(lay)) != 0:
        raise ValueError("shape does not fit format")
    return lay


def f8_matvec(W, scale_kind, scales, SR, SC, x):
    R, Cc = W.shape
    y = np.zeros(R, np.float32)
    lib().orc_f8_matvec(ptr(W), scale_kind, ptr(scales), R, Cc, SR, SC,
                        ptr(x), ptr(y))
    return y


def mxfp4_matvec(vals, scales, R, Cc, x, bsize=32):
    y = np.zeros(R, np.float32)
    scr = np.zeros(R * Cc, np.float32)
    lib().orc_mxfp4_matvec(ptr(vals), ptr(scales), R, Cc, bsize, ptr(x),
                           ptr(y), ptr(scr))
    return y


def bf16_matvec(W, x, bias=None):
    R, Cc = W.shape
    y = np.zeros(R, np.float32)
    lib().orc_bf16_matvec(ptr(W), R, Cc, ptr(x), ptr(bias), ptr(y))
    return y


def mlx4_matvec(vals, scales, biases, R, Cc, x):
    y = np.zeros(R, np.float32)
    lib().orc_mlx4_matvec(ptr(vals), ptr(scales), ptr(biases), R, Cc, ptr(x),
                          ptr(y))
    return y


def topk(scores, k, renorm=False):
    idx = np.zeros(k, np.int32)
    w = np.zeros(k, np.float32)
    lib().orc_topk(ptr(scores), len(scores), k, ptr(idx), ptr(w))
    if renorm:
        lib().orc_topk_renorm(k, ptr(w))
    return idx, w


def key(seed, layer, kind, x, t):
    L = lib()
    return L.fx_key(seed, L.fx_tid(layer, kind, x, t))


def fill_f32(n, k, sigma):
    a = np.zeros(n, np.float32)
    lib().fx_fill_f32(ptr(a), n, k, sigma)
    return a


def fill_bf16(n, k, sigma):
    a = np.zeros(n, np.uint16)
    lib().fx_fill_bf16(ptr(a), n, k, sigma)
    return a


def quant_fp8(R, Cc, k, sigma):
    v = np.zeros((R, Cc), np.uint8)
    s = np.zeros((R // 128, Cc // 128), np.float32)
    if lib().fx_quant_fp8(R, Cc, k, sigma, ptr(v), ptr(s)) != 0:
        raise ValueError("fp8 needs R, C multiples of 128")
    return v, s


def quant_mxfp4(R, Cc, k, sigma):
    v = np.zeros(R * Cc // 2, np.uint8)
    s = np.zeros(R * Cc // 32, np.uint8)
    if lib().fx_quant_mxfp4(R, Cc, k, sigma, ptr(v), ptr(s)) != 0:
        raise ValueError("mxfp4 needs C multiple of 32")
    return v, s


class Layer:
    """One layer's synthetic weights (trunk + E expert slots), CPU side."""

    def __init__(self, fmt, H, M, E, seed, layer, sigma=0.02, experts=None):
        L = lib()
        self.fmt, self.H, self.M, self.E = fmt, H, M, E
        self.lay = expert_layout(fmt, H, M)
        self.norm = np.zeros(H, np.uint16)
        self.router = np.zeros((E, H), np.uint16)
        self.sh_gate = np.zeros((M, H), np.uint16)
        self.sh_up = np.zeros((M, H), np.uint16)
        self.sh_down = np.zeros((H, M), np.uint16)
        self.sh_gw = np.zeros(H, np.uint16)
        L.fx_trunk(H, M, E, seed, layer, sigma, ptr(self.norm),
                   ptr(self.router), ptr(self.sh_gate), ptr(self.sh_up),
                   ptr(self.sh_down), ptr(self.sh_gw))
        if experts is not None:
            self.experts = np.ascontiguousarray(experts, np.uint8)
        else:
            self.experts = np.zeros((E, self.lay.nbytes), np.uint8)
            for x in range(E):
                row = self.experts[x]
                if L.fx_expert(fmt, H, M, seed, layer, x, sigma,
                               ptr(row)) != 0:
                    raise ValueError("bad expert shape")

    @classmethod
    def from_arrays(cls, fmt, H, M, E, trunk, experts):
        """A layer from given bytes: trunk = (norm, router, sh_gate, sh_up,
        sh_down, sh_gw) bf16 arrays, experts [E, slot_bytes] uint8."""
        self = cls.__new__(cls)
        self.fmt, self.H, self.M, self.E = fmt, H, M, E
        self.lay = expert_layout(fmt, H, M)
        (self.norm, self.router, self.sh_gate, self.sh_up, self.sh_down,
         self.sh_gw) = [np.ascontiguousarray(t, np.uint16) for t in trunk]
        self.experts = experts
        return self

    def route(self, state, K, renorm=True):
        """Router only (src/main.c:1014-1088 + topk + renorm)."""
        xin = np.array(state, np.float32, copy=True)
        lib().orc_rmsnorm(ptr(self.norm), self.H, ptr(xin))
        sc = bf16_matvec(self.router, xin)
        idx, w = topk(sc, K, renorm)
        return idx, w, sc, xin

    def w(self):
        return OrcLayerW(ptr(self.norm), ptr(self.router), ptr(self.sh_gate),
                         ptr(self.sh_up), ptr(self.sh_down), ptr(self.sh_gw),
                         ptr(self.experts))

    def moe(self, state, K, renorm=True):
        """One token through the layer; returns (new_state, idx, w, scores,
        acc)."""
        st = np.array(state, np.float32, copy=True)
        idx = np.zeros(K, np.int32)
        w = np.zeros(K, np.float32)
        sc = np.zeros(self.E, np.float32)
        acc = np.zeros(self.H, np.float32)
        lw = self.w()
        if lib().orc_moe_layer(self.fmt, self.H, self.M, self.E, K,
                               1 if renorm else 0, C.byref(lw),
                               C.byref(self.lay), ptr(st), ptr(idx), ptr(w),
                               ptr(sc), ptr(acc)) != 0:
            raise RuntimeError("orc_moe_layer failed")
        return st, idx, w, sc, acc

    def moe_batch(self, states, K, renorm=True):
        st = np.array(states, np.float32, copy=True)
        B = st.shape[0]
        idx = np.zeros((B, K), np.int32)
        w = np.zeros((B, K), np.float32)
        lw = self.w()
        if lib().orc_moe_batch(self.fmt, self.H, self.M, self.E, K,
                               1 if renorm else 0, C.byref(lw),
                               C.byref(self.lay), B, ptr(st), ptr(idx),
                               ptr(w)) != 0:
            raise RuntimeError("orc_moe_batch failed")
        return st, idx, w


def _layer_batch_sel(self, states, sel, w):
    """The reference batched step with the routing given (fp32)."""
    st = np.array(states, np.float32, copy=True)
    sel = np.ascontiguousarray(sel, np.int32)
    w = np.ascontiguousarray(w, np.float32)
    lw = self.w()
    if lib().orc_moe_batch_sel(self.fmt, self.H, self.M, sel.shape[1], C.byref(lw), C.byref(self.lay),
                               st.shape[0], ptr(st), ptr(sel), ptr(w)) != 0:
        raise RuntimeError("orc_moe_batch_sel failed")
    return st


def _layer_prefill(self, states, sel, w):
    """The GPU prefill's own arithmetic (quantised activations) restated."""
    st = np.array(states, np.float32, copy=True)
    sel = np.ascontiguousarray(sel, np.int32)
    w = np.ascontiguousarray(w, np.float32)
    lw = self.w()
    if lib().orc_prefill_layer(self.fmt, self.H, self.M, sel.shape[1], C.byref(lw), C.byref(self.lay), st.shape[0],
                               ptr(st), ptr(sel), ptr(w)) != 0:
        raise RuntimeError("orc_prefill_layer failed")
    return st


Layer.moe_batch_sel = _layer_batch_sel
Layer.prefill = _layer_prefill


def quant_f8_digits(x, nd=3):
    """Activation quantiser of the GPU prefill: x [N][C] fp32 ->
    (q [nd][N][C] uint8 E4M3 digit planes, s [N][C/128] fp32)."""
    x = np.ascontiguousarray(x, np.float32)
    N, Cc = x.shape
    q = np.zeros((nd, N, Cc), np.uint8)
    s = np.zeros((N, Cc // 128), np.float32)
    assert lib().orc_quant_f8_digits(ptr(x), N, Cc, nd, ptr(q), ptr(s)) == 0
    return q, s


def f8_gemm_digits(W, sW, q, sx):
    """Double-precision reference of the block-scaled digit GEMM: Y [N][R]."""
    W = np.ascontiguousarray(W, np.uint8)
    sW = np.ascontiguousarray(sW, np.float32)
    q = np.ascontiguousarray(q, np.uint8)
    sx = np.ascontiguousarray(sx, np.float32)
    R, Cc = W.shape
    nd, N, _ = q.shape
    Y = np.zeros((N, R), np.float64)
    assert lib().orc_f8_gemm_digits(ptr(W), ptr(sW), ptr(q), ptr(sx), ptr(Y), R, Cc, N, nd) == 0
    return Y
