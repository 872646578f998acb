"""The oracle's MoE step pinned to the reference's own ds4f_moe_step.

The kernels (matvecs, decode, top-k) are pinned bit for bit by the golden
vectors; this pins their composition. oracle/_ref holds the reference's
src/moe.c compiled in place with a caller (oracle/ref_step.c) that builds
the trunk and pool layouts of one Qwen3.5 layer of MXFP4 experts in memory:
the step's own RMSNorm, its K expert chains on threads, the selection-order
combine and the residual (src/moe.c:948-1456). The routing is the
reference's too: its bf16 router matvec and ds4f_topk (raw softmax weights:
the reference does not renormalise, src/moe.c:547-560).

The oracle is orc_moe_layer with renorm off and the shared expert's weights
zero (its contribution is then exactly +0). Indices, weights and the new
state must be bit-identical.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import pyoracle as po

R = po.ref()
pytestmark = pytest.mark.skipif(R is None or not hasattr(R, "orcref_moe_step_mxfp4"),
                                reason="oracle/_ref (the reference compiled in place) not built")


@pytest.mark.parametrize("H,M,E,K,seed", [(1024, 256, 64, 8, 3), (2048, 512, 48, 8, 4), (1024, 256, 32, 4, 5)])
def test_reference_moe_step_equals_oracle_step(H, M, E, K, seed):
    R.ds4f_kernels_set_simd(0)          # the scalar path (the AVX2 MXFP4 decode is wrong on x86)
    R.orcref_moe_step_mxfp4.argtypes = [C.c_int] * 4 + [C.c_void_p] * 4 + [C.c_int64] + [C.c_void_p] * 3
    R.orcref_moe_step_mxfp4.restype = C.c_int
    lay = po.Layer(po.FMT_MXFP4, H, M, E, seed, 0)
    for t in (lay.sh_gate, lay.sh_up, lay.sh_down, lay.sh_gw):
        t[...] = 0                      # no shared expert: the reference layer has none
    rel_v = np.array(lay.lay.rel_v[:], np.int64)
    rel_s = np.array(lay.lay.rel_s[:], np.int64)
    ptr = po.ptr
    for i in range(3):
        state = po.fill_f32(H, po.key(seed, 0, 4, i, 0), 1.0)
        # the reference's router: RMSNorm'd input, bf16 matvec, ds4f_topk
        xin = state.copy()
        po.lib().orc_rmsnorm(ptr(lay.norm), H, ptr(xin))
        scores = np.zeros(E, np.float32)
        R.ds4f_bf16_matvec(ptr(lay.router), E, H, ptr(xin), None, ptr(scores))
        sel = np.zeros(K, np.int32)
        w = np.zeros(K, np.float32)
        R.ds4f_topk(ptr(scores), E, K, ptr(sel), ptr(w))
        # the oracle's whole step, router included
        st_o, idx_o, w_o, sc_o, _ = lay.moe(state, K, renorm=False)
        assert np.array_equal(sc_o.view(np.uint32), scores.view(np.uint32))
        assert np.array_equal(idx_o, sel) and np.array_equal(w_o.view(np.uint32), w.view(np.uint32))
        # the reference's step on the same routing
        st_r = state.copy()
        rc = R.orcref_moe_step_mxfp4(H, M, E, K, ptr(lay.norm), ptr(lay.experts), ptr(rel_v), ptr(rel_s),
                                     lay.lay.nbytes, ptr(sel), ptr(w), ptr(st_r))
        assert rc == 0
        assert np.array_equal(st_o.view(np.uint32), st_r.view(np.uint32)), \
            float(np.abs(st_o - st_r).max())
