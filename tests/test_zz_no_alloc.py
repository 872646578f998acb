"""ds4f_gpu_moe_layer_static: the layer step for hosts that cannot let this
library allocate device memory (an engine that owns all of it through its
own pre-sized arena). The caller passes weights, state and outputs as device
pointers; the workspace is a static device array inside the library.

Checked through the C ABI against the existing entry point
ds4f_gpu_moe_layer_dev on the same weights and inputs, two calls in a row,
within the chain tolerance (2e-3 of max |output|; routing indices equal).
This file is collected last (test_zz_*) and passes alone or after the rest.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import pyoracle as po
from tests._lib import ds4f_cuda

pytestmark = pytest.mark.gpu
dc = ds4f_cuda()
TOL = 2e-3


class Ds4fLayerDev(C.Structure):
    _fields_ = [("fmt", C.c_int), ("hidden", C.c_int), ("moe_inter", C.c_int),
                ("n_experts", C.c_int), ("topk", C.c_int), ("renorm", C.c_int),
                ("experts", C.c_void_p), ("slot_bytes", C.c_int64),
                ("norm", C.c_void_p), ("router", C.c_void_p), ("sh_gate", C.c_void_p),
                ("sh_up", C.c_void_p), ("sh_down", C.c_void_p), ("sh_gw", C.c_void_p)]


def relerr(a, b):
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30))


def upload_layer(m, fmt):
    """The model's layer-0 weights copied into caller-owned device buffers."""
    import torch
    tr = [torch.from_numpy(t.reshape(-1).view(np.int16)).cuda() for t in m.get_trunk(0)]
    ex = np.stack([m.get_expert(0, e) for e in range(m.E)])
    ext = torch.from_numpy(ex).cuda()
    ld = Ds4fLayerDev(fmt, m.H, m.M, m.E, m.K, 1, ext.data_ptr(), m.slot_bytes,
                      *[t.data_ptr() for t in tr])
    return ld, tr + [ext]


@pytest.mark.parametrize("fmt,H,M,E", [(dc.FMT_FP8, 1024, 256, 64),
                                       (dc.FMT_MXFP4, 1024, 256, 64),
                                       (dc.FMT_FP8, 2048, 512, 256)])
def test_static_matches_model_path_two_calls(fmt, H, M, E):
    import torch
    L = dc.lib()
    L.ds4f_gpu_moe_layer_static.argtypes = [C.POINTER(Ds4fLayerDev), C.c_void_p,
                                            C.c_void_p, C.c_void_p, C.c_void_p]
    L.ds4f_gpu_moe_layer_static.restype = C.c_int
    dc.init()
    m = dc.Model(fmt, 1, H, M, E, 8)
    m.synth(77)
    ld, keep = upload_layer(m, fmt)
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    for call in range(2):                                  # two calls in a row
        x = po.fill_f32(H, po.key(77, 0, 4, call, 0), 1.0)
        s_new = torch.from_numpy(x).cuda()
        i_new = torch.zeros(8, dtype=torch.int32, device="cuda")
        w_new = torch.zeros(8, dtype=torch.float32, device="cuda")
        dc.check(L.ds4f_gpu_moe_layer_static(C.byref(ld), s_new.data_ptr(),
                                             i_new.data_ptr(), w_new.data_ptr(), sp))
        s_old = torch.from_numpy(x).cuda()
        i_old = torch.zeros(8, dtype=torch.int32, device="cuda")
        w_old = torch.zeros(8, dtype=torch.float32, device="cuda")
        m.layer_dev(0, s_old, i_old, w_old, sp)
        torch.cuda.synchronize()
        assert np.array_equal(i_new.cpu().numpy(), i_old.cpu().numpy())
        assert relerr(w_new.cpu().numpy(), w_old.cpu().numpy()) < TOL
        acc_new = s_new.cpu().numpy().astype(np.float64) - x
        acc_old = s_old.cpu().numpy().astype(np.float64) - x
        assert relerr(acc_new, acc_old) < TOL
    m.close()
    del keep


def test_static_rejects_sizes_beyond_its_maximum():
    L = dc.lib()
    L.ds4f_gpu_moe_layer_static.argtypes = [C.POINTER(Ds4fLayerDev), C.c_void_p,
                                            C.c_void_p, C.c_void_p, C.c_void_p]
    L.ds4f_gpu_moe_layer_static.restype = C.c_int
    dc.init()
    ld = Ds4fLayerDev(dc.FMT_FP8, 4096, 512, 256, 8, 1, 16, 3146496, 16, 16, 16, 16, 16, 16)
    assert L.ds4f_gpu_moe_layer_static(C.byref(ld), 16, None, None, None) == -1
    assert b"maximum" in L.ds4f_gpu_last_error()
