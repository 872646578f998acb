"""ctypes binding of libds4f_cuda (include/ds4f/gpu_cuda.h).

The C ABI is the product boundary; this module mirrors it for Python
callers (tests, bench). It loads the in-tree libds4f_cuda.so and fails
loudly when it is missing: there is no CPU fallback.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libds4f_cuda.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "ds4f", "gpu_cuda.h")

FMT_MXFP4, FMT_MLX4, FMT_FP8, FMT_BF16 = 0, 1, 2, 3
PATH_AUTO, PATH_LAYERED, PATH_PERSISTENT = 0, 1, 2
SCALE_E8M0, SCALE_F32 = 0, 1

_vp = C.c_void_p


class GpuError(RuntimeError):
    pass


class Ds4fMvJob(C.Structure):
    _fields_ = [("w", _vp), ("scales", _vp), ("x", _vp), ("y", _vp),
                ("R", C.c_int), ("C", C.c_int), ("SR", C.c_int), ("SC", C.c_int),
                ("fmt", C.c_int), ("scale_kind", C.c_int), ("bsize", C.c_int),
                ("canon", C.c_int)]


class Ds4fGpuModelDesc(C.Structure):
    _fields_ = [("fmt", C.c_int), ("n_layers", C.c_int), ("hidden", C.c_int),
                ("moe_inter", C.c_int), ("n_experts", C.c_int), ("topk", C.c_int),
                ("renorm", C.c_int), ("expert_first", C.c_int),
                ("expert_count", C.c_int), ("router_exact", C.c_int)]


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise GpuError(f"{LIB_PATH} is not built (run __graft_entry__.build())")
        L = C.CDLL(LIB_PATH)
        L.ds4f_gpu_last_error.restype = C.c_char_p
        L.ds4f_gpu_free.restype = None
        L.ds4f_gpu_model_destroy.restype = None
        L.ds4f_gpu_mv_plan_free.restype = None
        sig = {
            "ds4f_gpu_f8_matvec": [_vp, C.c_int, _vp] + [C.c_int] * 4 + [_vp, _vp],
            "ds4f_gpu_mxfp4_matvec": [_vp, _vp, C.c_int, C.c_int, C.c_int, _vp, _vp],
            "ds4f_gpu_bf16_matvec": [_vp, C.c_int, C.c_int, _vp, _vp, _vp],
            "ds4f_gpu_mlx4_matvec": [_vp, _vp, _vp, C.c_int, C.c_int, _vp, _vp],
            "ds4f_gpu_mlx4_batch": [_vp] * 6 + [C.c_int] * 3,
            "ds4f_gpu_f8_decode_rows": [_vp, C.c_int, _vp] + [C.c_int] * 6 + [_vp],
            "ds4f_gpu_mxfp4_decode": [_vp, _vp, C.c_int64, C.c_int, _vp],
            "ds4f_gpu_mv_plan": [_vp, C.c_int, _vp],
            "ds4f_gpu_mv_run": [_vp, _vp],
            "ds4f_gpu_mv_plan_free": [_vp],
            "ds4f_gpu_model_create": [C.POINTER(Ds4fGpuModelDesc), _vp],
            "ds4f_gpu_model_destroy": [_vp],
            "ds4f_gpu_model_slot": [_vp, _vp, _vp, _vp],
            "ds4f_gpu_model_synth": [_vp, C.c_uint64],
            "ds4f_gpu_model_set_trunk": [_vp, C.c_int] + [_vp] * 6,
            "ds4f_gpu_model_get_trunk": [_vp, C.c_int] + [_vp] * 6,
            "ds4f_gpu_model_set_expert": [_vp, C.c_int, C.c_int, _vp],
            "ds4f_gpu_model_get_expert": [_vp, C.c_int, C.c_int, _vp],
            "ds4f_gpu_pool_load": [_vp, C.c_char_p],
            "ds4f_gpu_moe_layer": [_vp, C.c_int, _vp, _vp, _vp],
            "ds4f_gpu_moe_layer_dev": [_vp, C.c_int, _vp, _vp, _vp, _vp],
            "ds4f_gpu_moe_stack": [_vp, _vp, C.c_int],
            "ds4f_gpu_moe_stack_dev": [_vp, _vp, C.c_int, _vp],
            "ds4f_gpu_model_stats": [_vp, _vp],
            "ds4f_gpu_model_set_path": [_vp, C.c_int],
            "ds4f_gpu_model_trace": [_vp, C.c_int64],
            "ds4f_gpu_model_trace_read": [_vp, _vp, C.c_int64],
            "ds4f_gpu_ep_unique_id": [_vp],
            "ds4f_gpu_ep_attach": [_vp, _vp, C.c_int, C.c_int],
            "ds4f_gpu_ep_detach": [_vp],
            "ds4f_gpu_ep_fused_ready": [_vp],
            "ds4f_gpu_ep_set_fused": [_vp, C.c_int],
            "ds4f_gpu_ep_abort": [_vp],
            "ds4f_gpu_ep_stack_dev": [_vp, _vp, C.c_int, C.c_int, _vp],
            "ds4f_gpu_ep_prefill": [_vp, _vp, C.c_int, _vp, _vp, _vp],
            "ds4f_ep_plan_dispatch": [_vp, C.c_int, C.c_int, C.c_int, C.c_int, _vp, _vp, _vp],
            "ds4f_gpu_model_set_wait_limit": [_vp, C.c_int64],
            "ds4f_gpu_model_inject_stall": [_vp, C.c_int, C.c_int],
            "ds4f_gpu_model_inject_peer_stall": [_vp, C.c_int],
            "ds4f_gpu_model_route_log": [_vp, C.c_int],
            "ds4f_gpu_model_route_log_read": [_vp, _vp, _vp, _vp, C.c_int],
            "ds4f_gpu_synth_f32": [_vp, C.c_int64, C.c_uint64, C.c_uint32, C.c_uint32,
                                   C.c_uint32, C.c_uint32, C.c_double, _vp],
            "ds4f_gpu_quant_f8_digits": [_vp, C.c_int, C.c_int, C.c_int, _vp, _vp, _vp],
            "ds4f_gpu_f8_gemm": [_vp] * 5 + [C.c_int] * 4 + [_vp],
            "ds4f_gpu_moe_prefill": [_vp, C.c_int, _vp, C.c_int, _vp, _vp, _vp],
            "ds4f_gpu_moe_layer_partial_dev": [_vp, C.c_int, _vp, C.c_int, _vp, C.c_int, _vp],
            "ds4f_gpu_prefill": [_vp, _vp, C.c_int, _vp, _vp, _vp],
            "ds4f_gpu_moe_prefill_partial": [_vp, C.c_int, _vp, C.c_int, _vp, _vp, _vp, C.c_int, _vp],
            "ds4f_gpu_moe_layer_batch_dev": [_vp, C.c_int, _vp, C.c_int, _vp, _vp, _vp],
            "ds4f_gpu_moe_layer_batch_partial_dev": [_vp, C.c_int, _vp, C.c_int, _vp, C.c_int, _vp],
            "ds4f_gpu_moe_stack_batch_dev": [_vp, _vp, C.c_int, C.c_int, _vp],
            "ds4f_slotcache_create": [C.c_int, C.c_int, _vp],
            "ds4f_slotcache_getmany": [_vp, C.c_int, _vp, C.c_int, _vp],
            "ds4f_slotcache_pin": [_vp, C.c_int, C.c_int],
            "ds4f_slotcache_stats": [_vp] * 5,
            "ds4f_gpu_model_create_streaming": [_vp, _vp, C.c_int, _vp],
            "ds4f_gpu_stream_stats": [_vp] * 4,
            "ds4f_pool_layout_plan": [C.c_char_p] + [C.c_int] * 5 + [_vp, _vp],
            "ds4f_gpu_pool_load_json": [_vp, C.c_char_p, C.c_char_p],
            "ds4f_gpu_head_create": [C.c_int, _vp, _vp, _vp] + [C.c_int] * 4 + [_vp],
            "ds4f_gpu_head_logits": [_vp] * 4,
            "ds4f_gpu_head_logits_dev": [_vp] * 5,
            "ds4f_gpu_argmax_dev": [_vp, C.c_int, _vp, _vp],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            if name not in ("ds4f_gpu_mv_plan_free", "ds4f_gpu_model_destroy"):
                fn.restype = C.c_int
        L.ds4f_slotcache_free.restype = None
        L.ds4f_gpu_head_free.restype = None
        L.ds4f_gpu_head_free.argtypes = [_vp]
        L.ds4f_slotcache_free.argtypes = [_vp]
        _lib = L
    return _lib


def header_symbols():
    """Function names declared in include/ds4f/gpu_cuda.h."""
    import re
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(ds4f_(?:gpu|slotcache|pool|ep)_\w+)\s*\(", txt)))


def check(rc):
    if rc != 0:
        raise GpuError(lib().ds4f_gpu_last_error().decode(errors="replace"))


def ptr(a):
    if a is None:
        return None
    if hasattr(a, "data_ptr"):
        return C.c_void_p(a.data_ptr())
    return a.ctypes.data_as(C.c_void_p)


def init():
    check(lib().ds4f_gpu_init())


# ---- matvec (host buffers) -------------------------------------------

def f8_matvec(W, scale_kind, scales, SR, SC, x):
    W = np.ascontiguousarray(W, np.uint8)
    R, Cc = W.shape
    y = np.zeros(R, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    s = None if scales is None else np.ascontiguousarray(scales)
    check(lib().ds4f_gpu_f8_matvec(ptr(W), scale_kind, ptr(s), R, Cc, SR, SC, ptr(x), ptr(y)))
    return y


def mxfp4_matvec(vals, scales, R, Cc, x, bsize=32):
    y = np.zeros(R, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    check(lib().ds4f_gpu_mxfp4_matvec(ptr(np.ascontiguousarray(vals)),
                                      ptr(np.ascontiguousarray(scales)), R, Cc, bsize,
                                      ptr(x), ptr(y)))
    return y


def bf16_matvec(W, x, bias=None):
    W = np.ascontiguousarray(W, np.uint16)
    R, Cc = W.shape
    y = np.zeros(R, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    check(lib().ds4f_gpu_bf16_matvec(ptr(W), R, Cc, ptr(x), ptr(b), ptr(y)))
    return y


def mlx4_matvec(vals, scales, biases, R, Cc, x):
    y = np.zeros(R, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    check(lib().ds4f_gpu_mlx4_matvec(ptr(np.ascontiguousarray(vals, np.uint32)),
                                     ptr(np.ascontiguousarray(scales, np.uint16)),
                                     ptr(None if biases is None else
                                         np.ascontiguousarray(biases, np.uint16)),
                                     R, Cc, ptr(x), ptr(y)))
    return y


def f8_decode_rows(W, scale_kind, scales, SR, SC, r0, r1):
    W = np.ascontiguousarray(W, np.uint8)
    R, Cc = W.shape
    out = np.zeros((r1 - r0, Cc), np.float32)
    s = None if scales is None else np.ascontiguousarray(scales)
    check(lib().ds4f_gpu_f8_decode_rows(ptr(W), scale_kind, ptr(s), R, Cc, SR, SC, r0, r1,
                                        ptr(out)))
    return out


def mxfp4_decode(vals, scales, n, bsize=32):
    out = np.zeros(n, np.float32)
    check(lib().ds4f_gpu_mxfp4_decode(ptr(np.ascontiguousarray(vals)),
                                      ptr(np.ascontiguousarray(scales)), n, bsize, ptr(out)))
    return out


class MvPlan:
    """A planned list of device matvec jobs (all run in one launch)."""

    def __init__(self, jobs):
        arr = (Ds4fMvJob * len(jobs))(*jobs)
        h = C.c_void_p()
        check(lib().ds4f_gpu_mv_plan(C.cast(arr, _vp), len(jobs), C.byref(h)))
        self.h = h

    def run(self, stream=None):
        check(lib().ds4f_gpu_mv_run(self.h, stream))

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.ds4f_gpu_mv_plan_free(self.h)
            self.h = None


# ---- model -----------------------------------------------------------

class SlotCache:
    """The reference's expert-cache policy (host only, no device); guard=True
    keeps a request's hits from being evicted by its own misses."""

    def __init__(self, n_slots, guard=False):
        self.h = None
        h = C.c_void_p()
        check(lib().ds4f_slotcache_create(n_slots, 1 if guard else 0, C.byref(h)))
        self.h = h

    def getmany(self, layer, experts):
        """-> (slot per expert, -1 = dropped; number of slots to fill)."""
        e = np.ascontiguousarray(experts, np.int32)
        out = np.zeros(len(e), np.int32)
        n = lib().ds4f_slotcache_getmany(self.h, layer, ptr(e), len(e), ptr(out))
        if n < 0:
            raise GpuError(lib().ds4f_gpu_last_error().decode(errors="replace"))
        return out, n

    def pin(self, slot, on=True):
        check(lib().ds4f_slotcache_pin(self.h, slot, 1 if on else 0))

    def stats(self):
        v = [C.c_int64() for _ in range(4)]
        check(lib().ds4f_slotcache_stats(self.h, *[C.byref(x) for x in v]))
        return [x.value for x in v]

    def close(self):
        if self.h and _lib is not None:
            _lib.ds4f_slotcache_free(self.h)
        self.h = None

    def __del__(self):
        self.close()


class Model:
    def __init__(self, fmt, n_layers, hidden=2048, moe_inter=512, n_experts=256, topk=8,
                 renorm=True, expert_first=0, expert_count=None, router_exact=False,
                 host_pool=None, stream_slots=0):
        """host_pool (uint8 array of every expert, packed) with stream_slots > 0:
        a streaming model (ds4f_gpu_model_create_streaming); the array must
        outlive the model."""
        self.h = None
        d = Ds4fGpuModelDesc(fmt, n_layers, hidden, moe_inter, n_experts, topk,
                             1 if renorm else 0, expert_first,
                             n_experts if expert_count is None else expert_count,
                             1 if router_exact else 0)
        h = C.c_void_p()
        if host_pool is not None:
            self.host_pool = host_pool
            check(lib().ds4f_gpu_model_create_streaming(C.byref(d), ptr(host_pool), stream_slots, C.byref(h)))
        else:
            check(lib().ds4f_gpu_model_create(C.byref(d), C.byref(h)))
        self.h, self.d = h, d
        self.H, self.M, self.E, self.K, self.L = hidden, moe_inter, n_experts, topk, n_layers
        rv = (C.c_int64 * 3)()
        rs = (C.c_int64 * 3)()
        nb = C.c_int64()
        check(lib().ds4f_gpu_model_slot(h, rv, rs, C.byref(nb)))
        self.rel_v, self.rel_s, self.slot_bytes = list(rv), list(rs), nb.value

    def close(self):
        if self.h and _lib is not None:
            _lib.ds4f_gpu_model_destroy(self.h)
        self.h = None

    def __del__(self):
        self.close()

    def synth(self, seed):
        check(lib().ds4f_gpu_model_synth(self.h, seed))

    def set_trunk(self, L, norm, router, sh_gate, sh_up, sh_down, sh_gw):
        a = [np.ascontiguousarray(t, np.uint16) for t in (norm, router, sh_gate, sh_up,
                                                          sh_down, sh_gw)]
        check(lib().ds4f_gpu_model_set_trunk(self.h, L, *[ptr(t) for t in a]))

    def get_trunk(self, L):
        H, M, E = self.H, self.M, self.E
        out = [np.zeros(H, np.uint16), np.zeros((E, H), np.uint16),
               np.zeros((M, H), np.uint16), np.zeros((M, H), np.uint16),
               np.zeros((H, M), np.uint16), np.zeros(H, np.uint16)]
        check(lib().ds4f_gpu_model_get_trunk(self.h, L, *[ptr(t) for t in out]))
        return out

    def set_expert(self, L, X, slot):
        check(lib().ds4f_gpu_model_set_expert(self.h, L, X,
                                              ptr(np.ascontiguousarray(slot, np.uint8))))

    def get_expert(self, L, X):
        out = np.zeros(self.slot_bytes, np.uint8)
        check(lib().ds4f_gpu_model_get_expert(self.h, L, X, ptr(out)))
        return out

    def pool_load(self, path):
        check(lib().ds4f_gpu_pool_load(self.h, path.encode()))

    def pool_load_json(self, pool_path, json_path):
        """A packed pool with the converter's layout file beside it."""
        check(lib().ds4f_gpu_pool_load_json(self.h, str(pool_path).encode(),
                                            str(json_path).encode()))

    def layer(self, L, state):
        st = np.array(state, np.float32, copy=True)
        idx = np.zeros(self.K, np.int32)
        w = np.zeros(self.K, np.float32)
        check(lib().ds4f_gpu_moe_layer(self.h, L, ptr(st), ptr(idx), ptr(w)))
        return st, idx, w

    def stack(self, state, n_steps):
        st = np.array(state, np.float32, copy=True)
        check(lib().ds4f_gpu_moe_stack(self.h, ptr(st), n_steps))
        return st

    def stack_host_inplace(self, st, n_steps):
        """End-to-end call on a caller-owned (e.g. pinned) host buffer."""
        check(lib().ds4f_gpu_moe_stack(self.h, ptr(st), n_steps))

    def layer_dev(self, L, state, idx=None, w=None, stream=None):
        check(lib().ds4f_gpu_moe_layer_dev(self.h, L, ptr(state), ptr(idx), ptr(w), stream))

    def stack_dev(self, state, n_steps, stream=None):
        check(lib().ds4f_gpu_moe_stack_dev(self.h, ptr(state), n_steps, stream))

    def layer_partial_dev(self, L, states, acc, add_shared, stream=None):
        """Expert-parallel shard step of layer L: states [B][H] -> acc [B][H]
        (device); the state is not updated."""
        B = states.shape[0] if states.dim() == 2 else 1
        check(lib().ds4f_gpu_moe_layer_partial_dev(self.h, L, ptr(states), B, ptr(acc),
                                                    1 if add_shared else 0, stream))

    def prefill_layer_dev(self, L, states, sel, w, stream=None):
        """Batched prefill of layer L: states [T][H], sel / w [T][K] (device)."""
        check(lib().ds4f_gpu_moe_prefill(self.h, L, ptr(states), states.shape[0], ptr(sel), ptr(w), stream))

    def prefill_partial_dev(self, L, states, sel, w, acc, add_shared, stream=None):
        """Expert-parallel partial prefill of layer L into acc [T][H]."""
        check(lib().ds4f_gpu_moe_prefill_partial(self.h, L, ptr(states), states.shape[0], ptr(sel), ptr(w),
                                                 ptr(acc), 1 if add_shared else 0, stream))

    def layer_batch_dev(self, L, states, idx=None, w=None, stream=None):
        """Batched decode of layer L: states [B][H] (device) in/out, the
        routing computed on the device into idx / w [B][K] (optional)."""
        check(lib().ds4f_gpu_moe_layer_batch_dev(self.h, L, ptr(states), states.shape[0],
                                                  ptr(idx) if idx is not None else None,
                                                  ptr(w) if w is not None else None, stream))

    def layer_batch_partial_dev(self, L, states, acc, add_shared, stream=None):
        """Expert-parallel batched decode of layer L: this shard's part of
        the combine into acc [B][H] (device); the states are not updated."""
        check(lib().ds4f_gpu_moe_layer_batch_partial_dev(self.h, L, ptr(states), states.shape[0], ptr(acc),
                                                          1 if add_shared else 0, stream))

    def stack_batch_dev(self, states, n_steps, stream=None):
        """n_steps batched decode steps of states [B][H] through every layer."""
        check(lib().ds4f_gpu_moe_stack_batch_dev(self.h, ptr(states), states.shape[0], n_steps, stream))

    def prefill_dev(self, states, sel, w, stream=None):
        """Every layer: sel / w [n_layers][T][K] (device)."""
        check(lib().ds4f_gpu_prefill(self.h, ptr(states), states.shape[0], ptr(sel), ptr(w), stream))

    def set_path(self, path):
        """0 auto, 1 per-layer kernels, 2 persistent decode kernel."""
        check(lib().ds4f_gpu_model_set_path(self.h, path))

    def trace(self, n_stamps):
        check(lib().ds4f_gpu_model_trace(self.h, n_stamps))

    def trace_read(self, n_stamps):
        out = np.zeros(n_stamps, np.uint64)
        check(lib().ds4f_gpu_model_trace_read(self.h, ptr(out), n_stamps))
        return out

    def set_wait_limit(self, polls):
        """Persistent kernel: polls before a bounded wait gives up (0: default)."""
        check(lib().ds4f_gpu_model_set_wait_limit(self.h, polls))

    def inject_peer_stall(self, layer_step):
        """Test hook of the fused multi-GPU step: no down rows stored to the
        other GPUs at layer_step (< 0: off)."""
        check(lib().ds4f_gpu_model_inject_peer_stall(self.h, layer_step))

    def inject_stall(self, cta, layer_step):
        """Test hook: CTA `cta` withholds its state words at `layer_step` (cta < 0: off)."""
        check(lib().ds4f_gpu_model_inject_stall(self.h, cta, layer_step))

    def route_log(self, n_layer_steps):
        check(lib().ds4f_gpu_model_route_log(self.h, n_layer_steps))

    def route_log_read(self, n_layer_steps):
        """(idx [n][K], w [n][K], states [n][H]) of the last persistent call."""
        idx = np.zeros((n_layer_steps, self.K), np.int32)
        w = np.zeros((n_layer_steps, self.K), np.float32)
        st = np.zeros((n_layer_steps, self.H), np.float32)
        check(lib().ds4f_gpu_model_route_log_read(self.h, ptr(idx), ptr(w), ptr(st), n_layer_steps))
        return idx, w, st

    # ---- expert parallelism (the library's NCCL data plane) ----
    def ep_attach(self, ep_id, rank, world):
        """ep_id: the 128 bytes of ep_unique_id() made on rank 0."""
        b = (C.c_uint8 * 128).from_buffer_copy(bytes(ep_id))
        check(lib().ds4f_gpu_ep_attach(self.h, b, rank, world))

    def ep_detach(self):
        check(lib().ds4f_gpu_ep_detach(self.h))

    def ep_fused_ready(self):
        """True when one-token EP steps run as one persistent launch per rank."""
        r = lib().ds4f_gpu_ep_fused_ready(self.h)
        if r < 0:
            check(r)
        return r == 1

    def ep_set_fused(self, on):
        """Fused one-token EP steps where ready (True) or the per-layer path."""
        check(lib().ds4f_gpu_ep_set_fused(self.h, 1 if on else 0))

    def ep_stack_dev(self, states, n_steps, stream=None):
        """states [B][H] (device), identical on every rank."""
        B = states.shape[0] if states.dim() == 2 else 1
        check(lib().ds4f_gpu_ep_stack_dev(self.h, ptr(states), B, n_steps, stream))

    def ep_prefill_dev(self, states, sel, w, stream=None):
        """This rank's states [T][H], routing sel / w [n_layers][T][K] (device)."""
        T = states.shape[0]
        check(lib().ds4f_gpu_ep_prefill(self.h, ptr(states) if T else None, T, ptr(sel) if T else None,
                                        ptr(w) if T else None, stream))

    def stats(self):
        out = (C.c_uint64 * 2)()
        check(lib().ds4f_gpu_model_stats(self.h, out))
        return list(out)

    def stream_stats(self):
        """Streaming model: [experts requested, hits, slots copied in]."""
        v = [C.c_int64() for _ in range(3)]
        check(lib().ds4f_gpu_stream_stats(self.h, *[C.byref(x) for x in v]))
        return [x.value for x in v]


HEAD_F8, HEAD_BF16, HEAD_MLX4 = 2, 4, 6


class Head:
    """The output head (ds4f_gpu_head_*): weights resident, logits + argmax."""

    def __init__(self, dtype, w, scales=None, biases=None, V=None, H=None, SR=1, SC=1):
        self.h = None
        self._keep = [np.ascontiguousarray(a) if a is not None else None for a in (w, scales, biases)]
        h = C.c_void_p()
        check(lib().ds4f_gpu_head_create(dtype, *[ptr(a) for a in self._keep], V, H, SR, SC,
                                         C.byref(h)))
        self.h, self.V, self.H = h, V, H
        self._keep = None

    def logits(self, state, want_logits=True):
        x = np.ascontiguousarray(state, np.float32)
        y = np.zeros(self.V, np.float32) if want_logits else None
        best = C.c_int(-1)
        check(lib().ds4f_gpu_head_logits(self.h, ptr(x), ptr(y), C.byref(best)))
        return y, best.value

    def logits_dev(self, state, logits=None, best=None, stream=None):
        check(lib().ds4f_gpu_head_logits_dev(self.h, ptr(state), ptr(logits), ptr(best), stream))

    def close(self):
        if self.h and _lib is not None:
            _lib.ds4f_gpu_head_free(self.h)
        self.h = None

    def __del__(self):
        self.close()


def argmax_dev(logits, out, stream=None):
    check(lib().ds4f_gpu_argmax_dev(ptr(logits), int(logits.numel()), ptr(out), stream))


def ep_unique_id():
    b = (C.c_uint8 * 128)()
    check(lib().ds4f_gpu_ep_unique_id(b))
    return bytes(b)


def ep_plan_dispatch(sel, n_experts, world):
    """Host-only dispatch plan of one layer: sel [T][K] global expert ids
    -> (counts [world], send_rows [sum counts], tok_rows [T][world])."""
    sel = np.ascontiguousarray(sel, np.int32)
    T, K = sel.shape
    counts = np.zeros(world, np.int32)
    rows = np.zeros(max(1, T * world), np.int32)
    tok = np.zeros((T, world), np.int32)
    check(lib().ds4f_ep_plan_dispatch(ptr(sel) if T else None, T, K, n_experts, world, ptr(counts), ptr(rows),
                                      ptr(tok)))
    return counts, rows[:int(counts.sum())].copy(), tok


def pool_layout_plan(json_path, fmt, hidden, moe_inter, n_layers, n_experts):
    """-> (offsets [n_layers, n_experts, 3 roles, 2 (values, scales)] int64
    absolute file offsets, roles gate/up/down; expert_nbytes). Host only."""
    off = np.zeros((n_layers, n_experts, 3, 2), np.int64)
    nb = C.c_int64()
    check(lib().ds4f_pool_layout_plan(str(json_path).encode(), fmt, hidden, moe_inter,
                                      n_layers, n_experts, ptr(off), C.byref(nb)))
    return off, nb.value


def synth_f32_dev(dst, n, seed, layer, kind, x, t, sigma, stream=None):
    check(lib().ds4f_gpu_synth_f32(ptr(dst), n, seed, layer, kind, x, t, sigma, stream))


def quant_f8_digits_dev(x, q, s, nd=3, stream=None):
    """x [N][C] fp32 (device) -> q [nd][N][C] uint8, s [N][C/128] fp32 (device)."""
    N, Cc = x.shape
    check(lib().ds4f_gpu_quant_f8_digits(ptr(x), N, Cc, nd, ptr(q), ptr(s), stream))


def f8_gemm_dev(W, sW, q, sx, Y, stream=None):
    """Y [N][R] = block-scaled FP8 GEMM of W [R][C] with the digit planes q."""
    R, Cc = W.shape
    nd, N, _ = q.shape
    check(lib().ds4f_gpu_f8_gemm(ptr(W), ptr(sW), ptr(q), ptr(sx), ptr(Y), R, Cc, N, nd, stream))
