"""The streaming pool's slot policy (ds4f_slotcache_*) against the reference's
own expert cache, src/cache.c:116-223, compiled from its sources into
oracle/_ref: the same request sequences, pins and drops must yield the same
slot for every expert, the same number of fetches per request and the same
request/hit/drop counters. CPU only."""
import ctypes as C
import os

import numpy as np
import pytest

from tests._lib import ROOT, ds4f_cuda

dc = ds4f_cuda()
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libds4f_ref.so")


class ExpertRef(C.Structure):          # include/ds4f/ds4f.h:112
    _fields_ = [("off", C.c_int64), ("nbytes", C.c_int64)]


class ExpertPool(C.Structure):         # include/ds4f/ds4f.h:114-119
    _fields_ = [("fd", C.c_int), ("ref", C.POINTER(ExpertRef)),
                ("n_layers", C.c_int), ("n_experts", C.c_int),
                ("nbytes", C.c_int64)]


class Cache(C.Structure):              # include/ds4f/ds4f.h:192-219 (x86-64 glibc)
    _fields_ = [("pool", C.c_void_p), ("nslot", C.c_int),
                ("slot_bytes", C.c_int64), ("arena", C.c_void_p),
                ("key", C.POINTER(C.c_uint64)),
                ("used_at", C.POINTER(C.c_uint64)), ("pinned", C.c_void_p),
                ("clock", C.c_uint64), ("nthreads", C.c_int),
                ("fth", C.c_void_p), ("fmu", C.c_uint64 * 5),
                ("fcv_work", C.c_uint64 * 6), ("fcv_done", C.c_uint64 * 6),
                ("fshutdown", C.c_int), ("fbusy", C.c_int),
                ("fclaim", C.c_int), ("fdone", C.c_int), ("fnjobs", C.c_int),
                ("fjobs", C.c_void_p), ("nreq", C.c_int64),
                ("nhit", C.c_int64), ("ndrop", C.c_int64),
                ("nread", C.c_int64),
                ("_pad", C.c_uint8 * 256)]


def _ref():
    if not os.path.exists(REF_LIB):
        pytest.skip("oracle/_ref not built (the reference's sources are absent)")
    R = C.CDLL(REF_LIB)
    if not hasattr(R, "ds4f_cache_getmany"):
        pytest.skip("oracle/_ref built without src/cache.c")
    R.ds4f_cache_init.argtypes = [C.POINTER(Cache), C.POINTER(ExpertPool),
                                  C.c_int, C.c_int]
    R.ds4f_cache_free.argtypes = [C.POINTER(Cache)]
    R.ds4f_cache_free.restype = None
    R.ds4f_cache_getmany.argtypes = [C.POINTER(Cache), C.c_int, C.c_void_p,
                                     C.c_int, C.c_void_p]
    R.ds4f_cache_pin.argtypes = [C.POINTER(Cache), C.c_int, C.c_int]
    R.ds4f_cache_pin.restype = None
    R.ds4f_cache_slot.argtypes = [C.POINTER(Cache), C.c_int]
    R.ds4f_cache_slot.restype = C.c_void_p
    return R


class RefCache:
    """The reference's cache over a packed pool file whose expert (l, e)
    payload is NB bytes equal to (l * E + e) mod 251 -- so a slot's bytes
    name the expert it holds."""
    NB = 64

    def __init__(self, R, tmp_path, n_layers, n_experts, nslot, nthreads):
        self.R = R
        path = tmp_path / "pool.bin"
        n = n_layers * n_experts
        payload = np.repeat((np.arange(n) % 251).astype(np.uint8), self.NB)
        payload.tofile(path)
        self.fd = os.open(path, os.O_RDONLY)
        self.refs = (ExpertRef * n)(*[ExpertRef(i * self.NB, self.NB)
                                      for i in range(n)])
        self.pool = ExpertPool(self.fd, self.refs, n_layers, n_experts,
                               self.NB)
        self.c = Cache()
        assert R.ds4f_cache_init(C.byref(self.c), C.byref(self.pool), nslot,
                                 nthreads) == 0
        # the mirrored layout is right: the slot accessor and the field agree
        assert R.ds4f_cache_slot(C.byref(self.c), 0) == self.c.arena
        assert self.c.nslot == nslot and self.c.slot_bytes == self.NB
        self.n_experts = n_experts

    def getmany(self, layer, experts):
        e = np.ascontiguousarray(experts, np.int32)
        out = np.full(max(len(e), 1), -7, np.int32)
        nj = self.R.ds4f_cache_getmany(C.byref(self.c), layer,
                                       e.ctypes.data, len(e), out.ctypes.data)
        return out[:len(e)], nj

    def slot_holds(self, slot):
        p = self.R.ds4f_cache_slot(C.byref(self.c), slot)
        return C.cast(p, C.POINTER(C.c_uint8))[0]

    def pin(self, slot, on):
        self.R.ds4f_cache_pin(C.byref(self.c), slot, on)

    def stats(self):
        return [self.c.nreq, self.c.nhit, self.c.ndrop]

    def close(self):
        self.R.ds4f_cache_free(C.byref(self.c))
        os.close(self.fd)


def _requests(rng, n_layers, n_experts, count):
    """Decode-shaped traffic: layers in turn, top-8 draws with a skew so some
    experts recur, plus ragged, empty and duplicated requests."""
    w = rng.pareto(1.2, n_experts) + 0.05
    w /= w.sum()
    for i in range(count):
        layer = i % n_layers
        kind = rng.random()
        if kind < 0.05:
            ex = np.zeros(0, np.int32)
        elif kind < 0.12:
            ex = rng.integers(0, n_experts, rng.integers(2, 9)).astype(np.int32)
        else:
            k = 8 if kind < 0.8 else int(rng.integers(1, 9))
            ex = rng.choice(n_experts, k, replace=False, p=w).astype(np.int32)
        yield layer, ex


@pytest.mark.parametrize("n_layers,n_experts,nslot,nthreads,seed", [
    (4, 32, 24, 2, 0),       # arena smaller than the pool: steady eviction
    (3, 16, 48, 1, 1),       # the whole pool fits: hits only after warm-up
    (2, 64, 5, 4, 2),        # fewer slots than a request: drops inside one
    (6, 256, 64, 2, 3),      # model-sized expert count
    (8, 256, 2000, 2, 4),    # a large arena: long eviction order, many free slots
])
def test_slot_policy_matches_reference_cache(tmp_path, n_layers, n_experts,
                                             nslot, nthreads, seed):
    R = _ref()
    ref = RefCache(R, tmp_path, n_layers, n_experts, nslot, nthreads)
    mine = dc.SlotCache(nslot)
    rng = np.random.default_rng(seed)
    pinned = set()
    fetched = 0
    try:
        for step, (layer, ex) in enumerate(
                _requests(rng, n_layers, n_experts, 600)):
            if step % 7 == 3:                  # pin / unpin a slot
                s = int(rng.integers(0, nslot))
                on = s not in pinned
                (pinned.add if on else pinned.discard)(s)
                ref.pin(s, int(on))
                mine.pin(s, int(on))
            if step % 150 == 100:              # every slot pinned: drops
                for s in range(nslot):
                    ref.pin(s, 1)
                    mine.pin(s, 1)
            if step % 150 == 104:
                for s in range(nslot):
                    ref.pin(s, int(s in pinned))
                    mine.pin(s, int(s in pinned))
            rs, rn = ref.getmany(layer, ex)
            ms, mn = mine.getmany(layer, ex)
            assert np.array_equal(rs, ms[:len(ex)]), (step, layer, ex, rs, ms)
            assert rn == mn, (step, rn, mn)
            fetched += mn
            for s in set(int(v) for v in rs if v >= 0):
                # the slot holds one of the request's experts mapped to it
                # (not always the selection's own: see the next test)
                names = {(layer * n_experts + int(e)) % 251
                         for e, v in zip(ex, rs) if v == s}
                assert ref.slot_holds(s) in names, (step, s, names)
        req, hit, drop, nf = mine.stats()
        assert [req, hit, drop] == ref.stats()
        assert nf == fetched
        assert drop > 0 or nslot >= 8
    finally:
        ref.close()
        mine.close()


def test_reference_hands_a_hit_slot_to_a_later_miss(tmp_path):
    """The reference's quirk the guarded mode departs from: expert 0 is a hit
    on the least recently fetched slot, so expert 2's miss, later in the same
    request, takes that slot and selection 0 reads expert 2's bytes."""
    R = _ref()
    ref = RefCache(R, tmp_path, 1, 4, 2, 1)
    try:
        ref.getmany(0, [0, 1])
        rs, rn = ref.getmany(0, [0, 2])
        assert list(rs) == [0, 0] and rn == 1
        assert ref.slot_holds(0) == 2                 # not expert 0
    finally:
        ref.close()
    mine = dc.SlotCache(2)
    mine.getmany(0, [0, 1])
    assert list(mine.getmany(0, [0, 2])[0]) == [0, 0]   # same as the reference
    mine.close()
    g = dc.SlotCache(2, guard=True)
    g.getmany(0, [0, 1])
    out, n = g.getmany(0, [0, 2])
    assert list(out) == [0, 1] and n == 1              # slot 0 kept for expert 0
    g.close()


@pytest.mark.parametrize("nslot,seed", [(8, 0), (24, 1), (200, 2)])
def test_guarded_policy_keeps_every_selection_on_its_expert(nslot, seed):
    """Guarded: after each request every selection's slot holds that expert,
    the request's fetch count is the number of its slots whose content
    changed, and nothing drops while unpinned slots are enough -- tracked
    here independently of the library."""
    n_layers, n_experts = 5, 64
    g = dc.SlotCache(nslot, guard=True)
    rng = np.random.default_rng(seed)
    content = {}
    pinned = set()
    for step, (layer, ex) in enumerate(
            _requests(rng, n_layers, n_experts, 800)):
        if step % 11 == 5 and len(pinned) < nslot - 8:
            s = int(rng.integers(0, nslot))
            on = s not in pinned
            (pinned.add if on else pinned.discard)(s)
            g.pin(s, int(on))
        out, n = g.getmany(layer, ex)
        out = out[:len(ex)]
        assert (out >= 0).all(), (step, out)
        changed = set()
        by_slot = {}
        for e, s in zip(ex, out):
            e, s = int(e), int(s)
            assert by_slot.setdefault(s, e) == e, (step, ex, out)
            if content.get(s) != (layer, e):
                changed.add(s)
                assert s not in pinned or s not in content, (step, s)
        assert n == len(changed), (step, ex, out, n, changed)
        for e, s in zip(ex, out):
            content[int(s)] = (layer, int(e))
    g.close()


def test_slot_cache_arguments():
    c = dc.SlotCache(3)
    out, n = c.getmany(0, [5, 6, 7, 8])       # one more than the arena
    assert list(out) == [0, 1, 2, -1] and n == 3
    out, n = c.getmany(0, [7])
    assert list(out) == [2] and n == 0
    assert c.stats() == [5, 1, 1, 3]
    c.close()
    with pytest.raises(dc.GpuError):
        dc.SlotCache(0)


def test_host_entry_points_reject_bad_arguments():
    """NULL pointers, bad sizes and unknown flags return -1 with a message
    (no device involved); a pin outside the arena is ignored, as the
    reference's ds4f_cache_pin ignores it (src/cache.c:221-223)."""
    L = dc.lib()
    h = C.c_void_p()
    assert L.ds4f_slotcache_create(0, 0, C.byref(h)) == -1
    assert L.ds4f_slotcache_create(4, 8, C.byref(h)) == -1          # unknown flag
    assert L.ds4f_slotcache_create(4, 0, None) == -1
    assert L.ds4f_slotcache_create(4, 0, C.byref(h)) == 0
    out = np.zeros(2, np.int32)
    ex = np.array([1, 2], np.int32)
    assert L.ds4f_slotcache_getmany(None, 0, ex.ctypes.data, 2, out.ctypes.data) == -1
    assert L.ds4f_slotcache_getmany(h, 0, None, 2, out.ctypes.data) == -1
    assert L.ds4f_slotcache_getmany(h, 0, ex.ctypes.data, -1, out.ctypes.data) == -1
    assert "slotcache_getmany" in L.ds4f_gpu_last_error().decode()
    neg = np.array([3, -1], np.int32)                  # the key of -1 would be the empty slot's
    assert L.ds4f_slotcache_getmany(h, 0, neg.ctypes.data, 2, out.ctypes.data) == -1
    assert "negative" in L.ds4f_gpu_last_error().decode()
    assert L.ds4f_slotcache_getmany(h, -2, ex.ctypes.data, 2, out.ctypes.data) == -1
    assert L.ds4f_slotcache_pin(h, 99, 1) == 0 and L.ds4f_slotcache_pin(h, -1, 1) == 0
    assert L.ds4f_slotcache_getmany(h, 0, ex.ctypes.data, 2, out.ctypes.data) == 2
    assert L.ds4f_slotcache_stats(None, None, None, None, None) == -1
    L.ds4f_slotcache_free(h)
    L.ds4f_slotcache_free(None)                                      # a no-op
    assert L.ds4f_pool_layout_plan(None, dc.FMT_MXFP4, 64, 32, 2, 3, None, None) == -1
    assert L.ds4f_pool_layout_plan(b"x.json", dc.FMT_MXFP4, 64, 32, 0, 3, None, None) == -1
    assert L.ds4f_pool_layout_plan(b"x.json", 7, 64, 32, 2, 3, None, None) == -1
