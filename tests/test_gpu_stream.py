"""Pools larger than HBM: the streaming model (experts in pinned host
memory, an HBM arena of slots run by the reference's cache policy,
src/cache.c:140-214) against the resident model holding the same bytes, and
against the oracle.

The streamed layer runs the resident layer's kernels on the arena slots, so
state, routing and weights must be bit-identical to the resident model's;
the cache counters must equal the host policy's (ds4f_slotcache_*, guarded)
driven with the same routing."""
import numpy as np
import pytest

from oracle import pyoracle as po
from tests._lib import ds4f_cuda

pytestmark = pytest.mark.gpu
dc = ds4f_cuda()


@pytest.fixture(scope="module", autouse=True)
def gpu():
    dc.init()
    yield


def resident_and_pool(fmt, L, H, M, E, K, seed):
    r = dc.Model(fmt, L, H, M, E, K)
    r.synth(seed)
    r.set_path(dc.PATH_LAYERED)
    pool = np.empty(L * E * r.slot_bytes, np.uint8)
    for l in range(L):
        for e in range(E):
            o = (l * E + e) * r.slot_bytes
            pool[o:o + r.slot_bytes] = r.get_expert(l, e)
    return r, pool


def streaming(r, pool, n_slots):
    s = dc.Model(r.d.fmt, r.L, r.H, r.M, r.E, r.K, host_pool=pool,
                 stream_slots=n_slots)
    for l in range(r.L):
        s.set_trunk(l, *r.get_trunk(l))
    return s


@pytest.mark.parametrize("fmt", [dc.FMT_FP8, dc.FMT_MXFP4])
@pytest.mark.parametrize("n_slots", [8, 40, 400])
def test_streamed_layers_equal_resident(fmt, n_slots):
    L, H, M, E, K = 4, 1024, 256, 64, 8
    r, pool = resident_and_pool(fmt, L, H, M, E, K, 31 + fmt)
    s = streaming(r, pool, n_slots)
    policy = dc.SlotCache(n_slots, guard=True)
    named = set()
    rng = np.random.default_rng(5)
    for tok in range(6):
        x = rng.standard_normal(H).astype(np.float32)
        for l in range(L):
            xr, ir, wr = r.layer(l, x)
            xs, i_s, ws = s.layer(l, x)
            assert np.array_equal(ir, i_s), (tok, l)
            assert np.array_equal(wr.view(np.uint32), ws.view(np.uint32))
            assert np.array_equal(xr.view(np.uint32), xs.view(np.uint32)), \
                (tok, l, np.abs(xr - xs).max())
            policy.getmany(l, ir)
            named |= {(l, int(e)) for e in ir}
            x = xr
    req, hit, drop, fetched = policy.stats()
    assert drop == 0
    assert s.stream_stats() == [req, hit, fetched]
    if n_slots >= L * E:                       # room for all: one fetch each
        assert fetched == len(named)
    else:
        assert fetched >= len(named)
    s.close()
    r.close()
    policy.close()


@pytest.mark.parametrize("fmt", [dc.FMT_FP8, dc.FMT_MXFP4])
def test_streamed_stack_equals_resident_and_oracle(fmt):
    L, H, M, E, K = 3, 1024, 256, 64, 8
    r, pool = resident_and_pool(fmt, L, H, M, E, K, 77)
    s = streaming(r, pool, 12)
    rng = np.random.default_rng(9)
    x = (rng.standard_normal(H) * 0.5).astype(np.float32)
    yr = r.stack(x, 3)
    ys = s.stack(x, 3)
    assert np.array_equal(yr.view(np.uint32), ys.view(np.uint32))
    # one streamed layer against the oracle (its own tolerance rules)
    xs, i_s, ws = s.layer(0, x)
    trunk = r.get_trunk(0)
    ex = pool[:E * r.slot_bytes].reshape(E, r.slot_bytes)
    lay = po.Layer.from_arrays(fmt, H, M, E, trunk, ex)
    st_o, idx_o, w_o, _, acc_o = lay.moe(x, K)
    assert np.array_equal(i_s, idx_o)
    acc_g = xs.astype(np.float64) - x.astype(np.float64)
    assert np.max(np.abs(acc_g - acc_o)) <= 2e-3 * np.max(np.abs(acc_o))
    s.close()
    r.close()


def test_streaming_model_refuses_resident_only_calls():
    L, H, M, E, K = 1, 1024, 256, 64, 8
    r, pool = resident_and_pool(dc.FMT_FP8, L, H, M, E, K, 3)
    s = streaming(r, pool, 8)
    with pytest.raises(dc.GpuError):
        s.synth(1)
    with pytest.raises(dc.GpuError):
        s.set_expert(0, 0, pool[:r.slot_bytes])
    with pytest.raises(dc.GpuError):
        dc.Model(dc.FMT_FP8, L, H, M, E, K, host_pool=pool, stream_slots=K - 1)
    s.close()
    r.close()
