"""The MoE layer and the decode stack on the GPU vs the oracle, through the
C ABI.

Parity rules:
  * router top-k indices bit-exact (no exact-tie cases here except where a
    test builds them on purpose, resolved by the reference's lower-index rule);
  * expert-chain output (the layer's acc = new_state - state) within max
    relative error 2e-3 of max |acc_ref|, fp32 accumulation;
  * routing weights within 1e-5 relative (logits are certified, not
    recomputed exactly, unless router_exact).
"""
import numpy as np
import pytest

from oracle import pyoracle as po
from tests._lib import ds4f_cuda

pytestmark = pytest.mark.gpu
dc = ds4f_cuda()
CHAIN_TOL = 2e-3          # max |y - y_ref| / max |y_ref|
W_TOL = 1e-5


@pytest.fixture(scope="module", autouse=True)
def gpu():
    dc.init()
    yield


def relerr(a, b):
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30))


def oracle_layer(m, L, fmt, state, sel=None):
    """The oracle's view of GPU layer L built from the GPU's own bytes; only
    the experts the oracle's router picks are downloaded."""
    trunk = m.get_trunk(L)
    ex = np.zeros((m.E, m.slot_bytes), np.uint8)        # lazily committed pages
    lay = po.Layer.from_arrays(fmt, m.H, m.M, m.E, trunk, ex)
    idx, _, _, _ = lay.route(state, m.K)
    for e in set(idx.tolist()) | set(sel or []):
        ex[e] = m.get_expert(L, e)
    return lay


def check_layer(m, L, fmt, state):
    st_g, idx_g, w_g = m.layer(L, state)
    lay = oracle_layer(m, L, fmt, state, idx_g.tolist())
    st_o, idx_o, w_o, sc, acc_o = lay.moe(state, m.K)
    assert np.array_equal(idx_g, idx_o), (idx_g, idx_o)
    assert relerr(w_g, w_o) < W_TOL
    acc_g = st_g.astype(np.float64) - np.asarray(state, np.float64)
    assert relerr(acc_g, acc_o) < CHAIN_TOL
    return st_g, st_o, idx_g


@pytest.mark.parametrize("fmt", [dc.FMT_FP8, dc.FMT_MXFP4])
def test_layer_small(fmt):
    m = dc.Model(fmt, 2, 1024, 256, 64, 8)
    m.synth(21)
    for t in range(6):
        x = po.fill_f32(1024, po.key(21, 0, 4, t, 0), 1.0)
        check_layer(m, t % 2, fmt, x)
    m.close()


@pytest.mark.parametrize("fmt", [dc.FMT_FP8, dc.FMT_MXFP4])
def test_layer_baseline_shape(fmt):
    """Config 0 shapes: H 2048, M 512, E 256, top-8, renormalised."""
    m = dc.Model(fmt, 1, 2048, 512, 256, 8)
    m.synth(0)
    for t in range(3):
        x = po.fill_f32(2048, po.key(0, 0, 4, t, 0), 1.0)
        check_layer(m, 0, fmt, x)
    m.close()


def test_no_renorm_matches_reference_raw_weights():
    m = dc.Model(dc.FMT_FP8, 1, 1024, 256, 64, 8, renorm=False)
    m.synth(4)
    x = po.fill_f32(1024, po.key(4, 0, 4, 0, 0), 1.0)
    st_g, idx_g, w_g = m.layer(0, x)
    lay = oracle_layer(m, 0, dc.FMT_FP8, x, idx_g.tolist())
    st_o, idx_o, w_o, _, acc_o = lay.moe(x, 8, renorm=False)
    assert np.array_equal(idx_g, idx_o)
    assert relerr(w_g, w_o) < W_TOL and float(np.sum(w_g)) < 1.0
    assert relerr(st_g.astype(np.float64) - x, acc_o) < CHAIN_TOL
    m.close()


@pytest.mark.parametrize("fmt", [dc.FMT_FP8, dc.FMT_MXFP4])
def test_stack_free_running_and_teacher_forced(fmt):
    L, steps = 4, 3
    m = dc.Model(fmt, L, 1024, 256, 64, 8)
    m.synth(33)
    x0 = po.fill_f32(1024, po.key(33, 0, 4, 0, 0), 1.0)
    got = m.stack(x0, steps)
    st = x0.copy()
    for s in range(steps):
        for layer in range(L):
            # teacher forcing: the GPU layer from the oracle's own input
            st_g, _, _ = check_layer(m, layer, fmt, st)
            lay = oracle_layer(m, layer, fmt, st)
            st, _, _, _, _ = lay.moe(st, 8)
    assert relerr(got, st) < CHAIN_TOL
    # device-pointer path gives the same bits as the host path
    import torch
    t = torch.from_numpy(x0.copy()).cuda()
    m.stack_dev(t, steps)
    torch.cuda.synchronize()
    assert np.array_equal(t.cpu().numpy(), got)
    m.close()


def test_router_exact_tie_falls_back_and_matches():
    """Two router rows made identical: exact logit tie. The certificate
    cannot separate them, the exact reference-order sums run, and the
    lower index wins (src/moe.c:537)."""
    m = dc.Model(dc.FMT_FP8, 1, 1024, 256, 64, 8)
    m.synth(8)
    tr = m.get_trunk(0)
    x = po.fill_f32(1024, po.key(8, 0, 4, 0, 0), 1.0)
    lay = oracle_layer(m, 0, dc.FMT_FP8, x)
    idx, _, sc, _ = lay.route(x, 8)
    a = int(idx[2])
    b = [e for e in range(64) if e not in idx and e > a][0]
    tr[1][b] = tr[1][a]
    m.set_trunk(0, *tr)
    before = m.stats()[1]
    st_g, idx_g, w_g = m.layer(0, x)
    lay = oracle_layer(m, 0, dc.FMT_FP8, x, idx_g.tolist())
    st_o, idx_o, w_o, sc, acc_o = lay.moe(x, 8)
    assert np.array_equal(idx_g, idx_o)
    assert a in idx_g.tolist() and b in idx_g.tolist()
    assert idx_g.tolist().index(a) < idx_g.tolist().index(b)
    assert m.stats()[1] > before
    assert relerr(st_g.astype(np.float64) - x, acc_o) < CHAIN_TOL
    m.close()


def test_router_exact_mode_weights_bit_exact():
    m = dc.Model(dc.FMT_FP8, 1, 1024, 256, 64, 8, router_exact=True)
    m.synth(12)
    for t in range(3):
        x = po.fill_f32(1024, po.key(12, 0, 4, t, 0), 1.0)
        st_g, idx_g, w_g = m.layer(0, x)
        lay = oracle_layer(m, 0, dc.FMT_FP8, x, idx_g.tolist())
        _, idx_o, w_o, _, _ = lay.moe(x, 8)
        assert np.array_equal(idx_g, idx_o)
        ulp = np.abs(w_g.view(np.int32).astype(np.int64) - w_o.view(np.int32).astype(np.int64))
        assert int(ulp.max()) <= 1          # CUDA vs glibc double exp: <= 1 ulp
    m.close()


@pytest.mark.parametrize("fmt", [dc.FMT_FP8, dc.FMT_MXFP4])
def test_pool_load_packed_file(tmp_path, fmt):
    """ds4f_pool_open_packed format (src/st.c:127-180): header + slots; FP8
    bytes with exponent 15 are canonicalised on load."""
    L, E, H, M = 2, 8, 1024, 256
    m = dc.Model(fmt, L, H, M, E, 4)
    m.synth(2)
    nb = m.slot_bytes
    rng = np.random.default_rng(0)
    slots = rng.integers(0, 256, (L, E, nb), dtype=np.uint16).astype(np.uint8)
    for l_ in range(L):
        for e in range(E):
            src = po.Layer(fmt, H, M, 1, seed=100 + l_, layer=l_).experts[0] if e == 0 else None
            if src is not None:
                slots[l_, e] = src
    if fmt == dc.FMT_FP8:       # keep scale regions sane: real fp32 scales
        for t in range(3):
            n = (m.rel_v[t + 1] if t < 2 else nb) - m.rel_s[t]
            slots[:, :, m.rel_s[t]:m.rel_s[t] + n] = np.frombuffer(
                np.full(n // 4, 1e-3, np.float32).tobytes(), np.uint8)
    path = tmp_path / "pool.bin"
    with open(path, "wb") as f:
        f.write(np.array([nb, L, E], "<u8").tobytes())
        f.write(slots.tobytes())
    m.pool_load(str(path))
    for l_ in range(L):
        for e in range(E):
            got = m.get_expert(l_, e)
            want = slots[l_, e].copy()
            if fmt == dc.FMT_FP8:
                for t in range(3):
                    v = want[m.rel_v[t]:m.rel_s[t]]
                    e15 = (v & 0x78) == 0x78
                    v[e15] = (v[e15] & 0x80) | 0x7E
            assert np.array_equal(got, want)
    # a header that does not match the model is refused
    with open(path, "r+b") as f:
        f.write(np.array([nb + 16], "<u8").tobytes())
    with pytest.raises(dc.GpuError, match="header"):
        m.pool_load(str(path))
    m.close()


def test_memory_plan_refuses_oversized_pool():
    with pytest.raises(dc.GpuError, match="refusing"):
        dc.Model(dc.FMT_FP8, 4000, 2048, 512, 256, 8)


# ---- the persistent decode kernel (one cooperative launch per step) ----------

def _stack_path(m, x0, steps, path):
    m.set_path(path)
    return m.stack(x0, steps)


@pytest.mark.parametrize("fmt", [dc.FMT_FP8, dc.FMT_MXFP4])
@pytest.mark.parametrize("shape", [(1024, 256, 64, 4), (2048, 512, 256, 2)])
def test_persistent_matches_layered_and_oracle(fmt, shape):
    H, M, E, L = shape
    m = dc.Model(fmt, L, H, M, E, 8)
    m.synth(41)
    x0 = po.fill_f32(H, po.key(41, 0, 4, 0, 0), 1.0)
    got_p = _stack_path(m, x0, 2, dc.PATH_PERSISTENT)
    got_l = _stack_path(m, x0, 2, dc.PATH_LAYERED)
    assert relerr(got_p - x0, got_l - x0) < CHAIN_TOL
    # free-running oracle over the same 2 steps
    st = x0.copy()
    for s in range(2):
        for layer in range(L):
            lay = oracle_layer(m, layer, fmt, st)
            st, _, _, _, _ = lay.moe(st, 8)
    assert relerr(got_p - x0, st - x0) < CHAIN_TOL
    m.close()


def test_persistent_multi_step_launch_equals_single_steps():
    import torch
    m = dc.Model(dc.FMT_FP8, 3, 1024, 256, 64, 8)
    m.synth(5)
    m.set_path(dc.PATH_PERSISTENT)
    x0 = po.fill_f32(1024, po.key(5, 0, 4, 0, 0), 1.0)
    a = torch.from_numpy(x0.copy()).cuda()
    b = torch.from_numpy(x0.copy()).cuda()
    m.stack_dev(a, 4)                      # one launch, 4 steps
    for _ in range(4):
        m.stack_dev(b, 1)                  # four launches
    torch.cuda.synchronize()
    assert np.array_equal(a.cpu().numpy(), b.cpu().numpy())
    assert m.stats()[0] > 0
    m.close()


def test_persistent_tie_uses_exact_fallback():
    m = dc.Model(dc.FMT_FP8, 1, 1024, 256, 64, 8)
    m.synth(8)
    tr = m.get_trunk(0)
    x = po.fill_f32(1024, po.key(8, 0, 4, 0, 0), 1.0)
    lay = oracle_layer(m, 0, dc.FMT_FP8, x)
    idx, _, _, _ = lay.route(x, 8)
    a = int(idx[3])
    b = [e for e in range(64) if e not in idx and e > a][0]
    tr[1][b] = tr[1][a]
    m.set_trunk(0, *tr)
    m.set_path(dc.PATH_PERSISTENT)
    before = m.stats()[1]
    got = m.stack(x, 1)
    lay = oracle_layer(m, 0, dc.FMT_FP8, x, [a, b])
    st_o, idx_o, _, _, acc_o = lay.moe(x, 8)
    assert a in idx_o.tolist() and b in idx_o.tolist()
    assert m.stats()[1] > before
    assert relerr(got.astype(np.float64) - x, acc_o) < CHAIN_TOL
    m.close()


def test_persistent_router_exact_mode():
    m = dc.Model(dc.FMT_MXFP4, 2, 1024, 256, 64, 8, router_exact=True)
    m.synth(9)
    m.set_path(dc.PATH_PERSISTENT)
    x = po.fill_f32(1024, po.key(9, 0, 4, 0, 0), 1.0)
    got = m.stack(x, 1)
    st = x.copy()
    for layer in range(2):
        st, _, _, _, _ = oracle_layer(m, layer, dc.FMT_MXFP4, st).moe(st, 8)
    assert relerr(got - x, st - x) < CHAIN_TOL
    m.close()
