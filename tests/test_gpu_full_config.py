"""The configurations the bench times, at their own sizes, against the oracle.

* BASELINE config 2 (40-layer FP8 stack, H 2048, M 512, E 256, top-8) and
  config 3 at batch 1 (the same stack with MXFP4 experts): the persistent
  decode kernel runs 4 free-running steps (160 layer-steps) in one call with
  its route log on; every layer-step is checked against the oracle twice:
    - fed the GPU's own input state: indices bit-exact, weights within 1e-5,
      the layer's acc (output - input state) within the 2e-3 chain tolerance;
    - on the oracle's own free-running trajectory from the same x0: indices
      equal at every layer, states within the chain tolerance.
* BASELINE config 4 (2048-token chunk, Zipf(1.1) expert load): one prefill
  layer at full size with the bench's own routing (every expert touched, the
  hottest with more than 1,000 rows, so multi-tile experts and the
  persistent GEMM's item walk run); a sample of tokens spread over the hot
  expert's rows and over the rest is checked against orc_prefill_layer (the
  GPU's arithmetic, 1e-4) and orc_moe_batch_sel (the reference's batched
  step with fp32 activations, 2e-3). A token's output depends only on its
  own state, selections and weights, so the sample is exact as a check.
"""
import numpy as np
import pytest

from oracle import pyoracle as po
from tests._lib import ds4f_cuda

pytestmark = pytest.mark.gpu
dc = ds4f_cuda()
CHAIN_TOL = 2e-3
OWN_TOL = 1e-4
W_TOL = 1e-5
H, M, E, K, LAYERS = 2048, 512, 256, 8, 40


@pytest.fixture(scope="module", autouse=True)
def gpu():
    dc.init()
    yield


def relerr(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def layer_of(m, L, fmt, experts):
    trunk = m.get_trunk(L)
    ex = np.zeros((m.E, m.slot_bytes), np.uint8)          # lazily committed pages
    for e in sorted(set(int(v) for v in experts if v >= 0)):
        ex[e] = m.get_expert(L, e)
    return po.Layer.from_arrays(fmt, m.H, m.M, m.E, trunk, ex)


@pytest.mark.parametrize("fmt", [dc.FMT_FP8, dc.FMT_MXFP4], ids=["config2-fp8", "config3-mxfp4-b1"])
def test_decode_40_layers_free_running(fmt):
    steps = 4
    n = steps * LAYERS
    m = dc.Model(fmt, LAYERS, H, M, E, K)
    m.synth(0)
    m.set_path(dc.PATH_PERSISTENT)
    m.route_log(n)
    x0 = po.fill_f32(H, po.key(0, 0, 4, 0, 0), 1.0)
    got = m.stack(x0, steps)                                # one launch, 160 layer-steps
    idx_g, w_g, st_g = m.route_log_read(n)
    assert np.array_equal(got, st_g[-1])
    st_free = x0.copy()
    for t in range(n):
        L = t % LAYERS
        s_in = x0 if t == 0 else st_g[t - 1]
        lay = layer_of(m, L, fmt, idx_g[t])
        # the oracle's own routing must pick the experts the GPU logged
        _, idx_o, w_o, _, acc_o = lay.moe(s_in, K)
        assert np.array_equal(idx_g[t], idx_o), (t, idx_g[t], idx_o)
        assert relerr(w_g[t], w_o) < W_TOL, t
        assert relerr(st_g[t].astype(np.float64) - s_in, acc_o) < CHAIN_TOL, t
        # free-running oracle trajectory: same selections at every layer
        ix, _, _, _ = lay.route(st_free, K)
        if not np.array_equal(ix, idx_g[t]):
            lay = layer_of(m, L, fmt, ix)
        st_free, idx_f, _, _, _ = lay.moe(st_free, K)
        assert np.array_equal(idx_f, idx_g[t]), (t, idx_f, idx_g[t])
        assert relerr(st_g[t] - x0, st_free - x0) < CHAIN_TOL, t
    m.route_log(0)
    m.close()


def test_prefill_layer_2048_token_zipf():
    """Config 4 at full size, FP8 and MXFP4 pools, layer 3 of the stack."""
    import torch
    from bench import zipf_routing
    T, L = 2048, 3
    sel_all, w_all = zipf_routing(L + 1, T, E, K, seed=100)
    sel, w = sel_all[L], w_all[L]
    load = np.bincount(sel.ravel(), minlength=E)
    assert load.min() > 0 and load.max() > 1000, (load.min(), load.max())
    hot = int(np.argmax(load))
    rows_hot = np.nonzero((sel == hot).any(1))[0]
    rng = np.random.default_rng(3)
    sample = np.unique(np.concatenate([rows_hot[:4], rows_hot[-4:],
                                       rng.choice(rows_hot, 40, replace=False),
                                       rng.choice(T, 40, replace=False),
                                       np.nonzero((sel == int(np.argmin(load))).any(1))[0]]))
    states = po.fill_f32(T * H, po.key(0, 0, 4, 0, 1), 1.0).reshape(T, H)
    states = torch.from_numpy(states).bfloat16().float().numpy()     # bf16 activations, as the bench
    for fmt in (dc.FMT_FP8, dc.FMT_MXFP4):
        m = dc.Model(fmt, L + 1, H, M, E, K)
        m.synth(0)
        st = torch.from_numpy(states.copy()).cuda()
        m.prefill_layer_dev(L, st, torch.from_numpy(sel).cuda(), torch.from_numpy(w).cuda())
        got = st.cpu().numpy()
        assert np.isfinite(got).all()
        lay = layer_of(m, L, fmt, sel[sample].ravel())
        own = lay.prefill(states[sample], sel[sample], w[sample])
        ref = lay.moe_batch_sel(states[sample], sel[sample], w[sample])
        acc = got[sample].astype(np.float64) - states[sample]
        assert relerr(acc, own - states[sample]) < OWN_TOL, fmt
        assert relerr(acc, ref - states[sample]) < CHAIN_TOL, fmt
        m.close()


@pytest.mark.parametrize("path", [dc.PATH_LAYERED, dc.PATH_PERSISTENT])
def test_nan_state_routes_like_the_reference(path):
    """A NaN in the state makes every router logit NaN; the reference's
    insertion top-k (src/moe.c:531-546) then selects experts 0..K-1. Both
    decode paths must return exactly that (every index valid)."""
    Hs, Ms, Es = 1024, 256, 64
    m = dc.Model(dc.FMT_FP8, 2, Hs, Ms, Es, K)
    m.synth(4)
    m.set_path(path)
    x = po.fill_f32(Hs, po.key(4, 0, 4, 0, 0), 1.0)
    x[17] = np.nan
    lay = layer_of(m, 0, dc.FMT_FP8, range(K))
    idx_o, _, _, _ = lay.route(x, K)
    assert idx_o.tolist() == list(range(K))
    if path == dc.PATH_LAYERED:
        _, idx_g, _ = m.layer(0, x)
    else:
        m.route_log(2)
        m.stack(x, 1)
        idx_log, _, _ = m.route_log_read(2)
        idx_g = idx_log[0]
        assert idx_log[1].tolist() == list(range(K))        # the NaN state carries on
        m.route_log(0)
    assert idx_g.tolist() == list(range(K))
    m.close()
