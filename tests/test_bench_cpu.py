"""bench.py's host-side pieces on CPU: the k_decode phase table over a
synthetic trace (every stamp slot the kernel writes, the multi-GPU rows
included), the synthetic Zipf routing of config 4, and the decode config
both bench arms print."""
import numpy as np

import bench


def _trace(L=3, G=5):
    """Stamps that grow along the layer in the order the kernel writes them."""
    order = [0, 1, 2, 3, 18, 27, 28, 29, 30, 31, 4, 5, 6, 7, 8, 21, 22, 23, 24, 25, 9, 10, 12, 26, 13, 19, 20, 11]
    tr = np.zeros((L, G, bench.N_STAMPS), np.int64)
    for layer in range(L):
        for c in range(G):
            t = 100_000 * layer + 7 * c
            for k in order:
                t += 100 + 10 * k
                tr[layer, c, k] = t
            tr[layer, c, 14:17] = [1, 2, 1]          # copy rounds
            tr[layer, c, 17] = 0b0011                # groups landed early
    return tr


def test_phase_table_every_row():
    out = bench.phase_table(_trace(), ep=True)
    names = [n for n, _, _ in out["phases_us"]]
    for want in ["start -> state", "down: chain gather", "routes: top-8 network", "routes: group 0 issue",
                 "  +gate/up: group 3 landed", "down: first row-dot pair", "ep: peers' rows arrived"]:
        assert want in names, want
    for _, med, mx in out["phases_us"]:
        assert np.isfinite(med) and np.isfinite(mx) and med >= 0.0
    assert out["gather_rounds_mean"] == {"state": 1.0, "router": 2.0, "chains": 1.0}
    assert out["group_landed_early"] == [1.0, 1.0, 0.0, 0.0]
    assert out["layer_period_us"]["median"] == 100.0


def test_zipf_routing_shape_and_load():
    sel, w = bench.zipf_routing(2, 2048, 256, 8, seed=100)
    assert sel.shape == (2, 2048, 8) and w.shape == (2, 2048, 8)
    for L in range(2):
        assert all(len(set(r)) == 8 for r in sel[L])              # K distinct experts per token
        load = np.bincount(sel[L].ravel(), minlength=256)
        assert load.max() > 1000 and load.min() >= 1              # every expert touched, a hot one
    assert np.allclose(w.sum(-1), 1.0, atol=1e-6)


def test_decode_config_same_in_both_arms():
    a = bench.decode_config(True, 1)
    b = bench.decode_config(True, 1)
    assert a == b and a["layers"] == 40 and a["experts"] == 256 and a["topk"] == 8
    assert bench.bytes_per_token(True) == 40 * 32_520_192
