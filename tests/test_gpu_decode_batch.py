"""Batched decode (ds4f_gpu_moe_layer_batch_dev / _partial_dev /
ds4f_gpu_moe_stack_batch_dev) against the oracle, through the C ABI.

Per token the routing must be the reference's (src/main.c:1014-1088 +
ds4f_topk, src/moe.c:531-561, renormalised): indices bit-exact, weights
within 1e-5. The chain is the batched step on the tensor cores, checked
against two references fed the GPU's own weight bytes and routing:
  * orc_prefill_layer -- the GPU's arithmetic restated (3-digit E4M3
    activations): within 1e-4 of max |acc|;
  * orc_moe_batch_sel -- the reference's batched step with fp32 activations
    (src/moe.c:1480-1707): within the BASELINE chain tolerance 2e-3.
"""
import numpy as np
import pytest

from oracle import pyoracle as po
from tests._lib import ds4f_cuda

pytestmark = pytest.mark.gpu
dc = ds4f_cuda()
OWN_TOL = 1e-4
CHAIN_TOL = 2e-3
W_TOL = 1e-5


@pytest.fixture(scope="module", autouse=True)
def gpu():
    dc.init()
    yield


def relerr(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def oracle_layer(m, L, fmt, used):
    trunk = m.get_trunk(L)
    ex = np.zeros((m.E, m.slot_bytes), np.uint8)
    for e in sorted(set(int(v) for v in np.ravel(used))):
        ex[e] = m.get_expert(L, e)
    return po.Layer.from_arrays(fmt, m.H, m.M, m.E, trunk, ex)


def run_batch_layer(m, L, states):
    import torch
    B = states.shape[0]
    st = torch.from_numpy(states.copy()).cuda()
    idx = torch.full((B, m.K), -7, dtype=torch.int32, device="cuda")
    w = torch.zeros((B, m.K), dtype=torch.float32, device="cuda")
    m.layer_batch_dev(L, st, idx, w)
    return st.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy()


@pytest.mark.parametrize("fmt", [dc.FMT_FP8, dc.FMT_MXFP4])
@pytest.mark.parametrize("shape", [(1024, 256, 64, 8), (1024, 256, 64, 1), (2048, 512, 256, 8)])
def test_layer_batch_matches_oracle(shape, fmt):
    H, M, E, B = shape
    K = 8
    m = dc.Model(fmt, 2, H, M, E, K)
    m.synth(31)
    states = po.fill_f32(B * H, po.key(31, 0, 4, 0, 0), 1.0).reshape(B, H)
    got, gi, gw = run_batch_layer(m, 1, states)
    lay = oracle_layer(m, 1, fmt, gi)
    for b in range(B):
        ri, rw, _, _ = lay.route(states[b], K)
        assert np.array_equal(gi[b], ri), (b, gi[b], ri)
        assert relerr(gw[b], rw) < W_TOL
    own = lay.prefill(states, gi, gw)
    ref = lay.moe_batch_sel(states, gi, gw)
    acc = got.astype(np.float64) - states
    assert relerr(acc, own - states) < OWN_TOL
    assert relerr(acc, ref - states) < CHAIN_TOL
    m.close()


def test_stack_batch_equals_layer_steps():
    """ds4f_gpu_moe_stack_batch_dev (an eager step, then a captured step
    replayed, across calls) = the per-layer batched steps in order, bit for
    bit (row order inside an expert's group changes no result)."""
    import torch
    H, M, E, K, B, NL = 1024, 256, 64, 8, 6, 2
    m = dc.Model(dc.FMT_FP8, NL, H, M, E, K)
    m.synth(33)
    states = po.fill_f32(B * H, po.key(33, 0, 4, 0, 0), 1.0).reshape(B, H)
    a = torch.from_numpy(states.copy()).cuda()
    m.stack_batch_dev(a, 2)
    m.stack_batch_dev(a, 1)
    b = torch.from_numpy(states.copy()).cuda()
    for _ in range(3):
        for L in range(NL):
            m.layer_batch_dev(L, b)
    assert np.array_equal(a.cpu().numpy().view(np.uint32), b.cpu().numpy().view(np.uint32))
    m.close()


def test_batch_partial_shards_sum_to_full_step():
    """Two expert shards' partial steps (the shared expert on the first)
    add up to the full batched step."""
    import torch
    H, M, E, K, B = 1024, 256, 64, 8, 8
    full = dc.Model(dc.FMT_FP8, 1, H, M, E, K)
    full.synth(35)
    shards = [dc.Model(dc.FMT_FP8, 1, H, M, E, K, expert_first=r * E // 2, expert_count=E // 2) for r in range(2)]
    for s in shards:
        s.synth(35)
    states = po.fill_f32(B * H, po.key(35, 0, 4, 0, 0), 1.0).reshape(B, H)
    st = torch.from_numpy(states.copy()).cuda()
    acc = torch.zeros_like(st)
    for r, s in enumerate(shards):
        part = torch.zeros_like(st)
        s.layer_batch_partial_dev(0, st, part, r == 0)
        acc += part
    assert np.array_equal(st.cpu().numpy(), states)          # partial steps leave the states alone
    want, _, _ = run_batch_layer(full, 0, states)
    assert relerr(acc.cpu().numpy(), want - states) < 1e-5
    for s in shards + [full]:
        s.close()
