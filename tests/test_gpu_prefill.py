"""Batched prefill on the tensor cores (ds4f_gpu_moe_prefill /
ds4f_gpu_prefill) against the oracle, through the C ABI.

Two references, both fed the GPU's own weight bytes:
  * orc_prefill_layer -- the GPU prefill's arithmetic restated (the same
    3-digit E4M3 activations, bf16 hi/lo digits in the shared expert; FP8
    weights with their block scales in the promotion, MXFP4 weights exactly
    dequantised as the block-scaled MMA reads them): within 1e-4 of max |acc|
    (block-sum order and CUDA vs libm exp only);
  * orc_moe_batch_sel -- the reference's batched step with fp32
    activations (src/moe.c:1480-1707): within the BASELINE chain tolerance
    2e-3 of max |acc|.
"""
import numpy as np
import pytest

from oracle import pyoracle as po
from tests._lib import ds4f_cuda

pytestmark = pytest.mark.gpu
dc = ds4f_cuda()
OWN_TOL = 1e-4
CHAIN_TOL = 2e-3


@pytest.fixture(scope="module", autouse=True)
def gpu():
    dc.init()
    yield


def relerr(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def routing(T, K, experts, seed, hot=None):
    """K distinct experts per token from `experts` (Zipf-skewed), softmax
    weights renormalised over the K (float32)."""
    rng = np.random.default_rng(seed)
    experts = np.asarray(experts)
    p = 1.0 / np.arange(1, len(experts) + 1) ** 1.1
    p /= p.sum()
    sel = np.zeros((T, K), np.int32)
    for t in range(T):
        sel[t] = rng.choice(experts, size=K, replace=False, p=p)
        if hot is not None and hot not in sel[t]:
            sel[t, 0] = hot
    logits = rng.normal(size=(T, K)).astype(np.float32)
    w = np.exp(logits - logits.max(1, keepdims=True)).astype(np.float32)
    w /= w.sum(1, keepdims=True)
    return sel, w.astype(np.float32)


def oracle_layer(m, L, used, fmt=None):
    trunk = m.get_trunk(L)
    ex = np.zeros((m.E, m.slot_bytes), np.uint8)
    for e in sorted(set(int(v) for v in used if v >= 0)):
        ex[e] = m.get_expert(L, e)
    return po.Layer.from_arrays(dc.FMT_FP8 if fmt is None else fmt, m.H, m.M, m.E, trunk, ex)


def run_layer(m, L, states, sel, w):
    import torch
    st = torch.from_numpy(states.copy()).cuda()
    m.prefill_layer_dev(L, st, torch.from_numpy(sel).cuda(), torch.from_numpy(w).cuda())
    return st.cpu().numpy()


@pytest.mark.parametrize("fmt", [dc.FMT_FP8, dc.FMT_MXFP4])
@pytest.mark.parametrize("shape", [(1024, 256, 64, 80), (2048, 512, 256, 20)])
def test_prefill_layer_matches_oracle(shape, fmt):
    H, M, E, T = shape
    K = 8
    m = dc.Model(fmt, 2, H, M, E, K)
    m.synth(7)
    states = po.fill_f32(T * H, po.key(7, 0, 4, 0, 0), 1.0).reshape(T, H)
    sel, w = routing(T, K, np.arange(0, E, max(1, E // 24)), seed=1, hot=0)   # expert 0 in every token
    sel[3, 5] = -1                                   # a skipped selection
    w[4, 2] = 0.0                                    # a zero weight
    got = run_layer(m, 1, states, sel, w)
    lay = oracle_layer(m, 1, sel.ravel(), fmt)
    own = lay.prefill(states, sel, w)
    ref = lay.moe_batch_sel(states, sel, w)
    acc = got.astype(np.float64) - states
    assert relerr(acc, own - states) < OWN_TOL
    assert relerr(acc, ref - states) < CHAIN_TOL
    m.close()


def test_prefill_stack_two_layers():
    import torch
    H, M, E, K, T, NL = 1024, 256, 64, 8, 48, 2
    m = dc.Model(dc.FMT_FP8, NL, H, M, E, K)
    m.synth(9)
    states = po.fill_f32(T * H, po.key(9, 0, 4, 0, 0), 1.0).reshape(T, H)
    sels, ws = zip(*[routing(T, K, np.arange(E), seed=10 + L) for L in range(NL)])
    sel = np.stack(sels)
    w = np.stack(ws)
    st = torch.from_numpy(states.copy()).cuda()
    m.prefill_dev(st, torch.from_numpy(sel).cuda(), torch.from_numpy(w).cuda())
    got = st.cpu().numpy()
    want = states.copy()
    for L in range(NL):
        want = oracle_layer(m, L, sel[L].ravel()).prefill(want, sel[L], w[L])
    assert relerr(got - states, want - states) < OWN_TOL
    m.close()


def test_prefill_mxfp4_wide_exponent_spread():
    """MXFP4 experts whose four E8M0 sub-block scales in each 128-column block
    lie up to 14 binades apart (offsets -9, 0, +2, -12 on the synthetic
    scales): legal MXFP4 that the reference decodes (src/kernels.c:34-62),
    read by the block-scaled MMA as stored. The layer must match both
    references as for ordinary pools."""
    H, M, E, K, T = 1024, 256, 64, 8, 48
    m = dc.Model(dc.FMT_MXFP4, 1, H, M, E, K)
    m.synth(31)
    offs = np.array([-9, 0, 2, -12], np.int16)
    ends = [m.rel_v[1], m.rel_v[2], m.slot_bytes]
    for e in range(16):
        slot = m.get_expert(0, e).copy()
        for t in range(3):
            sc = slot[m.rel_s[t]:ends[t]].astype(np.int16)
            sc = np.clip(sc + np.resize(offs, sc.size), 1, 254)
            slot[m.rel_s[t]:ends[t]] = sc.astype(np.uint8)
        m.set_expert(0, e, slot)
    states = po.fill_f32(T * H, po.key(31, 0, 4, 0, 0), 1.0).reshape(T, H)
    sel, w = routing(T, K, np.arange(16), seed=4)
    got = run_layer(m, 0, states, sel, w)
    lay = oracle_layer(m, 0, sel.ravel(), dc.FMT_MXFP4)
    sv = lay.experts[sel[0, 0]]
    spread = np.ptp(sv[m.rel_s[0]:m.rel_v[1]].reshape(-1, 4).astype(int), axis=1)
    assert spread.max() > 6
    own = lay.prefill(states, sel, w)
    ref = lay.moe_batch_sel(states, sel, w)
    acc = got.astype(np.float64) - states
    assert np.isfinite(got).all()
    assert relerr(acc, own - states) < OWN_TOL
    assert relerr(acc, ref - states) < CHAIN_TOL
    m.close()
