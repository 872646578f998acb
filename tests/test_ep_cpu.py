"""Expert-parallel decode (disk-qwen35ba3b_b200/ep.py) on CPU ranks: two gloo
processes, each holding half of the experts, drive the same decoder as the
GPUs with an oracle backend (the per-rank partial restated from the
oracle's own pieces); the result must equal the single-host oracle step
(orc_moe_layer) within fp32 reassociation of the combine."""
import importlib.util
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import pyoracle as po

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
H, M, E, K, NL, B = 256, 128, 16, 4, 2, 3
TOL = 1e-5


def _ep_module():
    spec = importlib.util.spec_from_file_location("ep", os.path.join(ROOT, "disk-qwen35ba3b_b200", "ep.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class OracleShard:
    """The per-rank partial step, from oracle pieces: route on the full
    state, this shard's chains in selection order, the shared expert."""

    def __init__(self, layers, first, count):
        self.layers, self.first, self.count = layers, first, count
        self.n_layers, self.hidden = len(layers), H

    def layer_partial(self, L, states, acc, add_shared, stream=None):
        lay = self.layers[L]
        for b in range(states.shape[0]):
            idx, w, _, xin = lay.route(states[b].numpy(), K)
            a = np.zeros(H, np.float32)
            for j in range(K):
                e = int(idx[j])
                if not (self.first <= e < self.first + self.count):
                    continue
                out = np.zeros(H, np.float32)
                po.lib().orc_expert_chain(lay.fmt, po.ptr(lay.experts[e]), po.C.byref(lay.lay), H, M,
                                          po.ptr(xin), po.ptr(out))
                a = (a + np.float32(w[j]) * out).astype(np.float32)
            if add_shared:
                lw = lay.w()
                po.lib().orc_shared_add(po.C.byref(lw), H, M, po.ptr(xin), po.ptr(a))
            acc[b] = torch.from_numpy(a)


def _layers():
    return [po.Layer(po.FMT_FP8, H, M, E, seed=3, layer=L, sigma=0.05) for L in range(NL)]


def _rank(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ep = _ep_module()
    first, count = ep.shard_of(rank, world, E)
    dec = ep.ExpertParallelDecoder(OracleShard(_layers(), first, count))
    st = torch.from_numpy(po.fill_f32(B * H, po.key(3, 0, 4, 0, 0), 1.0).reshape(B, H).copy())
    dec.step(st)
    out[rank] = st.numpy().copy()
    dist.barrier()
    dist.destroy_process_group()


def test_shard_of():
    ep = _ep_module()
    assert ep.shard_of(3, 8, 256) == (96, 32)
    with pytest.raises(ValueError):
        ep.shard_of(0, 3, 256)


def test_expert_parallel_decode_two_ranks_matches_single_host():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    got0, got1 = out[0], out[1]
    assert np.array_equal(got0, got1)                 # every rank holds the same state
    want = po.fill_f32(B * H, po.key(3, 0, 4, 0, 0), 1.0).reshape(B, H).copy()
    for L, lay in enumerate(_layers()):
        for b in range(B):
            want[b], _, _, _, _ = lay.moe(want[b], K)
    err = np.abs(got0 - want).max() / np.abs(want).max()
    assert err < TOL, err


# ---- expert-parallel prefill ------------------------------------------------

T_PF = 6


class OraclePrefillShard:
    """Per-rank partial of the batched step, from the oracle's reference
    batched step (orc_moe_batch_sel): the shard's selections (others -1),
    minus the shared expert's part on ranks other than 0."""

    def __init__(self, layers, first, count):
        self.layers, self.first, self.count = layers, first, count
        self.n_layers, self.hidden = len(layers), H

    def prefill_partial(self, L, states, sel, w, acc, add_shared, stream=None):
        lay = self.layers[L]
        st = states.numpy()
        s = sel.numpy().copy()
        s[(s < self.first) | (s >= self.first + self.count)] = -1
        part = lay.moe_batch_sel(st, s, w.numpy()) - st
        if not add_shared:
            part = part - (lay.moe_batch_sel(st, np.full_like(s, -1), w.numpy()) - st)
        acc.copy_(torch.from_numpy(part.astype(np.float32)))


def _routing_pf():
    rng = np.random.default_rng(5)
    sel = np.stack([np.stack([rng.choice(E, K, replace=False) for _ in range(T_PF)]) for _ in range(NL)])
    w = rng.random((NL, T_PF, K)).astype(np.float32)
    w /= w.sum(-1, keepdims=True)
    return sel.astype(np.int32), w.astype(np.float32)


def _rank_pf(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ep = _ep_module()
    first, count = ep.shard_of(rank, world, E)
    pf = ep.ExpertParallelPrefill(OraclePrefillShard(_layers(), first, count))
    st = torch.from_numpy(po.fill_f32(T_PF * H, po.key(4, 0, 4, 0, 0), 1.0).reshape(T_PF, H).copy())
    sel, w = _routing_pf()
    pf.step(st, torch.from_numpy(sel), torch.from_numpy(w))
    out[rank] = st.numpy().copy()
    dist.barrier()
    dist.destroy_process_group()


def test_expert_parallel_prefill_two_ranks_matches_single_host():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    procs = [ctx.Process(target=_rank_pf, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert np.array_equal(out[0], out[1])
    want = po.fill_f32(T_PF * H, po.key(4, 0, 4, 0, 0), 1.0).reshape(T_PF, H).copy()
    sel, w = _routing_pf()
    for L, lay in enumerate(_layers()):
        want = lay.moe_batch_sel(want, sel[L], w[L])
    err = np.abs(out[0] - want).max() / np.abs(want).max()
    assert err < TOL, err
