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


# ---- the fused one-token step's algorithm: rows exchanged, combined in order --

class OracleSelections:
    """Backend of ep.SelectionExchangeDecoder from oracle pieces: the
    oracle's own routing (orc_moe_layer's, so indices and weights carry the
    same bits), one expert chain, the shared expert add."""

    def __init__(self, layers):
        self.layers = layers
        self.n_layers, self.hidden, self.n_experts = len(layers), H, E

    def route(self, L, x):
        lay = self.layers[L]
        _, idx, w, _, _ = lay.moe(x, K)
        xin = np.array(x, np.float32, copy=True)
        po.lib().orc_rmsnorm(po.ptr(lay.norm), H, po.ptr(xin))
        return idx, w, xin

    def chain(self, L, e, xin):
        lay = self.layers[L]
        out = np.zeros(H, np.float32)
        po.lib().orc_expert_chain(lay.fmt, po.ptr(lay.experts[e]), po.C.byref(lay.lay), H, M,
                                  po.ptr(xin), po.ptr(out))
        return out

    def shared_add(self, L, xin, acc):
        lw = self.layers[L].w()
        po.lib().orc_shared_add(po.C.byref(lw), H, M, po.ptr(xin), po.ptr(acc))


def _rank_sel(rank, world, port, by_index, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ep = _ep_module()
    dec = ep.SelectionExchangeDecoder(OracleSelections(_layers()), by_index=by_index)
    st = torch.from_numpy(po.fill_f32(B * H, po.key(3, 0, 4, 0, 0), 1.0).reshape(B, H).copy())
    dec.step(st)
    out[rank] = st.numpy().copy()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("by_index", [False, True], ids=["by-expert-owner", "by-selection-index"])
def test_selection_exchange_two_ranks_bit_exact(by_index):
    """Two gloo ranks run the fused step's algorithm (each rank its own
    selections' chains, the rows exchanged, every row combined in selection
    order on every rank): both ranks hold exactly the single-host oracle's
    bits after every layer, with the selections split by expert owner (half
    of the experts per rank) or by index (every expert on every rank)."""
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    procs = [ctx.Process(target=_rank_sel, args=(r, 2, port, by_index, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    want = po.fill_f32(B * H, po.key(3, 0, 4, 0, 0), 1.0).reshape(B, H).copy()
    for lay in _layers():
        for b in range(B):
            want[b], _, _, _, _ = lay.moe(want[b], K)
    for r in (0, 1):
        assert np.array_equal(out[r].view(np.uint32), want.view(np.uint32))


def test_selection_owner():
    ep = _ep_module()
    idx = np.array([3, 12, 7, 9, 0, 15, 8, 1])
    assert [ep.selection_owner(j, idx, 16, 2, False) for j in range(8)] == [0, 1, 0, 1, 0, 1, 1, 0]
    assert [ep.selection_owner(j, idx, 16, 2, True) for j in range(8)] == [0, 0, 0, 0, 1, 1, 1, 1]
    assert [ep.selection_owner(j, idx, 16, 3, True) for j in range(8)] == [0, 0, 1, 1, 1, 2, 2, 2]
    assert [ep.selection_owner(j, idx, 16, 8, True) for j in range(8)] == list(range(8))


# ---- token-parallel prefill with all-to-all dispatch / combine ----------------

T_PF = 7                 # tokens per rank (rank 1 holds T_PF - 2: uneven on purpose)


def _dc():
    spec = importlib.util.spec_from_file_location("ds4f_cuda", os.path.join(ROOT, "disk-qwen35ba3b_b200",
                                                                            "ds4f_cuda.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class OracleTokenShard:
    """One rank of the token-parallel prefill from oracle pieces: each
    received row's partial combine over this rank's experts (its own
    RMSNorm, the chains in selection order), and the shared expert of the
    rank's own tokens."""

    def __init__(self, layers, first, count):
        self.layers, self.first, self.count = layers, first, count
        self.n_layers, self.hidden = len(layers), H

    def _xin(self, lay, st):
        xin = np.array(st, np.float32, copy=True)
        po.lib().orc_rmsnorm(po.ptr(lay.norm), H, po.ptr(xin))
        return xin

    def rows_partial(self, L, states, sel, w):
        lay = self.layers[L]
        out = np.zeros((states.shape[0], H), np.float32)
        for i in range(states.shape[0]):
            xin = self._xin(lay, states[i].numpy())
            a = np.zeros(H, np.float32)
            for j in range(K):
                e = int(sel[i, j])
                if not (self.first <= e < self.first + self.count):
                    continue
                o = np.zeros(H, np.float32)
                po.lib().orc_expert_chain(lay.fmt, po.ptr(lay.experts[e]), po.C.byref(lay.lay), H, M,
                                          po.ptr(xin), po.ptr(o))
                a = (a + np.float32(w[i, j]) * o).astype(np.float32)
            out[i] = a
        return torch.from_numpy(out)

    def shared(self, L, states):
        lay = self.layers[L]
        out = np.zeros((states.shape[0], H), np.float32)
        lw = lay.w()
        for t in range(states.shape[0]):
            xin = self._xin(lay, states[t].numpy())
            po.lib().orc_shared_add(po.C.byref(lw), H, M, po.ptr(xin), po.ptr(out[t]))
        return torch.from_numpy(out)


def _tokens_pf(rank):
    T = T_PF if rank == 0 else T_PF - 2
    x = po.fill_f32(T * H, po.key(4, 0, 4, rank, 0), 1.0).reshape(T, H).copy()
    rng = np.random.default_rng(5 + rank)
    # every token on rank 1's experts for layer 0 and on rank 0's for layer
    # 1 of rank 1's tokens: some peers receive nothing from a rank
    sel = np.stack([np.stack([rng.choice(E, K, replace=False) for _ in range(T)]) for _ in range(NL)])
    if rank == 1:
        sel[0] = np.stack([rng.choice(np.arange(E // 2, E), K, replace=False) for _ in range(T)])
    sel[0, 0, 3] = -1                                    # a skipped selection
    w = rng.random((NL, T, K)).astype(np.float32)
    w /= w.sum(-1, keepdims=True)
    return x, sel.astype(np.int32), w.astype(np.float32)


def _rank_pf(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ep = _ep_module()
    dc = _dc()
    first, count = ep.shard_of(rank, world, E)
    pf = ep.TokenParallelPrefill(OracleTokenShard(_layers(), first, count), dc.ep_plan_dispatch, E)
    x, sel, w = _tokens_pf(rank)
    st = torch.from_numpy(x)
    pf.step(st, torch.from_numpy(sel), torch.from_numpy(w))
    out[rank] = st.numpy().copy()
    dist.barrier()
    dist.destroy_process_group()


def test_token_parallel_prefill_two_ranks_matches_single_host():
    """Each rank's tokens, after every layer of the all-to-all prefill, equal
    the single-host reference batched step (orc_moe_batch_sel) on the same
    tokens within fp32 reassociation of the combine."""
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
        p.join(180)
        assert p.exitcode == 0
    for r in range(2):
        x, sel, w = _tokens_pf(r)
        want = x.copy()
        for L, lay in enumerate(_layers()):
            want = lay.moe_batch_sel(want, sel[L], w[L])
        err = np.abs(out[r] - want).max() / np.abs(want - x).max()
        assert err < TOL, (r, err)


def test_dispatch_plan():
    """ds4f_ep_plan_dispatch (host only) against a direct restatement:
    random routing, skipped selections, a rank nobody selects, one token,
    none, and the refusals."""
    dc = _dc()
    rng = np.random.default_rng(2)
    for T, Kp, Ep, N in [(37, 8, 64, 4), (1, 8, 64, 8), (0, 8, 64, 2), (50, 4, 16, 16), (20, 8, 256, 1)]:
        sel = np.array([rng.choice(Ep // 2 if N > 1 else Ep, Kp, replace=False) for _ in range(T)],
                       np.int32).reshape(T, Kp)
        if T:
            sel[rng.random(sel.shape) < 0.1] = -1
        counts, rows, tok = dc.ep_plan_dispatch(sel, Ep, N)
        per = Ep // N
        need = np.zeros((T, N), bool)
        for t in range(T):
            for e in sel[t]:
                if e >= 0:
                    need[t, e // per] = True
        want_rows = [t for d in range(N) for t in range(T) if need[t, d]]
        assert counts.tolist() == need.sum(0).tolist()
        assert rows.tolist() == want_rows
        for t in range(T):
            for d in range(N):
                i = tok[t, d]
                assert (i >= 0) == need[t, d]
                if i >= 0:
                    assert rows[i] == t and sum(counts[:d]) <= i < sum(counts[:d + 1])
        if N > 1:
            assert counts[N - 1] == 0                     # the upper half of the experts is never selected
    with pytest.raises(dc.GpuError, match="expert 64 of 64"):
        dc.ep_plan_dispatch(np.full((2, 4), 64, np.int32), 64, 4)
    with pytest.raises(dc.GpuError):
        dc.ep_plan_dispatch(np.zeros((2, 4), np.int32), 64, 3)            # 64 experts over 3 ranks
