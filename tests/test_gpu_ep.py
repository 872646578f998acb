"""Expert-parallel decode on 2 GPUs (one process per GPU, NCCL): each rank
holds half of every layer's experts; after each step every rank's state
equals the single-GPU full model's within fp32 reassociation of the combine
(the partial sums meet in the all-reduce): one token against the per-token
layer steps, a batch against the batched (tensor-core) stack, which is in
turn within the chain tolerance of the per-token fp32 path. Skipped with
fewer than 2 GPUs."""
import importlib.util
import os

import numpy as np
import pytest

from oracle import pyoracle as po
from tests._lib import ds4f_cuda, gpu_available

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
H, M, E, K, NL = 1024, 256, 64, 8, 3
REASSOC_TOL = 1e-5
CHAIN_TOL = 2e-3


def _ngpu():
    if not gpu_available():
        return 0
    import torch
    return torch.cuda.device_count()


def _ep_module():
    spec = importlib.util.spec_from_file_location("ep", os.path.join(ROOT, "disk-qwen35ba3b_b200", "ep.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _x0(B):
    return po.fill_f32(B * H, po.key(21, 0, 4, 0, 0), 1.0).reshape(B, H).copy()


def _init(rank, world, port):
    """The caller's process group carries only the communicator id (gloo):
    the data plane is the library's NCCL."""
    import datetime
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    dc = ds4f_cuda()
    dc.init()
    return dc, dist


def _rank(rank, world, port, fmt, B, out):
    import torch
    dc, dist = _init(rank, world, port)
    ep = _ep_module()
    shard = ep.GpuShard(dc, fmt, NL, H, M, E, K, rank, world, seed=21)
    shard.attach()
    st = torch.from_numpy(_x0(B)).cuda()
    sp = torch.cuda.current_stream().cuda_stream
    shard.decode(st, 1, sp)                  # eager first step
    shard.decode(st, 2, sp)                  # then the captured step, twice
    torch.cuda.synchronize()
    out[rank] = st.cpu().numpy()
    shard.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(_ngpu() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("B", [1, 2])
@pytest.mark.parametrize("fmt", [2, 0])            # FP8, MXFP4
def test_expert_parallel_two_gpus(fmt, B):
    import socket
    import torch
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, fmt, B, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    assert np.array_equal(out[0], out[1])
    # the single-GPU full model (two steps): per-token layer steps, and for
    # a batch the batched stack
    dc = ds4f_cuda()
    dc.init()
    m = dc.Model(fmt, NL, H, M, E, K)
    m.synth(21)
    m.set_path(dc.PATH_LAYERED)
    x0 = _x0(B)
    exact = np.stack([m.stack(x0[b], 3) for b in range(B)])
    want = exact
    if B > 1:
        st = torch.from_numpy(x0.copy()).cuda()
        m.stack_batch_dev(st, 3)
        want = st.cpu().numpy()
        assert np.abs(want - exact).max() / np.abs(exact - x0).max() < CHAIN_TOL
    m.close()
    err = np.abs(out[0] - want).max() / np.abs(want - x0).max()
    assert err < REASSOC_TOL, err


# ---- expert-parallel prefill ------------------------------------------------

T_PF = 96


def _routing_pf():
    rng = np.random.default_rng(7)
    sel = np.stack([np.stack([rng.choice(E, K, replace=False) for _ in range(T_PF)]) for _ in range(NL)])
    w = rng.random((NL, T_PF, K)).astype(np.float32)
    w /= w.sum(-1, keepdims=True)
    return sel.astype(np.int32), w.astype(np.float32)


def _x0_pf():
    return po.fill_f32(T_PF * H, po.key(23, 0, 4, 0, 0), 1.0).reshape(T_PF, H).copy()


SPLIT = (60, 36)          # tokens per rank: uneven on purpose


def _rank_pf(rank, world, port, fmt, out):
    import torch
    dc, dist = _init(rank, world, port)
    ep = _ep_module()
    shard = ep.GpuShard(dc, fmt, NL, H, M, E, K, rank, world, seed=23)
    shard.attach()
    sel, w = _routing_pf()
    t0 = sum(SPLIT[:rank])
    t1 = t0 + SPLIT[rank]
    st = torch.from_numpy(_x0_pf()[t0:t1].copy()).cuda()
    shard.prefill(st, torch.from_numpy(np.ascontiguousarray(sel[:, t0:t1])).cuda(),
                  torch.from_numpy(np.ascontiguousarray(w[:, t0:t1])).cuda(),
                  torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    out[rank] = st.cpu().numpy()
    shard.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(_ngpu() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("fmt", [2, 0])            # FP8, MXFP4
def test_token_parallel_prefill_two_gpus(fmt):
    """Tokens partitioned 60 / 36 over two GPUs, each holding half of the
    experts; rows dispatched to the experts' GPUs and combined back by the
    library (NCCL send/recv). Every token equals the single-GPU prefill of
    the whole chunk within fp32 reassociation of the combine."""
    import socket
    import torch
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    procs = [ctx.Process(target=_rank_pf, args=(r, 2, port, fmt, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    dc = ds4f_cuda()
    dc.init()
    m = dc.Model(fmt, NL, H, M, E, K)
    m.synth(23)
    sel, w = _routing_pf()
    x0 = _x0_pf()
    st = torch.from_numpy(x0.copy()).cuda()
    m.prefill_dev(st, torch.from_numpy(sel).cuda(), torch.from_numpy(w).cuda())
    want = st.cpu().numpy()
    m.close()
    got = np.concatenate([out[0], out[1]])
    err = np.abs(got - want).max() / np.abs(want - x0).max()
    assert err < REASSOC_TOL, err
