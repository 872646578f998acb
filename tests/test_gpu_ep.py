"""Expert-parallel decode on 2 GPUs (one process per GPU): each rank holds
half of every layer's experts.

* The fused one-token step (one persistent launch per rank, the down
  outputs of each rank's selections stored into the other GPU's memory,
  every row combined in selection order on every rank) gives the same bits
  as the single-GPU persistent kernel with every expert.
* The per-layer path (NCCL all-reduce of the partial combine per layer)
  equals the single-GPU full model within fp32 reassociation of the
  combine: one token against the per-token layer steps, a batch against the
  batched (tensor-core) stack, which is in turn within the chain tolerance
  of the per-token fp32 path.

Skipped with fewer than 2 GPUs."""
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


def _x0(B, h=H):
    return po.fill_f32(B * h, po.key(21, 0, 4, 0, 0), 1.0).reshape(B, h).copy()


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


def _rank(rank, world, port, fmt, B, out, fused=False, shape=(H, M, E, NL), whole=False):
    import torch
    dc, dist = _init(rank, world, port)
    ep = _ep_module()
    h, m, e, nl = shape
    shard = ep.GpuShard(dc, fmt, nl, h, m, e, K, rank, world, seed=21, whole=whole)
    shard.attach()
    shard.model.ep_set_fused(fused)
    out[f"ready{rank}"] = shard.model.ep_fused_ready()
    st = torch.from_numpy(_x0(B, h)).cuda()
    sp = torch.cuda.current_stream().cuda_stream
    shard.decode(st, 1, sp)                  # per-layer path: the eager first step
    shard.decode(st, 2, sp)                  # then the captured step, twice
    torch.cuda.synchronize()
    out[rank] = st.cpu().numpy()
    shard.close()
    dist.barrier()
    dist.destroy_process_group()


def _spawn(target, args_of):
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    procs = [ctx.Process(target=target, args=args_of(r, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    return dict(out)


@pytest.mark.skipif(_ngpu() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("whole", [False, True], ids=["shard", "whole-split-by-selection"])
@pytest.mark.parametrize("shape", [(1024, 256, 64, 3), (2048, 512, 256, 4)], ids=["small", "config2-4-layers"])
@pytest.mark.parametrize("fmt", [2, 0])            # FP8, MXFP4
def test_fused_one_token_two_gpus_bit_exact(fmt, shape, whole):
    """3 steps (two launches) of the fused step on 2 GPUs against the
    single-GPU persistent kernel holding every expert: identical bits, with
    each GPU holding half of the experts (selections split by owner) or all
    of them (selections split by index)."""
    out = _spawn(_rank, lambda r, port, out: (r, 2, port, fmt, 1, out, True, shape, whole))
    assert out["ready0"] and out["ready1"]
    assert np.array_equal(out[0], out[1])
    h, m, e, nl = shape
    dc = ds4f_cuda()
    dc.init()
    full = dc.Model(fmt, nl, h, m, e, K)
    full.synth(21)
    full.set_path(dc.PATH_PERSISTENT)
    want = full.stack(_x0(1, h)[0], 3)
    full.close()
    assert np.array_equal(out[0][0].view(np.uint32), want.view(np.uint32)), \
        float(np.abs(out[0][0] - want).max())


@pytest.mark.skipif(_ngpu() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("B", [1, 2])
@pytest.mark.parametrize("fmt", [2, 0])            # FP8, MXFP4
def test_expert_parallel_two_gpus(fmt, B):
    """The per-layer path (fused off)."""
    import torch
    out = _spawn(_rank, lambda r, port, out: (r, 2, port, fmt, B, out, False))
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


# ---- failure detection of the fused step (no GPU fault) ----------------------

def _rank_stall(rank, world, port, fmt, out):
    """Rank 1 withholds its down rows at layer-step 2 of a 2-step launch
    (6 layer-steps): rank 0's bounded wait for them runs out (code 11), then
    rank 1's wait for rank 0's rows of layer-step 3. Both calls return -1
    within the limit's time; the next launch, hook off, gives the clean bits."""
    import time
    import torch
    dc, dist = _init(rank, world, port)
    ep = _ep_module()
    shard = ep.GpuShard(dc, fmt, NL, H, M, E, K, rank, world, seed=21)
    shard.attach()
    assert shard.model.ep_fused_ready()
    sp = torch.cuda.current_stream().cuda_stream
    st = torch.from_numpy(_x0(1)).cuda()
    shard.model.set_wait_limit(1 << 14)
    if rank == 1:
        shard.model.inject_peer_stall(2)
    dist.barrier()
    t0 = time.time()
    try:
        shard.decode(st, 2, sp)              # enqueued; the kernel's error word is read next
        torch.cuda.synchronize()
        shard.model.stats()
        out[f"err{rank}"] = ""
    except dc.GpuError as e:
        out[f"err{rank}"] = str(e)
    out[f"secs{rank}"] = time.time() - t0
    shard.model.inject_peer_stall(-1)
    shard.model.set_wait_limit(0)
    dist.barrier()
    st = torch.from_numpy(_x0(1)).cuda()
    shard.decode(st, 1, sp)
    shard.decode(st, 2, sp)
    torch.cuda.synchronize()
    out[rank] = st.cpu().numpy()
    shard.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(_ngpu() < 2, reason="needs 2 GPUs")
def test_fused_peer_stall_times_out_and_recovers():
    out = _spawn(_rank_stall, lambda r, port, out: (r, 2, port, 2, out))
    for r in (0, 1):
        assert "gave up waiting (code 11" in out[f"err{r}"], out[f"err{r}"]
        assert out[f"secs{r}"] < 10.0
    assert np.array_equal(out[0], out[1])
    dc = ds4f_cuda()
    dc.init()
    full = dc.Model(2, NL, H, M, E, K)
    full.synth(21)
    full.set_path(dc.PATH_PERSISTENT)
    want = full.stack(_x0(1)[0], 3)
    full.close()
    assert np.array_equal(out[0][0].view(np.uint32), want.view(np.uint32))
