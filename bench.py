#!/usr/bin/env python
"""bench.py: 40-layer FP8 MoE-stack decode on B200.

One step = one token through all 40 MoE layers (router over 256 experts,
top-8 renormalised, 8 FP8 expert chains, bf16 shared expert, combine,
residual), the hidden state carried from step to step. Synthetic seeded
weights generated on the device (~32 GB FP8 pool), synthetic N(0, 1) input.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

value      tok/s over K device-timed steps, state resident in HBM (CUDA
           events on the launching stream), whole job over N ranks.
e2e        tok/s through the C ABI's host-buffer call ds4f_gpu_moe_stack
           (8 KB state H2D + D2H every step, host clock around the
           synchronous call).
roofline   algorithmic bytes per token / time per token vs the measured
           HBM copy bandwidth (MEASURED_PEAKS.json).
cpu_baseline  the reference's own kernels (oracle/_ref: ds4f_f8_matvec AVX2,
           ds4f_bf16_matvec, ds4f_topk; expert chains on 8 threads as
           ds4f_moe_step does) on a bounded sample of layer-tokens.
N > 1      the same 40-layer FP8 decode with the experts partitioned E / N
           per GPU (config 3's partition; ds4f_gpu_ep_stack_dev: per layer
           each GPU's partial chains and one NCCL all-reduce of acc);
           strong scaling: one token per step, the same on every rank.
"""
import argparse
import ctypes as C
import json
import os
import shutil
import signal
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "disk-qwen35ba3b_b200")
sys.path.insert(0, ROOT)


def ds4f_cuda():
    """The product's ctypes binding (the package directory name is not a
    Python identifier, so it is loaded by path)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("ds4f_cuda", os.path.join(PKG, "ds4f_cuda.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod

H, M, E, K, LAYERS = 2048, 512, 256, 8, 40
METRIC = "MoE-stack decode tok/s (40-layer FP8, 1 B200 per rank)"
METRIC_MX = "MoE-stack decode tok/s (40-layer MXFP4, 1 B200 per rank)"
METRIC_EP = "MoE-stack decode tok/s (40-layer, experts sharded over the GPUs)"


def bytes_per_token(fmt_fp8=True):
    if fmt_fp8:
        slot = 3 * (M * H + (M // 128) * (H // 128) * 4)
    else:
        slot = 3 * (M * H // 2 + M * H // 32)
    per_layer = E * H * 2 + K * slot + 3 * M * H * 2 + 2 * H * 2
    return LAYERS * per_layer


# DRAM bytes (read + write) of one 40-layer k_decode launch: an ncu capture
# (dram__bytes_read.sum + dram__bytes_write.sum) of the 4-layer case of this
# script (--layers 4, 3.2 GB pool, 130 MB of weights per launch, larger than
# L2), scaled by 10: every layer reads its own weights. Re-measured whenever
# k_decode changes; KERNEL_REV names the kernel revision it belongs to.
KERNEL_REV = "k_decode r2"
TRAFFIC_PER_LAUNCH = 10 * (130_202_368 + 5_310_976)
# kernels of one batched-prefill layer (csrc/prefill.cu): count, plan, place,
# front end, gate/up GEMM, SiLU digits, down GEMM, shared gate/up and down
# GEMMs, shared SiLU digits, combine
PREFILL_LAUNCHES_PER_LAYER = 11


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """SM clock and throttle reasons sampled during the timed region: NVML
    every 10 ms from a thread (so short regions still get samples), else
    nvidia-smi at 200 ms."""
    BITS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
            0x4: "sw_power_cap"}

    def __init__(self, dev):
        import threading
        self.sm, self.mx, self.reasons, self.p, self.t = [], 0.0, set(), None, None
        try:
            import pynvml
            pynvml.nvmlInit()
            h = None
            try:
                import torch
                uid = str(torch.cuda.get_device_properties(dev).uuid)
                h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + uid) if not uid.startswith("GPU-") else uid)
            except Exception:
                h = pynvml.nvmlDeviceGetHandleByIndex(dev)
            self.mx = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            get_r = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            self.stop_ev = threading.Event()

            def run():
                while not self.stop_ev.is_set():
                    try:
                        self.sm.append(float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)))
                        r = get_r(h)
                        for bit, name in self.BITS.items():
                            if r & bit:
                                self.reasons.add(name)
                    except Exception:
                        pass
                    self.stop_ev.wait(0.01)
            self.t = threading.Thread(target=run, daemon=True)
            self.t.start()
            self.src = "nvml"
            return
        except Exception:
            pass
        cmd = ["nvidia-smi", "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
               "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
               "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits", "-lms", "200",
               "-i", str(dev)]
        if shutil.which("stdbuf"):
            cmd = ["stdbuf", "-oL"] + cmd
        try:
            self.p = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.src = "nvidia-smi"
        except Exception:
            self.p = None

    def stop(self):
        if self.t is not None:
            self.stop_ev.set()
            self.t.join(timeout=2)
        elif self.p is not None:
            self.p.send_signal(signal.SIGINT)
            try:
                out, _ = self.p.communicate(timeout=5)
            except Exception:
                self.p.kill()
                out, _ = self.p.communicate()
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for line in out.strip().splitlines():
                f = [x.strip() for x in line.split(",")]
                if len(f) < 6:
                    continue
                try:
                    self.sm.append(float(f[0]))
                    self.mx = max(self.mx, float(f[1]))
                except ValueError:
                    continue
                for n, v in zip(names, f[2:6]):
                    if v == "Active":
                        self.reasons.add(n)
        else:
            return None
        if not self.sm:
            return None
        return {"sm_mhz": statistics.median(self.sm), "sm_max_mhz": self.mx,
                "reasons": sorted(self.reasons), "samples": len(self.sm), "source": self.src}


# ---- CPU baseline: the reference's own kernels on the host cores -------------

CPU_POOL_SLOTS = 128          # distinct FP8 expert slots of the CPU working set


def cpu_reference_sampler(threads=8):
    """Build the reference CPU path once and return (sample, close):
    sample(seconds) times layer-tokens of it (its own compiled kernels) and
    returns tok/s for the 40-layer stack plus a description; the state
    restarts from the input every 40 layers, one token.
    Per layer: RMSNorm, bf16 router matvec (ds4f_bf16_matvec), ds4f_topk,
    8 expert chains (3 x ds4f_f8_matvec each, E8M0 128x128 block scales --
    the reference's FP8 scale format, same work per element as fp32 scales)
    on one thread per expert as ds4f_moe_step does (src/moe.c:1162-1192),
    selection-order combine, bf16 shared expert with its sigmoid gate.
    Working set: 40 layers, each with its own router, shared expert and
    gate (293 MB of bf16), and 128 distinct FP8 expert slots (403 MB);
    expert e of layer L reads slot (L E + e) mod 128. That is ~700 MB, far
    beyond the host's caches, so a token streams its 1.3 GB of weights from
    DRAM as config 2's 32 GB pool would make it (the full pool is not built
    on the host)."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor
    from oracle import pyoracle as po
    R = po.ref()
    kind = "reference" if R is not None else "port"
    rng = np.random.default_rng(0)
    canon = np.array([b for b in range(256) if (b >> 3) & 15 != 15], np.uint8)
    ex = []
    for _ in range(CPU_POOL_SLOTS):
        mats = []
        for (r, c) in ((M, H), (M, H), (H, M)):
            w = canon[rng.integers(0, len(canon), r * c, dtype=np.uint8)].reshape(r, c)
            sc = rng.integers(112, 120, (r // 128) * (c // 128), dtype=np.uint8)
            mats.append((w, sc, r, c))
        ex.append(mats)

    def bf16(shape):
        f = (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)).view(np.uint32)
        return (f >> 16).astype(np.uint16)
    trunks = [(bf16((E, H)), bf16((M, H)), bf16((M, H)), bf16((H, M)), bf16((1, H))) for _ in range(LAYERS)]
    norm = np.full(H, 0x3F80, np.uint16)
    x = po.fill_f32(H, po.key(0, 0, 4, 0, 0), 1.0)
    ptr = po.ptr
    if R is not None:
        R.ds4f_kernels_set_simd(1)

    def f8mv(w, sc, r, c, xin):
        y = np.zeros(r, np.float32)
        if R is not None:
            R.ds4f_f8_matvec(ptr(w), ptr(sc), r, c, r // 128, c // 128, ptr(xin), ptr(y))
        else:
            po.lib().orc_f8_matvec(ptr(w), 0, ptr(sc), r, c, r // 128, c // 128, ptr(xin), ptr(y))
        return y

    def bfmv(w, xin):
        r, c = w.shape
        y = np.zeros(r, np.float32)
        if R is not None:
            R.ds4f_bf16_matvec(ptr(w), r, c, ptr(xin), None, ptr(y))
        else:
            po.lib().orc_bf16_matvec(ptr(w), r, c, ptr(xin), None, ptr(y))
        return y

    def chain(slot, xin):
        (wg, sg, r, c), (wu, su, _, _), (wd, sd, rd, cd) = ex[slot]
        g = f8mv(wg, sg, r, c, xin)
        u = f8mv(wu, su, r, c, xin)
        ch = (g * (1.0 / (1.0 + np.exp(-g))) * u).astype(np.float32)
        return f8mv(wd, sd, rd, cd, ch)

    pool = ThreadPoolExecutor(threads)

    def layer(L, state):
        router, shg, shu, shd, shw = trunks[L]
        xin = state.copy()
        po.lib().orc_rmsnorm(ptr(norm), H, ptr(xin))
        sc = bfmv(router, xin)
        idx = np.zeros(K, np.int32)
        w = np.zeros(K, np.float32)
        if R is not None:
            R.ds4f_topk(ptr(sc), E, K, ptr(idx), ptr(w))
        else:
            po.lib().orc_topk(ptr(sc), E, K, ptr(idx), ptr(w))
        w = w / w.sum()
        outs = list(pool.map(lambda e: chain((L * E + int(e)) % CPU_POOL_SLOTS, xin), idx))
        acc = np.zeros(H, np.float32)
        for j in range(K):
            acc += w[j] * outs[j]
        g = bfmv(shg, xin)
        u = bfmv(shu, xin)
        so = bfmv(shd, (g * (1.0 / (1.0 + np.exp(-g))) * u).astype(np.float32))
        sgt = bfmv(shw, xin)[0]
        acc += (1.0 / (1.0 + np.exp(-sgt))) * so
        return state + acc

    run = {"st": x.copy(), "done": 0}

    def sample(seconds):
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds or n < 2:
            L = run["done"] % LAYERS
            if L == 0:
                run["st"] = x.copy()
            run["st"] = layer(L, run["st"])
            run["done"] += 1
            n += 1
        dt = time.perf_counter() - t0
        return (n / LAYERS) / dt, n, dt

    desc = {"cores": threads, "kind": kind, "nproc": os.cpu_count(),
            "working_set": f"40 distinct layers of router + shared expert (293 MB bf16) and "
                           f"{CPU_POOL_SLOTS} distinct FP8 expert slots (403 MB): beyond the host caches"}
    return sample, pool.shutdown, desc


def cpu_reference_median(n_samples, seconds_each, warm_seconds, threads=8):
    """The reference CPU path timed the same way in both bench arms: one
    warm-up sample, then the median tok/s of n_samples samples."""
    sample, close, desc = cpu_reference_sampler(threads)
    try:
        sample(warm_seconds)
        runs = [sample(seconds_each) for _ in range(n_samples)]
    finally:
        close()
    vals = sorted(r[0] for r in runs)
    value = statistics.median(vals)
    layers = sum(r[1] for r in runs)
    secs = sum(r[2] for r in runs)
    return value, dict(desc, sample=f"median of {n_samples} warmed samples ({layers} layer-tokens of the "
                                    f"40-layer FP8 stack in {secs:.1f} s; reference "
                                    f"{'AVX2' if desc['kind'] == 'reference' else 'scalar port'} kernels, "
                                    f"expert chains on {threads} threads), tok/s = layer-tokens / 40 / s",
                       spread=[round(vals[0], 4), round(vals[-1], 4)])


def cpu_matvec_sample(seconds=4.0):
    """The reference's own ds4f_f8_matvec (oracle/_ref, AVX2; E8M0 block
    scales, the reference's FP8 scale format, same work per element) over the
    24 config-1 matvecs, one thread as the reference runs one matvec: GB/s."""
    import numpy as np
    from oracle import pyoracle as po
    R_ = po.ref()
    rng = np.random.default_rng(0)
    canon = np.array([b for b in range(256) if (b >> 3) & 15 != 15], np.uint8)
    mats = []
    for e in range(8):
        for (r, c) in ((M, H), (M, H), (H, M)):
            w = canon[rng.integers(0, len(canon), r * c)].reshape(r, c)
            sc = rng.integers(112, 120, (r // 128) * (c // 128), dtype=np.uint16).astype(np.uint8)
            mats.append((w, sc, r, c, po.fill_f32(c, po.key(1, 0, 4, e, 0), 1.0), np.zeros(r, np.float32)))
    if R_ is not None:
        R_.ds4f_kernels_set_simd(1)
    nbytes = sum(w.nbytes + sc.nbytes for w, sc, _, _, _, _ in mats)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds or n < 1:
        for w, sc, r, c, x, y in mats:
            if R_ is not None:
                R_.ds4f_f8_matvec(po.ptr(w), po.ptr(sc), r, c, r // 128, c // 128, po.ptr(x), po.ptr(y))
            else:
                po.lib().orc_f8_matvec(po.ptr(w), 0, po.ptr(sc), r, c, r // 128, c // 128, po.ptr(x), po.ptr(y))
        n += 1
    dt = time.perf_counter() - t0
    return n * nbytes / dt / 1e9, {"cores": 1, "kind": "reference" if R_ is not None else "port",
                                   "sample": f"{n} passes over the 24 config-1 FP8 matvecs in {dt:.1f} s "
                                             f"({'reference AVX2' if R_ is not None else 'scalar port'}, one thread)",
                                   "nproc": os.cpu_count()}


# ---- GPU arm ------------------------------------------------------------------

def decode_config(fp8, world, layers=LAYERS, parallelism=None):
    """The `config` of a decode line: the same dict in both bench arms."""
    bpt = bytes_per_token(fp8) * layers // LAYERS
    return {"workload": ("config 2: 40-layer FP8 MoE decode, 1 token/step" if fp8 else
                         "config 3 (1 GPU, batch 1): 40-layer MXFP4 MoE decode, 1 token/step")
            if layers == LAYERS else f"profiling case: {layers}-layer {'FP8' if fp8 else 'MXFP4'} decode",
            "hidden": H, "moe_inter": M, "experts": E, "topk": K, "layers": layers,
            "pool_gb": round(layers * E * (3146496 if fp8 else 1671168) / 1e9, 2),
            "l2": f"inputs larger than L2 ({bpt / 1e9:.2f} GB of weights per step)",
            "parallelism": parallelism or ("single GPU" if world == 1 else f"replicas x{world}")}


N_STAMPS = 32          # phase-trace stamp slots per (layer-step, CTA) in k_decode
PHASES = ["start", "state", "norm", "rows_done", "routes_vis", "topk", "issued",
          "softmax", "grp0", "chains", "down_in", "written"]


def phase_table(tr, ep=False):
    """k_decode's %globaltimer phase trace of one step (the counterpart of
    the reference's per-phase timers, src/main.c:253-258, 1522-1546):
    tr int64 [L, G, N_STAMPS] -> per phase the median over layers of the
    median and of the max over CTAs (us), gather rounds, layer period."""
    import numpy as np
    L = tr.shape[0]
    out = {}
    d = np.diff(tr[:, :, :12], axis=2)
    rows = []
    for k in range(11):
        rows.append((f"{PHASES[k]} -> {PHASES[k + 1]}",
                     float(np.median(np.median(d[:, :, k], axis=1)) / 1e3),
                     float(np.median(np.max(d[:, :, k], axis=1)) / 1e3)))
    inner = np.diff(tr[:, :, [10, 12, 13, 11]], axis=2)
    for k, name in enumerate(["down: chain gather", "down: row-dots", "down: combine"]):
        rows.append((name, float(np.median(inner[:, :, k]) / 1e3),
                     float(np.median(np.max(inner[:, :, k], axis=1)) / 1e3)))
    inner = np.diff(tr[:, :, [3, 18, 27, 28, 29, 30, 31, 4]], axis=2)
    for k, name in enumerate(["routes: gather", "routes: keys", "routes: top-8 network", "routes: certificate",
                              "routes: byte counts", "routes: group 0 issue", "routes: to barrier"]):
        rows.append((name, float(np.median(inner[:, :, k]) / 1e3),
                     float(np.median(np.max(inner[:, :, k], axis=1)) / 1e3)))
    # gate/up: groups landing and dots finishing, as offsets from the softmax
    # (stamp 7); down: warp 0's first row-dot pair and the rest
    for k, name in [(8, "gate/up: group 0 landed"), (21, "gate/up: group 1 landed"),
                    (22, "gate/up: group 2 landed"), (23, "gate/up: group 3 landed"),
                    (24, "gate/up: warp 0 dots done"), (25, "gate/up: all warps done"),
                    (9, "gate/up: chains published")]:
        off = (tr[:, :, k] - tr[:, :, 7]).astype(np.float64)
        ok = tr[:, :, k] > 0
        if ok.any():
            rows.append(("  +" + name, float(np.median(off[ok]) / 1e3), float(np.median(np.max(np.where(ok, off, 0), axis=1)) / 1e3)))
    inner = np.diff(tr[:, :, [12, 26, 13]], axis=2)
    for k, name in enumerate(["down: first row-dot pair", "down: other row-dots"]):
        rows.append((name, float(np.median(inner[:, :, k]) / 1e3),
                     float(np.median(np.max(inner[:, :, k], axis=1)) / 1e3)))
    if ep:
        # the other GPUs' rows: stored to them (after the row-dots), theirs arrived
        inner = np.diff(tr[:, :, [13, 19, 20, 11]], axis=2)
        for k, name in enumerate(["ep: rows stored to peers", "ep: peers' rows arrived", "ep: combine + state"]):
            rows.append((name, float(np.median(inner[:, :, k]) / 1e3),
                         float(np.median(np.max(inner[:, :, k], axis=1)) / 1e3)))
    out["phases_us"] = rows
    rounds = tr[:, :, 14:17].astype(np.float64)
    if L > 1:
        rounds = rounds[1:]          # layer 0 reads the state directly
    out["gather_rounds_mean"] = {n: round(float(rounds[:, :, k].mean()), 2)
                                 for k, n in enumerate(["state", "router", "chains"])}
    landed = tr[:, :, 17]
    out["group_landed_early"] = [round(float(((landed >> g) & 1).mean()), 3) for g in range(4)]
    if L > 1:
        lay = (tr[1:, :, 0].min(axis=1) - tr[:-1, :, 0].min(axis=1)) / 1e3
        out["layer_period_us"] = {"median": float(np.median(lay)), "min": float(lay.min()),
                                  "max": float(lay.max())}
    out["step_us"] = float((tr[-1, :, 11].max() - tr[0, :, 0].min()) / 1e3)
    return out


def run_gpu(args, rank, world, local_rank):
    import torch
    dc = ds4f_cuda()
    torch.cuda.set_device(local_rank)
    dc.init()
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    fp8 = args.fmt == "fp8"
    layers = args.layers
    model = dc.Model(dc.FMT_FP8 if fp8 else dc.FMT_MXFP4, layers, H, M, E, K)
    model.synth(0)
    model.set_path(dc.PATH_LAYERED if args.layered else dc.PATH_PERSISTENT)
    state = torch.empty(H, dtype=torch.float32, device="cuda")
    dc.synth_f32_dev(state, H, 0, 0, 4, rank, 0, 1.0)
    torch.cuda.synchronize()
    sp = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(args.warmup):
        model.stack_dev(state, 1, sp)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clk = Clocks(local_rank)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        model.stack_dev(state, 1, sp)
    e1.record()
    torch.cuda.synchronize()
    t_ms = e0.elapsed_time(e1)
    clocks = clk.stop()
    if dist:
        dist.barrier()
    # e2e: the reference-facing host-buffer call, pinned host state
    hst = torch.empty(H, dtype=torch.float32).pin_memory()
    hst.copy_(state.cpu())
    hnp = hst.numpy()
    for _ in range(max(1, args.warmup)):
        model.stack_host_inplace(hnp, 1)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        model.stack_host_inplace(hnp, 1)
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    trace = None
    if args.trace and not args.layered:
        import numpy as np
        G = torch.cuda.get_device_properties(local_rank).multi_processor_count
        n = layers * G * N_STAMPS
        model.trace(n)
        model.stack_dev(state, 1, sp)
        torch.cuda.synchronize()
        trace = phase_table(model.trace_read(n).astype(np.int64).reshape(layers, G, N_STAMPS))
        model.trace(0)
    fallbacks = model.stats()[1]
    if dist:
        t = torch.tensor([t_ms, e2e_s], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_ms, e2e_s = float(t[0]), float(t[1])
    model.close()
    res = None
    if rank == 0:
        ms = t_ms / args.steps
        value = world * args.steps / (t_ms / 1e3)
        bpt = bytes_per_token(fp8) * layers // LAYERS
        peak, src = peaks()
        achieved = bpt / (ms / 1e3) / 1e9
        res = {
            "metric": METRIC if fp8 else METRIC_MX, "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": ("fp8-e4m3" if fp8 else "mxfp4 (e2m1 + e8m0/32)") + " weights, fp32 accumulate",
            "data": "synthetic (seeded, device-generated)",
            "config": decode_config(fp8, world, layers),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": (TRAFFIC_PER_LAUNCH * layers // LAYERS
                                     if fp8 and not args.layered else None),
                         "traffic_unit": f"bytes per launch (ncu of the 4-layer case x 10; {KERNEL_REV})",
                         "peak_source": src,
                         "kernel": ("whole decode step: 4 kernels per layer in a CUDA graph" if args.layered
                                    else "k_decode: the whole 40-layer step in one persistent launch"),
                         "algorithmic_bytes_per_token": bpt},
            "e2e": {"value": round(world * args.steps / e2e_s, 2), "unit": "tok/s",
                    "h2d_bytes_per_step": H * 4, "d2h_bytes_per_step": H * 4,
                    "timer": "host clock around the synchronous C-ABI call"},
            "gpu_launches": (4 * layers if args.layered else 1) * args.steps,
            "router_exact_fallbacks": int(fallbacks),
            "clocks": clocks,
        }
        if trace is not None:
            for name, med, mx in trace.pop("phases_us"):
                print(f"  {name:<24s} {med:8.2f} {mx:8.2f}   (us: median, max over CTAs)", file=sys.stderr)
            res["trace"] = trace
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return res


# ---- config 4: batched prefill --------------------------------------------------

T_PREFILL = 2048
METRIC_PREFILL = "MoE-stack prefill tok/s (2048-token chunk, 40-layer FP8, 1 B200 per rank)"


def zipf_routing(n_layers, T, E, K, seed):
    """Seeded synthetic routing with expert load ~ Zipf(1.1): K distinct
    experts per token sampled without replacement with p(e) ~ (e+1)^-1.1
    (Gumbel top-k), softmax weights of seeded logits renormalised over K."""
    import numpy as np
    rng = np.random.default_rng(seed)
    logp = -1.1 * np.log(np.arange(1, E + 1, dtype=np.float64))
    perm = np.stack([rng.permutation(E) for _ in range(n_layers)])        # which expert is hot, per layer
    sel = np.zeros((n_layers, T, K), np.int32)
    for L in range(n_layers):
        keys = logp[None, :] + rng.gumbel(size=(T, E))
        top = np.argpartition(-keys, K, axis=1)[:, :K]
        sel[L] = perm[L][top]
    logits = rng.normal(size=(n_layers, T, K)).astype(np.float32)
    w = np.exp(logits - logits.max(-1, keepdims=True)).astype(np.float32)
    w /= w.sum(-1, keepdims=True)
    return sel, w.astype(np.float32)


def run_gpu_prefill(args, rank, world, local_rank):
    import numpy as np
    import torch
    dc = ds4f_cuda()
    torch.cuda.set_device(local_rank)
    dc.init()
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    T = args.tokens
    NL = args.layers
    fp8 = args.fmt != "mxfp4"
    model = dc.Model(dc.FMT_FP8 if fp8 else dc.FMT_MXFP4, NL, H, M, E, K)
    model.synth(0)
    sel, w = zipf_routing(NL, T, E, K, seed=100 + rank)
    selg = torch.from_numpy(sel).cuda()
    wg = torch.from_numpy(w).cuda()
    x0 = torch.empty((T, H), dtype=torch.float32, device="cuda")
    dc.synth_f32_dev(x0, T * H, 0, 0, 4, rank, 1, 1.0)
    x0 = x0.bfloat16().float()                                   # bf16 activations ~ N(0, 1)
    states = torch.empty_like(x0)
    sp = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(args.warmup):
        states.copy_(x0)
        model.prefill_dev(states, selg, wg, sp)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clk = Clocks(local_rank)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        states.copy_(x0)
        model.prefill_dev(states, selg, wg, sp)
    e1.record()
    torch.cuda.synchronize()
    t_ms = e0.elapsed_time(e1)
    clocks = clk.stop()
    # e2e: host states and routing in, states out, every step
    hx = x0.cpu().pin_memory()
    hsel = torch.from_numpy(sel).pin_memory()
    hw = torch.from_numpy(w).pin_memory()
    hout = torch.empty_like(hx).pin_memory()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        states.copy_(hx, non_blocking=True)
        selg.copy_(hsel, non_blocking=True)
        wg.copy_(hw, non_blocking=True)
        model.prefill_dev(states, selg, wg, sp)
        hout.copy_(states, non_blocking=True)
        torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    if dist:
        tt = torch.tensor([t_ms, e2e_s], device="cuda", dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_ms, e2e_s = float(tt[0]), float(tt[1])
    model.close()
    res = None
    if rank == 0:
        ms = t_ms / args.steps
        # algorithmic work: the weights of every expert a layer's tokens touch
        # (read once), the shared expert and norm, plus FLOPs 2 * rows * K * R
        uniq = [len(np.unique(sel[L])) for L in range(NL)]
        # algorithmic bytes: every touched expert once in the pool's own format
        # (the MXFP4 path streams its exact FP8 copy: 2x these bytes)
        slot = 3 * (M * H + (M // 128) * (H // 128) * 4) if fp8 else 3 * (M * H // 2 + M * H // 32)
        bytes_step = sum(u * slot + 3 * M * H * 2 + 2 * H * 2 for u in uniq)
        flops_step = NL * (2 * T * K * 3 * M * H + 2 * T * 3 * M * H)
        peak, src = peaks()
        bw = bytes_step / (ms / 1e3) / 1e9
        tf = flops_step / (ms / 1e3) / 1e12
        loads = np.bincount(sel[0].ravel(), minlength=E)
        res = {
            "metric": METRIC_PREFILL if fp8 else METRIC_PREFILL.replace("FP8", "MXFP4"),
            "value": round(world * T * args.steps / (t_ms / 1e3), 1),
            "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": ("fp8-e4m3" if fp8 else "mxfp4 (as its exact fp8 copy)") +
                     " weights x 3-digit e4m3 activations, fp32 accumulate (tcgen05)",
            "data": "synthetic (seeded weights, bf16 N(0,1) activations, Zipf(1.1) routing)",
            "config": {"workload": (f"config 4: prefill of a 2048-token chunk, 40-layer {'FP8' if fp8 else 'MXFP4'}"
                                    if (NL, T) == (LAYERS, T_PREFILL) else
                                    f"profiling case: {T}-token chunk, {NL}-layer {'FP8' if fp8 else 'MXFP4'}"),
                       "tokens": T, "hidden": H, "moe_inter": M, "experts": E, "topk": K, "layers": NL,
                       "max_tokens_per_expert_L0": int(loads.max()),
                       "median_tokens_per_expert_L0": float(np.median(loads)),
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2 (32 GB of expert weights per step)"},
            "roofline": {"bound": "hbm", "achieved": round(bw, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(bw / peak, 4), "traffic": None, "peak_source": src,
                         "algorithmic_bytes_per_step": bytes_step,
                         "tensor": {"achieved_tflops": round(tf, 1), "peak_tflops": 4500.0,
                                    "peak_source": "nominal dense FP8", "frac": round(tf / 4500.0, 4),
                                    "flops_per_step": flops_step}},
            "e2e": {"value": round(world * T * args.steps / e2e_s, 1), "unit": "tok/s",
                    "h2d_bytes_per_step": T * H * 4 + sel.nbytes + w.nbytes,
                    "d2h_bytes_per_step": T * H * 4, "timer": "host clock, synchronous steps"},
            "gpu_launches": args.steps * NL * PREFILL_LAUNCHES_PER_LAYER,
            "clocks": clocks,
        }
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return res


# ---- config 3: expert-parallel decode ------------------------------------------

def _ep_module():
    import importlib.util
    spec = importlib.util.spec_from_file_location("ep", os.path.join(PKG, "ep.py"))
    ep = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ep)
    return ep


def _init_group(world, local_rank):
    """torch.distributed for the barriers, the timing max over ranks and the
    communicator id; the data plane is the library's own NCCL."""
    import datetime
    import torch
    import torch.distributed as dist
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    else:
        import tempfile
        dist.init_process_group("gloo", init_method="file://" + tempfile.mktemp(), rank=0, world_size=1)
    return dist


def run_gpu_ep(args, rank, world, local_rank):
    """Config 3 (and the N > 1 default): decode with E / N experts per GPU
    through ds4f_gpu_ep_stack_dev. Strong scaling: every rank works on the
    same B tokens, the experts (and their bytes) are partitioned."""
    import torch
    dc = ds4f_cuda()
    torch.cuda.set_device(local_rank)
    dc.init()
    dist = _init_group(world, local_rank)
    ep = _ep_module()
    fp8 = args.fmt == "fp8"
    layers = args.layers
    shard = ep.GpuShard(dc, dc.FMT_FP8 if fp8 else dc.FMT_MXFP4, layers, H, M, E, K, rank, world, seed=0,
                        whole=args.ep_whole and world > 1)
    shard.attach()
    Bt = args.batch
    shard.model.ep_set_fused(not args.ep_layered)
    fused = Bt == 1 and shard.model.ep_fused_ready()
    st = torch.empty((Bt, H), dtype=torch.float32, device="cuda")
    dc.synth_f32_dev(st, Bt * H, 0, 0, 4, 0, 2, 1.0)            # the same tokens on every rank
    sp = torch.cuda.current_stream().cuda_stream
    for _ in range(max(1, args.warmup)):
        shard.decode(st, 1, sp)
    torch.cuda.synchronize()
    dist.barrier()
    clk = Clocks(local_rank)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):                 # one call (fused: one launch per rank) per token
        shard.decode(st, 1, sp)
    e1.record()
    torch.cuda.synchronize()
    t_ms = e0.elapsed_time(e1)
    clocks = clk.stop()
    # e2e: host state in, host state out each step
    hst = st.cpu().pin_memory()
    dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        st.copy_(hst, non_blocking=True)
        shard.decode(st, 1, sp)
        hst.copy_(st, non_blocking=True)
        torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    trace = None
    if args.trace and fused:
        # every rank records (they run in step); rank 0's stamps are printed
        import numpy as np
        G = torch.cuda.get_device_properties(local_rank).multi_processor_count
        n = layers * G * N_STAMPS
        shard.model.trace(n)
        dist.barrier()
        shard.decode(st, 1, sp)
        torch.cuda.synchronize()
        raw = shard.model.trace_read(n).astype(np.int64).reshape(layers, G, N_STAMPS)
        trace = phase_table(raw, ep=True)
        shard.model.trace(0)
        if args.trace_dump:
            np.save(f"{args.trace_dump}.r{rank}.npy", raw)
    tt = torch.tensor([t_ms, e2e_s], dtype=torch.float64, device="cuda" if world > 1 else "cpu")
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    t_ms, e2e_s = float(tt[0]), float(tt[1])
    shard.close()
    res = None
    if rank == 0:
        ms = t_ms / args.steps
        slot = 3 * (M * H + (M // 128) * (H // 128) * 4) if fp8 else 3 * (M * H // 2 + M * H // 32)
        # experts a layer touches for B distinct tokens (expected value; K at
        # B = 1), each read once by the job, plus router and shared expert
        uniq = K if Bt == 1 else E * (1 - (1 - K / E) ** Bt)
        bytes_step = int(layers * (uniq * slot + E * H * 2 + 3 * M * H * 2 + 2 * H * 2))
        peak, src = peaks()
        bw = bytes_step / (ms / 1e3) / 1e9
        headline = world > 1 and args.workload == "decode"
        res = {
            "metric": METRIC_EP, "value": round(Bt * args.steps / (t_ms / 1e3), 2), "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": ("fp8-e4m3" if fp8 else "mxfp4 (e2m1 + e8m0/32)") + " weights, " +
                     ("fp32 accumulate" if Bt == 1 else
                      "3-digit e4m3 activations, fp32 accumulate (tcgen05 grouped chain)"),
            "data": "synthetic (seeded, device-generated)",
            "config": {"workload": (f"config {'2' if fp8 else '3'} sharded: {layers}-layer {'FP8' if fp8 else 'MXFP4'} "
                                    f"decode, batch {Bt}, {E // world} experts per GPU"),
                       "batch": Bt, "hidden": H, "moe_inter": M, "experts": E, "topk": K, "layers": layers,
                       "parallelism": (f"expert-parallel x{world}, fused: one persistent launch per GPU per token; "
                                       + ("every expert on every GPU, the K selections split by index"
                                          if args.ep_whole else f"{E // world} experts per GPU") +
                                       f"; each GPU's selections' down rows stored into the others' memory over "
                                       f"NVLink, every row combined in selection order on every GPU (no "
                                       f"collective call)" if fused else
                                       f"expert-parallel x{world}: per layer the partial chains of each GPU's "
                                       f"experts, one NCCL all-reduce of acc [{Bt}][{H}] fp32, residual; "
                                       f"one CUDA graph per step"),
                       "l2": "inputs larger than L2"},
            "roofline": {"bound": "hbm", "achieved": round(bw, 1), "peak": peak * world, "unit": "GB/s",
                         "frac": round(bw / (peak * world), 4), "traffic": None, "peak_source": src,
                         "algorithmic_bytes_per_step": bytes_step,
                         "note": "expected unique experts per layer for the batch; peak = N x per-GPU"},
            "e2e": {"value": round(Bt * args.steps / e2e_s, 2), "unit": "tok/s",
                    "h2d_bytes_per_step": Bt * H * 4, "d2h_bytes_per_step": Bt * H * 4,
                    "timer": "host clock, synchronous steps"},
            # per layer: route, top-K, gate/up, down (B = 1; a batch: route,
            # top-K and the grouped tensor-core layer), the all-reduce, the add
            "gpu_launches": (args.steps if fused else
                             args.steps * layers * ((4 if Bt == 1 else 2 + PREFILL_LAUNCHES_PER_LAYER) + 2)),
            "clocks": clocks,
            # what bounds this N (measured on 2 x B200, NVLink 5; see the design notes)
            "limiter": ("one token is latency-bound: per layer the serial chain of one GPU (norm, router, "
                        "top-8, three on-GPU exchanges) plus one cross-GPU exchange of the down rows "
                        "(~1 us NVLink store latency + the slower GPU's skew); sharding divides only the "
                        "gate/up and down work" if fused else
                        "per layer: 4 kernel launches and one NCCL all-reduce of acc (launch and "
                        "collective latency, not bytes)"),
        }
        if trace is not None:
            for name, med, mx in trace.pop("phases_us"):
                print(f"  {name:<24s} {med:8.2f} {mx:8.2f}   (us: median, max over CTAs)", file=sys.stderr)
            res["trace"] = trace
        if headline:
            res["metric"] = METRIC
            res["note"] = ("N > 1: the 40-layer FP8 decode of config 2 with its experts sharded over the GPUs "
                           "(config 3's partition); 1 token per step, the same token on every rank")
    dist.barrier()
    dist.destroy_process_group()
    return res


# ---- config 4 at N GPUs: token-parallel prefill with all-to-all dispatch ----------

def run_gpu_ep_prefill(args, rank, world, local_rank):
    """Config 4 at N GPUs: the 2048-token chunk partitioned T / N per rank,
    E / N experts per rank, rows dispatched to the experts' ranks and
    combined back (ds4f_gpu_ep_prefill). value = the chunk's tokens / time."""
    import numpy as np
    import torch
    dc = ds4f_cuda()
    torch.cuda.set_device(local_rank)
    dc.init()
    dist = _init_group(world, local_rank)
    ep = _ep_module()
    T, NL = args.tokens, args.layers
    fp8 = args.fmt != "mxfp4"
    shard = ep.GpuShard(dc, dc.FMT_FP8 if fp8 else dc.FMT_MXFP4, NL, H, M, E, K, rank, world, seed=0)
    shard.attach()
    sel, w = zipf_routing(NL, T, E, K, seed=100)            # the whole chunk's routing, sliced per rank
    t0, t1 = rank * T // world, (rank + 1) * T // world
    selg = torch.from_numpy(np.ascontiguousarray(sel[:, t0:t1])).cuda()
    wg = torch.from_numpy(np.ascontiguousarray(w[:, t0:t1])).cuda()
    x0 = torch.empty((T, H), dtype=torch.float32, device="cuda")
    dc.synth_f32_dev(x0, T * H, 0, 0, 4, 0, 1, 1.0)
    x0 = x0.bfloat16().float()[t0:t1].contiguous()
    st = torch.empty_like(x0)
    sp = torch.cuda.current_stream().cuda_stream
    for _ in range(args.warmup):
        st.copy_(x0)
        shard.prefill(st, selg, wg, sp)
    torch.cuda.synchronize()
    dist.barrier()
    clk = Clocks(local_rank)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        st.copy_(x0)
        shard.prefill(st, selg, wg, sp)
    e1.record()
    torch.cuda.synchronize()
    t_ms = e0.elapsed_time(e1)
    clocks = clk.stop()
    hx = x0.cpu().pin_memory()
    hout = torch.empty_like(hx).pin_memory()
    dist.barrier()
    torch.cuda.synchronize()
    ts = time.perf_counter()
    for _ in range(args.steps):
        st.copy_(hx, non_blocking=True)
        shard.prefill(st, selg, wg, sp)
        hout.copy_(st, non_blocking=True)
        torch.cuda.synchronize()
    e2e_s = time.perf_counter() - ts
    tt = torch.tensor([t_ms, e2e_s], dtype=torch.float64, device="cuda" if world > 1 else "cpu")
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    t_ms, e2e_s = float(tt[0]), float(tt[1])
    shard.close()
    res = None
    if rank == 0:
        ms = t_ms / args.steps
        uniq = [len(np.unique(sel[L])) for L in range(NL)]
        slot = 3 * (M * H + (M // 128) * (H // 128) * 4) if fp8 else 3 * (M * H // 2 + M * H // 32)
        bytes_step = sum(u * slot + 3 * M * H * 2 + 2 * H * 2 for u in uniq)
        flops_step = NL * (2 * T * K * 3 * M * H + 2 * T * 3 * M * H)
        peak, src = peaks()
        bw = bytes_step / (ms / 1e3) / 1e9
        tf = flops_step / (ms / 1e3) / 1e12
        res = {
            "metric": METRIC_PREFILL.replace("1 B200 per rank", "tokens and experts partitioned over the GPUs"),
            "value": round(T * args.steps / (t_ms / 1e3), 1), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": ("fp8-e4m3" if fp8 else "mxfp4 (as its exact fp8 copy)") +
                     " weights x 3-digit e4m3 activations, fp32 accumulate (tcgen05)",
            "data": "synthetic (seeded weights, bf16 N(0,1) activations, Zipf(1.1) routing)",
            "config": {"workload": f"config 4: prefill of a {T}-token chunk, {NL}-layer {'FP8' if fp8 else 'MXFP4'}, "
                                   f"{T // world} tokens and {E // world} experts per GPU",
                       "tokens": T, "hidden": H, "moe_inter": M, "experts": E, "topk": K, "layers": NL,
                       "parallelism": f"expert-parallel x{world}: per layer an all-to-all dispatch of each token's "
                                      f"row to its experts' GPUs and an all-to-all combine back (NCCL send/recv)",
                       "l2": "inputs larger than L2"},
            "roofline": {"bound": "hbm", "achieved": round(bw, 1), "peak": peak * world, "unit": "GB/s",
                         "frac": round(bw / (peak * world), 4), "traffic": None, "peak_source": src,
                         "algorithmic_bytes_per_step": bytes_step,
                         "tensor": {"achieved_tflops": round(tf, 1), "peak_tflops": 4500.0 * world,
                                    "peak_source": "nominal dense FP8 x N", "frac": round(tf / 4500.0 / world, 4),
                                    "flops_per_step": flops_step}},
            "e2e": {"value": round(T * args.steps / e2e_s, 1), "unit": "tok/s",
                    "h2d_bytes_per_step": (t1 - t0) * H * 4, "d2h_bytes_per_step": (t1 - t0) * H * 4,
                    "timer": "host clock, synchronous steps (rank 0's share of the copies)"},
            "gpu_launches": args.steps * NL * (2 * PREFILL_LAUNCHES_PER_LAYER + 3),
            "clocks": clocks,
        }
    dist.barrier()
    dist.destroy_process_group()
    return res


# ---- config 1: dequant-matvec microbench ------------------------------------------

def run_gpu_matvec(args, rank, world, local_rank):
    """8 experts x (gate 512x2048, up 512x2048, down 2048x512) as one job list
    per format (FP8 with fp32 128x128 scales; MXFP4), x ~ N(0, 1), batch 1.
    Sixteen copies of the 24 matrices are rotated (a 16 x 38 MB working set,
    larger than L2; a plain flush by copying 256 MB did not evict them here),
    and each launch is timed alone with CUDA events."""
    import numpy as np
    import torch
    from oracle import pyoracle as po
    dc = ds4f_cuda()
    torch.cuda.set_device(local_rank)
    dc.init()
    NSET = 16                     # distinct copies, rotated: 16 x 38 MB, every launch misses L2
    keep, jobs = [], {"fp8": [[] for _ in range(NSET)], "mxfp4": [[] for _ in range(NSET)]}
    host = []
    bytes_fmt = {"fp8": 0, "mxfp4": 0}
    for e in range(8):
        for t, (R, Cc) in enumerate(((M, H), (M, H), (H, M))):
            k = po.key(1, 0, 3, e, t)
            x = po.fill_f32(Cc, po.key(1, 0, 4, e, t), 1.0)
            W, s = po.quant_fp8(R, Cc, k, 0.02)
            v, sm = po.quant_mxfp4(R, Cc, k, 0.02)
            tx = torch.from_numpy(x).cuda()
            y8 = torch.zeros(R, device="cuda")
            ym = torch.zeros(R, device="cuda")
            keep += [tx, y8, ym]
            for c in range(NSET):
                tW, ts, tv, tsm = (torch.from_numpy(a).cuda() for a in (W, s, v, sm))
                keep += [tW, ts, tv, tsm]
                jobs["fp8"][c].append(dc.Ds4fMvJob(tW.data_ptr(), ts.data_ptr(), tx.data_ptr(), y8.data_ptr(),
                                                   R, Cc, R // 128, Cc // 128, dc.FMT_FP8, dc.SCALE_F32, 32, 1))
                jobs["mxfp4"][c].append(dc.Ds4fMvJob(tv.data_ptr(), tsm.data_ptr(), tx.data_ptr(), ym.data_ptr(),
                                                     R, Cc, 1, 1, dc.FMT_MXFP4, 0, 32, 0))
            bytes_fmt["fp8"] += W.nbytes + s.nbytes
            bytes_fmt["mxfp4"] += v.nbytes + sm.nbytes
            host.append((W, s, R, Cc, x))
    sp = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    out = {}
    for fmt in ("fp8", "mxfp4"):
        plans = [dc.MvPlan(j) for j in jobs[fmt]]
        for i in range(max(args.warmup, NSET)):
            plans[i % NSET].run(sp)
        torch.cuda.synchronize()
        clk = Clocks(local_rank) if fmt == "fp8" else None
        ts = []
        for i in range(args.steps):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            plans[i % NSET].run(sp)
            e1.record()
            ts.append((e0, e1))
        torch.cuda.synchronize()
        clocks = clk.stop() if clk else None
        ms = sum(a.elapsed_time(b) for a, b in ts) / args.steps
        out[fmt] = (ms, bytes_fmt[fmt] / (ms / 1e3) / 1e9, clocks)
        del plans
    # e2e: the 24 matvecs through the reference-facing host-buffer call
    # ds4f_gpu_f8_matvec (ds4f_f8_matvec's arguments: weights, scales and x
    # in host memory, y back), one call per matrix as the reference calls it
    for W, s_, R, Cc, x in host[:3]:
        dc.f8_matvec(W, dc.SCALE_F32, s_, R // 128, Cc // 128, x)
    n_e2e = max(1, min(args.steps, 20))
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        for W, s_, R, Cc, x in host:
            dc.f8_matvec(W, dc.SCALE_F32, s_, R // 128, Cc // 128, x)
    e2e_s = (time.perf_counter() - t0) / n_e2e
    peak, src = peaks()
    ms8, gbs8, clocks = out["fp8"]
    msm, gbsm, _ = out["mxfp4"]
    return {
        "metric": "expert dequant-matvec HBM GB/s (8 experts x gate/up/down, FP8 128x128 fp32 scales)",
        "value": round(gbs8, 1), "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms8, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp8-e4m3 weights, fp32 x and accumulate", "data": "synthetic (seeded, N(0,0.02) weights)",
        "config": {"workload": "config 1: 24 matvecs (8 x 512x2048, 8 x 512x2048, 8 x 2048x512), batch 1",
                   "l2": "16 copies of the weights rotated (608 MB working set > 126 MB L2)",
                   "mxfp4": {"gb_s": round(gbsm, 1), "ms_per_step": round(msm, 4),
                             "frac": round(gbsm / peak, 4), "bytes": bytes_fmt["mxfp4"]}},
        "roofline": {"bound": "hbm", "achieved": round(gbs8, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(gbs8 / peak, 4), "traffic": None, "peak_source": src,
                     "algorithmic_bytes_per_step": bytes_fmt["fp8"]},
        "e2e": {"value": round(bytes_fmt["fp8"] / e2e_s / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": bytes_fmt["fp8"] + sum(x.nbytes for _, _, _, _, x in host),
                "d2h_bytes_per_step": sum(R * 4 for _, _, R, _, _ in host),
                "timer": "host clock around 24 synchronous ds4f_gpu_f8_matvec calls on host buffers "
                         "(weights copied in every call)"},
        "gpu_launches": args.steps * 1,
        "clocks": clocks,
    }


def mem_available_bytes():
    try:
        for line in open("/proc/meminfo"):
            if line.startswith("MemAvailable:"):
                return int(line.split()[1]) * 1024
    except OSError:
        pass
    return 0


def run_gpu_stream(args, rank, world, local_rank):
    """Pools larger than HBM (the reference's disk-streaming configuration,
    src/cache.c:140-214 over pool-mxfp4.bin): the 40-layer pool stays in
    pinned host memory, the HBM holds the trunk and an arena of --slots
    expert slots run by the reference's cache policy; every layer reads its
    routing back and copies its misses in before the chain runs. One step =
    one token through all layers. The host link is the bound: achieved =
    bytes copied in per second against a pinned host-to-device copy measured
    in the same run."""
    import numpy as np
    import torch
    dc = ds4f_cuda()
    torch.cuda.set_device(local_rank)
    dc.init()
    fp8 = args.fmt == "fp8"
    fmt = dc.FMT_FP8 if fp8 else dc.FMT_MXFP4
    slot_b = 3146496 if fp8 else 1671168
    pool_b = LAYERS * E * slot_b
    if mem_available_bytes() < pool_b * 1.5:
        return {"workload": "stream-decode", "unavailable":
                f"needs {pool_b * 1.5 / 1e9:.1f} GB of host memory for the pinned pool, "
                f"{mem_available_bytes() / 1e9:.1f} GB available"}
    # the pool: the device generator's bytes, read back once into host memory
    r = dc.Model(fmt, LAYERS, H, M, E, K)
    r.synth(0)
    host = np.empty(pool_b, np.uint8)
    L_ = dc.lib()
    for l in range(LAYERS):
        for x in range(E):
            o = (l * E + x) * slot_b
            dc.check(L_.ds4f_gpu_model_get_expert(r.h, l, x, dc.ptr(host[o:o + slot_b])))
    trunks = [r.get_trunk(l) for l in range(LAYERS)]
    r.close()
    torch.cuda.empty_cache()
    n_slots = args.slots or LAYERS * E // 4
    try:
        s = dc.Model(fmt, LAYERS, H, M, E, K, host_pool=host, stream_slots=n_slots)
    except dc.GpuError as ex:
        return {"workload": "stream-decode", "unavailable": str(ex)}
    for l in range(LAYERS):
        s.set_trunk(l, *trunks[l])
    state = torch.empty(H, dtype=torch.float32, device="cuda")
    dc.synth_f32_dev(state, H, 0, 0, 4, rank, 0, 1.0)
    sp = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(args.warmup):
        s.stack_dev(state, 1, sp)
    torch.cuda.synchronize()
    req0, hit0, fet0 = s.stream_stats()
    clk = Clocks(local_rank)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        s.stack_dev(state, 1, sp)
    e1.record()
    torch.cuda.synchronize()
    t_ms = e0.elapsed_time(e1)
    clocks = clk.stop()
    req, hit, fet = (a - b for a, b in zip(s.stream_stats(), (req0, hit0, fet0)))
    # e2e through the host-buffer call
    hst = torch.empty(H, dtype=torch.float32).pin_memory()
    hst.copy_(state.cpu())
    hnp = hst.numpy()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        s.stack_host_inplace(hnp, 1)
    e2e_s = time.perf_counter() - t0
    s.close()
    # the host link's measured copy rate: 1 GiB pinned -> device, event-timed
    src = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    dst = torch.empty(1 << 30, dtype=torch.uint8, device="cuda")
    for _ in range(2):
        dst.copy_(src, non_blocking=True)
    torch.cuda.synchronize()
    c0 = torch.cuda.Event(enable_timing=True)
    c1 = torch.cuda.Event(enable_timing=True)
    c0.record()
    for _ in range(4):
        dst.copy_(src, non_blocking=True)
    c1.record()
    torch.cuda.synchronize()
    link_gbs = 4 * (1 << 30) / (c0.elapsed_time(c1) / 1e3) / 1e9
    del src, dst
    ms = t_ms / args.steps
    moved = fet * slot_b / args.steps
    achieved = moved / (ms / 1e3) / 1e9
    return {
        "metric": f"MoE-stack decode tok/s, experts streamed from host memory (40-layer "
                  f"{'FP8' if fp8 else 'MXFP4'}, 1 B200)",
        "value": round(args.steps / (t_ms / 1e3), 2), "unit": "tok/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": ("fp8-e4m3" if fp8 else "mxfp4 (e2m1 + e8m0/32)") + " weights, fp32 accumulate",
        "data": "synthetic (seeded, device-generated, read back into host memory)",
        "config": {"workload": f"stream-decode: 40-layer {'FP8' if fp8 else 'MXFP4'} decode, pool "
                               f"{pool_b / 1e9:.1f} GB in pinned host memory, {n_slots} HBM slots",
                   "slots": n_slots, "pool_experts": LAYERS * E,
                   "hit_rate": round(hit / max(req, 1), 4),
                   "fetched_per_step": round(fet / args.steps, 2),
                   "parallelism": "single GPU"},
        "roofline": {"bound": "host link", "achieved": round(achieved, 2), "peak": round(link_gbs, 2),
                     "unit": "GB/s", "frac": round(achieved / link_gbs, 4), "traffic": None,
                     "peak_source": "pinned host-to-device copy of 1 GiB, measured in this run",
                     "bytes_copied_per_step": round(moved)},
        "e2e": {"value": round(args.steps / e2e_s, 2), "unit": "tok/s",
                "h2d_bytes_per_step": H * 4 + round(moved), "d2h_bytes_per_step": H * 4,
                "timer": "host clock around the synchronous C-ABI call"},
        "gpu_launches": 4 * LAYERS * args.steps,   # route, top-K, gate/up, down per layer
        "clocks": clocks,
    }


# DRAM bytes (read + write) of one k_head_bf16 launch over the 248,320-row head:
# the ncu capture of a 62,080-row head (--workload head --head-rows 62080),
# 254,331,904 + 2,894,848 bytes, times 4 (a launch reads its weights once)
HEAD_TRAFFIC_PER_LAUNCH = 4 * (254_331_904 + 2_894_848)


def run_gpu_head(args, rank, world, local_rank):
    """The output head after the MoE stack (ds4f_head_logits + ds4f_argmax,
    src/head.c:243-309): Qwen3.5's 248,320 x 2048 vocabulary matrix in BF16,
    logits and the greedy pick per step. Bytes per step = the weights
    (1.02 GB, larger than L2) + x + logits."""
    import numpy as np
    import torch
    dc = ds4f_cuda()
    torch.cuda.set_device(local_rank)
    dc.init()
    V, Hh = args.head_rows, H
    w = torch.empty(V * Hh, dtype=torch.bfloat16).normal_(0, 0.02, generator=torch.Generator().manual_seed(0))
    hd = dc.Head(dc.HEAD_BF16, w.view(torch.int16).numpy(), V=V, H=Hh)
    del w
    x = torch.randn(Hh, device="cuda", generator=torch.Generator("cuda").manual_seed(1))
    logits = torch.empty(V, device="cuda")
    best = torch.empty(1, dtype=torch.int32, device="cuda")
    sp = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(args.warmup):
        hd.logits_dev(x, logits, best, sp)
    torch.cuda.synchronize()
    clk = Clocks(local_rank)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        hd.logits_dev(x, logits, best, sp)
    e1.record()
    torch.cuda.synchronize()
    t_ms = e0.elapsed_time(e1)
    clocks = clk.stop()
    xh = x.cpu().numpy()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        _, b = hd.logits(xh, want_logits=False)
    e2e_s = time.perf_counter() - t0
    hd.close()
    ms = t_ms / args.steps
    algo = V * Hh * 2 + Hh * 4 + V * 4
    peak, src = peaks()
    gbs = algo / (ms / 1e3) / 1e9
    return {
        "metric": f"output head tokens/s ({V:,} x 2048 BF16 logits + argmax, 1 B200)",
        "value": round(1e3 / ms, 2), "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 weights, fp32 accumulate", "data": "synthetic (seeded N(0, 0.02) weights)",
        "config": {"workload": f"head: vocabulary head, {V:,} x 2048 BF16, batch 1",
                   "l2": "inputs larger than L2 (1.02 GB of weights per step)", "parallelism": "single GPU"},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(gbs / peak, 4), "traffic": round(HEAD_TRAFFIC_PER_LAUNCH * V / 248_320),
                     "traffic_unit": "bytes per k_head_bf16 launch (ncu of a 62,080-row head scaled by rows)",
                     "kernel": "k_head_bf16 (one warp per row, 4 blocks per SM) + argmax",
                     "peak_source": src, "algorithmic_bytes_per_step": algo},
        "e2e": {"value": round(args.steps / e2e_s, 2), "unit": "tok/s", "h2d_bytes_per_step": Hh * 4,
                "d2h_bytes_per_step": 4, "timer": "host clock around ds4f_gpu_head_logits"},
        "gpu_launches": 3 * args.steps,           # matvec, argmax partials, argmax final
        "clocks": clocks,
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--layered", action="store_true",
                    help="per-layer kernels (CUDA graph) instead of the persistent kernel")
    ap.add_argument("--workload", default="decode",
                    choices=["decode", "prefill", "ep-decode", "ep-prefill", "matvec", "stream-decode", "head"],
                    help="decode: config 2 (the headline); prefill: config 4; ep-decode: config 3 "
                         "(experts sharded over the ranks); stream-decode: the pool in host memory")
    ap.add_argument("--fmt", default=None, choices=["fp8", "mxfp4"],
                    help="expert format (decode default fp8; ep-decode default mxfp4)")
    ap.add_argument("--batch", type=int, default=1, help="ep-decode: tokens per step")
    ap.add_argument("--head-rows", type=int, default=248_320,
                    help="head: vocabulary rows (default Qwen3.5's 248,320; smaller for profiling)")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="decode / prefill: layers of the stack (fewer: a profiling case, not a bench line)")
    ap.add_argument("--tokens", type=int, default=2048, help="prefill: tokens per chunk")
    ap.add_argument("--ep-whole", action="store_true",
                    help="N > 1 decode: every expert on every GPU, the K selections split by index (fused step)")
    ap.add_argument("--ep-layered", action="store_true",
                    help="ep-decode / N > 1: the per-layer kernels with an NCCL all-reduce per layer instead of "
                         "the fused persistent launch")
    ap.add_argument("--trace-dump", default=None,
                    help="N > 1 decode with --trace: save each rank's raw stamps to <prefix>.r<rank>.npy")
    ap.add_argument("--trace", action="store_true",
                    help="decode: print k_decode's per-phase trace (stderr) and add it to the line")
    ap.add_argument("--slots", type=int, default=0,
                    help="stream-decode: HBM expert slots (default a quarter of the pool)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return
        n = max(1, args.steps)
        # built once; K samples sized so that warm-up and timing take ~2 minutes
        per = max(0.25, min(20.0, 120.0 / (n + 0.25)))
        value, desc = cpu_reference_median(n, per, per / 4, threads=min(8, os.cpu_count() or 1))
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "tok/s",
            "n_gpus": 0, "steps": n, "warmup": args.warmup, "higher_is_better": True,
            "config": decode_config(True, 1),
            "cpu_baseline": dict(desc, value=round(value, 4), unit="tok/s"),
            "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}))
        return
    if args.fmt is None:
        args.fmt = "mxfp4" if args.workload in ("ep-decode", "stream-decode") else "fp8"
    fn = {"prefill": run_gpu_prefill, "ep-decode": run_gpu_ep,
          "ep-prefill": run_gpu_ep_prefill, "matvec": run_gpu_matvec,
          "stream-decode": run_gpu_stream, "head": run_gpu_head}.get(args.workload, run_gpu)
    if world > 1 and args.workload == "decode":
        fn = run_gpu_ep            # N > 1: the expert-sharded design, not replicas
    res = fn(args, rank, world, local_rank)
    if rank == 0:
        if "unavailable" in res or args.workload in ("stream-decode", "head"):
            pass
        elif world == 1 and args.workload == "matvec":
            v, desc = cpu_matvec_sample(args.cpu_seconds)
            res["cpu_baseline"] = dict(desc, value=round(v, 4), unit="GB/s")
        elif world == 1 and args.workload == "decode":
            # the reference arm's procedure on a smaller budget: one warm-up
            # sample, the median of five
            per = max(0.2, args.cpu_seconds / 6)
            v, desc = cpu_reference_median(5, per, per, threads=min(8, os.cpu_count() or 1))
            res["cpu_baseline"] = dict(desc, value=round(v, 4), unit="tok/s")
        print(json.dumps(res))


if __name__ == "__main__":
    main()
