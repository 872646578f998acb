#!/usr/bin/env python
"""decode_profile.py -- run the persistent decode kernel on a seeded model
of a chosen depth and, optionally, print its phase trace.

The per-phase timers of the reference's decode loop (src/main.c:253-258,
1522-1546) have their counterpart in the kernel's %globaltimer stamps
(ds4f_gpu_model_trace); this script reads them back and prints, per phase,
the median over layers of the median (and max) over CTAs.

    python decode_profile.py [--fmt fp8|mxfp4] [--layers L] [--steps N]
                             [--warmup W] [--trace]

It is also the small case for ncu captures of k_decode: with --layers 4 the
FP8 pool is 3.2 GB and one launch reads 130 MB of weights (larger than the
126 MB L2). The times it prints are wall-clock-free CUDA-event figures of a
reduced model, not bench values.
"""
import argparse
import importlib.util
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))

PHASES = ["start", "state", "norm", "rows_done", "routes_vis", "topk", "issued",
          "softmax", "grp0", "chains", "down_in", "written"]
N_STAMPS = 20          # stamp slots per (layer-step, CTA) in the kernel


def _binding():
    spec = importlib.util.spec_from_file_location("ds4f_cuda", os.path.join(HERE, "ds4f_cuda.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def phase_table(tr):
    """tr: int64 [L, G, N_STAMPS] %globaltimer stamps of one step."""
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
    # slot 18: every router word visible (between rows_done and routes_vis)
    inner = np.diff(tr[:, :, [3, 18, 4]], axis=2)
    for k, name in enumerate(["routes: gather", "routes: top-K"]):
        rows.append((name, float(np.median(inner[:, :, k]) / 1e3),
                     float(np.median(np.max(inner[:, :, k], axis=1)) / 1e3)))
    out["phases_us"] = rows
    # slots 14-16: copy rounds of the state, router and chain gathers
    rounds = tr[:, :, 14:17].astype(np.float64)
    if L > 1:
        rounds = rounds[1:]          # layer 0 reads the state directly
    out["gather_rounds_mean"] = {n: round(float(rounds[:, :, k].mean()), 2)
                                 for k, n in enumerate(["state", "router", "chains"])}
    # slot 17: bit g set when gate/up group g had landed before its compute
    landed = tr[:, :, 17]
    out["group_landed_early"] = [round(float(((landed >> g) & 1).mean()), 3) for g in range(4)]
    if L > 1:
        lay = (tr[1:, :, 0].min(axis=1) - tr[:-1, :, 0].min(axis=1)) / 1e3
        out["layer_period_us"] = {"median": float(np.median(lay)), "min": float(lay.min()),
                                  "max": float(lay.max())}
    out["step_us"] = float((tr[-1, :, 11].max() - tr[0, :, 0].min()) / 1e3)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--fmt", default="fp8", choices=["fp8", "mxfp4"])
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--trace", action="store_true")
    args = ap.parse_args()

    import torch
    dc = _binding()
    dc.init()
    H, M, E, K = 2048, 512, 256, 8
    fmt = dc.FMT_FP8 if args.fmt == "fp8" else dc.FMT_MXFP4
    m = dc.Model(fmt, args.layers, H, M, E, K)
    m.synth(0)
    m.set_path(dc.PATH_PERSISTENT)
    st = torch.empty(H, device="cuda")
    dc.synth_f32_dev(st, H, 0, 0, 4, 0, 0, 1.0)
    sp = torch.cuda.current_stream().cuda_stream
    for _ in range(args.warmup):
        m.stack_dev(st, 1, sp)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        m.stack_dev(st, 1, sp)
    e1.record()
    torch.cuda.synchronize()
    res = {"fmt": args.fmt, "layers": args.layers, "steps": args.steps,
           "us_per_step": round(e0.elapsed_time(e1) * 1e3 / max(1, args.steps), 2)}
    if args.trace:
        import numpy as np
        G = torch.cuda.get_device_properties(0).multi_processor_count
        n = args.layers * G * N_STAMPS
        m.trace(n)
        m.stack_dev(st, 1, sp)
        torch.cuda.synchronize()
        tr = m.trace_read(n).astype(np.int64).reshape(args.layers, G, N_STAMPS)
        m.trace(0)
        res.update(phase_table(tr))
    res["router_exact_fallbacks"] = int(m.stats()[1])
    m.close()
    if args.trace:
        for name, med, mx in res.pop("phases_us"):
            print(f"  {name:<24s} {med:8.2f} {mx:8.2f}   (us: median, max over CTAs)")
    print(json.dumps(res))
    return 0


if __name__ == "__main__":
    sys.exit(main())
