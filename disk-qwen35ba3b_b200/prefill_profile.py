#!/usr/bin/env python
"""prefill_profile.py -- run the tensor-core batched prefill
(ds4f_gpu_prefill) on a seeded FP8 model of a chosen depth and chunk size.

    python prefill_profile.py [--layers L] [--tokens T] [--steps N] [--warmup W]

The small case for ncu captures of the prefill kernels (for example
--layers 2: a 1.6 GB pool; every layer's GEMMs read ~805 MB of expert
weights, larger than the 126 MB L2). The times it prints are CUDA-event
figures of a reduced model, not bench values.
"""
import argparse
import importlib.util
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))


def _binding():
    spec = importlib.util.spec_from_file_location("ds4f_cuda", os.path.join(HERE, "ds4f_cuda.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--tokens", type=int, default=2048)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=1)
    args = ap.parse_args()

    import torch
    from bench import zipf_routing
    dc = _binding()
    dc.init()
    H, M, E, K, T = 2048, 512, 256, 8, args.tokens
    m = dc.Model(dc.FMT_FP8, args.layers, H, M, E, K)
    m.synth(0)
    sel, w = zipf_routing(args.layers, T, E, K, seed=100)
    selg, wg = torch.from_numpy(sel).cuda(), torch.from_numpy(w).cuda()
    x0 = torch.empty((T, H), dtype=torch.float32, device="cuda")
    dc.synth_f32_dev(x0, T * H, 0, 0, 4, 0, 1, 1.0)
    x0 = x0.bfloat16().float()
    st = torch.empty_like(x0)
    sp = torch.cuda.current_stream().cuda_stream
    for _ in range(args.warmup):
        st.copy_(x0)
        m.prefill_dev(st, selg, wg, sp)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        st.copy_(x0)
        m.prefill_dev(st, selg, wg, sp)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / max(1, args.steps)
    m.close()
    print(json.dumps({"layers": args.layers, "tokens": T, "steps": args.steps,
                      "ms_per_step": round(ms, 3), "ms_per_layer": round(ms / args.layers, 3)}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
