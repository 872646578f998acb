"""Generate tests/golden/refpool/: an expert pool written by the reference's
own converter (tools/convert-ds4f.py quantize, run unmodified from the
reference tree) from a tiny Qwen3.5-named FP8 checkpoint made here.

The checkpoint: 2 layers x 4 experts, hidden 64, moe_inter 32; each
gate_proj / up_proj / down_proj weight is F8_E4M3 bytes with an F32 scale
per row (the converter's "row" scheme, tools/convert-ds4f.py:1262-1263).
The converter dequantises them with its E4M3 table, requantises to MXFP4 and
writes pool-mxfp4.bin + pool-mxfp4.json; both are kept with the source bytes
and scales (source.npz) so the tests can check where each tensor landed.

Run from the repository root, in a container that holds the reference:
    python tests/golden/make_refpool.py [/path/to/reference]
"""
import json
import os
import shutil
import struct
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "refpool")
NL, NE, H, M = 2, 4, 64, 32


def main(ref_root):
    conv = os.path.join(ref_root, "tools", "convert-ds4f.py")
    work = os.path.join(HERE, "_refpool_work")
    src, dst = os.path.join(work, "src"), os.path.join(work, "out")
    if os.path.exists(work):
        shutil.rmtree(work)
    os.makedirs(src)
    cfg = {"architectures": ["Qwen3_5MoeForConditionalGeneration"],
           "model_type": "qwen3_5_moe",
           "text_config": {"num_hidden_layers": NL, "hidden_size": H,
                           "num_experts": NE, "num_experts_per_tok": 2,
                           "moe_intermediate_size": M,
                           "shared_expert_intermediate_size": M}}
    with open(os.path.join(src, "config.json"), "w") as f:
        json.dump(cfg, f, indent=2)
    rng = np.random.default_rng(2024)
    hdr, payload, source = {}, bytearray(), {}
    shapes = {"gate_proj": (M, H), "up_proj": (M, H), "down_proj": (H, M)}
    for L in range(NL):
        for X in range(NE):
            for role, (R, Cc) in shapes.items():
                # E4M3 bytes with exponent field <= 14 (finite in every
                # reading of the format), either sign
                mag = rng.integers(0, 0x78, R * Cc, dtype=np.uint8)
                sign = rng.integers(0, 2, R * Cc, dtype=np.uint8) << 7
                w = (mag | sign).astype(np.uint8)
                s = (rng.uniform(0.5, 2.0, R) * 2.0 ** -9).astype(np.float32)
                base = f"model.language_model.layers.{L}.mlp.experts.{X}.{role}"
                for name, dt, shp, raw in ((base + ".weight", "F8_E4M3", [R, Cc], w.tobytes()),
                                           (base + ".scale", "F32", [R], s.tobytes())):
                    hdr[name] = {"dtype": dt, "shape": shp,
                                 "data_offsets": [len(payload), len(payload) + len(raw)]}
                    payload += raw
                source[f"w_{L}_{X}_{role}"] = w
                source[f"s_{L}_{X}_{role}"] = s
    hj = json.dumps(hdr).encode()
    with open(os.path.join(src, "model.safetensors"), "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        f.write(bytes(payload))
    subprocess.run([sys.executable, conv, "quantize", src, "--out", dst], check=True)
    os.makedirs(OUT, exist_ok=True)
    for fn in ("pool-mxfp4.bin", "pool-mxfp4.json"):
        shutil.copy(os.path.join(dst, fn), os.path.join(OUT, fn))
    np.savez_compressed(os.path.join(OUT, "source.npz"), **source)
    shutil.rmtree(work)
    print("wrote", OUT)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_refpool.py <reference tree>")
    main(sys.argv[1])
