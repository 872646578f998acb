"""Write a packed expert pool and its layout file in the converter's format
(tools/convert-ds4f.py:1321-1393): [u64 expert_nbytes][u64 n_layers]
[u64 n_experts], then one fixed-size slot per expert, layer-major; in a slot
each tensor's values then its scales; beside it a JSON with one entry per
tensor (name, layer, expert, shape, absolute v_off / s_off, byte counts).

"mxfp4-pool-v1" is the converter's MXFP4 pool (e2m1 two per byte, even
index in the low nibble, E8M0 per 32). "fp8-pool-v1" is the same container
for FP8 experts: E4M3 bytes row-major and one fp32 scale per 128x128 block,
row-major [R/128][C/128]. The tensor order in a slot defaults to the
converter's (sorted names: down, gate, up); ds4f_gpu_pool_load_json reads
any order.
"""
import json
import struct

import numpy as np

FMT_MXFP4, FMT_FP8 = 0, 2                    # DS4F_FMT_* of gpu_cuda.h
ROLES = ("gate", "up", "down")
CONVERTER_ORDER = ("down", "gate", "up")     # sorted(...) of the Qwen names


def tensor_bytes(fmt, rows, cols):
    """(value bytes, scale bytes) of one expert tensor."""
    n = rows * cols
    if fmt == FMT_FP8:
        return n, (rows // 128) * (cols // 128) * 4
    if fmt == FMT_MXFP4:
        return (n + 1) // 2, (n + 31) // 32
    raise ValueError(f"no pool format for fmt {fmt}")


def split_slot(fmt, hidden, moe_inter, slot):
    """This library's slot bytes (gate, up, down; values then scales each)
    -> {role: (values, scales)}."""
    out, o = {}, 0
    for r in ROLES:
        R, Cc = (hidden, moe_inter) if r == "down" else (moe_inter, hidden)
        vb, sb = tensor_bytes(fmt, R, Cc)
        out[r] = (slot[o:o + vb], slot[o + vb:o + vb + sb])
        o += vb + sb
    assert o == len(slot), (o, len(slot))
    return out


def write_pool(bin_path, json_path, fmt, n_layers, n_experts, hidden, moe_inter,
               get_slot, order=CONVERTER_ORDER, names=True):
    """get_slot(L, X) -> this library's slot bytes for expert X of layer L.
    order: tensor order within a file slot; names=False omits the "n" keys
    (the reader then takes entries in gate, up, down order, so the entries are
    listed in that order while the bytes keep `order`)."""
    fmt_name = "fp8-pool-v1" if fmt == FMT_FP8 else "mxfp4-pool-v1"
    shapes = {r: ([hidden, moe_inter] if r == "down" else [moe_inter, hidden])
              for r in ROLES}
    slot_nb = sum(sum(tensor_bytes(fmt, *shapes[r])) for r in ROLES)
    tensors = []
    with open(bin_path, "wb") as f:
        f.write(struct.pack("<QQQ", slot_nb, n_layers, n_experts))
        off = 24
        for L in range(n_layers):
            for X in range(n_experts):
                parts = split_slot(fmt, hidden, moe_inter,
                                   np.asarray(get_slot(L, X), np.uint8))
                ents = {}
                for r in order:
                    v, s = parts[r]
                    f.write(v.tobytes())
                    f.write(s.tobytes())
                    e = {"layer": L, "expert": X, "shape": shapes[r],
                         "v_off": off, "v_nbytes": int(v.size),
                         "s_off": off + int(v.size), "s_nbytes": int(s.size)}
                    if names:
                        e = {"n": f"model.language_model.layers.{L}.mlp.experts."
                                  f"{X}.{r}_proj.weight", **e}
                    ents[r] = e
                    off += int(v.size) + int(s.size)
                tensors += [ents[r] for r in (order if names else ROLES)]
    meta = {"format": fmt_name,
            "n_layers": n_layers, "n_experts": n_experts,
            "expert_nbytes": slot_nb, "tensors": tensors}
    if fmt_name == "mxfp4-pool-v1":
        meta.update({"block_size": 32,
                     "value_layout": "2 per byte, even index low nibble",
                     "scale_format": "E8M0 per 32-element block"})
    else:
        meta.update({"block_size": 128,
                     "value_layout": "E4M3 bytes, row-major",
                     "scale_format": "f32 per 128x128 block, row-major"})
    with open(json_path, "w") as f:
        json.dump(meta, f, indent=1)
    return slot_nb
