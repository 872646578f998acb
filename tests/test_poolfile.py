"""The converter's pool layout file (pool-*.json beside a packed pool,
tools/convert-ds4f.py:1321-1393; the engine's reader src/moe.c:51-160) as
read by ds4f_pool_layout_plan. CPU only: the plan is host code.

Pinned on a pool written by the reference's own converter
(tests/golden/refpool, made by tests/golden/make_refpool.py): every tensor
the plan places as gate, up or down decodes to that tensor's source
weights."""
import copy
import ctypes as C
import importlib.util
import json
import os

import numpy as np
import pytest

from tests._lib import PKG, ROOT, ds4f_cuda

dc = ds4f_cuda()
spec = importlib.util.spec_from_file_location("poolfile", os.path.join(PKG, "poolfile.py"))
pf = importlib.util.module_from_spec(spec)
spec.loader.exec_module(pf)

REF = os.path.join(ROOT, "tests", "golden", "refpool")
ROLES = ("gate_proj", "up_proj", "down_proj")


def e4m3(b):
    """E4M3 byte -> value, exponent field below 15 (src/kernels.c:228-237)."""
    b = b.astype(np.int64)
    e, m = (b >> 3) & 15, b & 7
    v = np.where(e == 0, m * 2.0 ** -9, (1 + m / 8.0) * 2.0 ** (e - 7))
    return np.where(b & 0x80, -v, v)


def mxfp4(vals, scales, R, Cc):
    """e2m1 pairs (even index low nibble) x E8M0 per 32 (src/kernels.c:24-46)."""
    mag = np.array([0, .5, 1, 1.5, 2, 3, 4, 6])
    nib = np.stack([vals & 15, vals >> 4], 1).reshape(-1).astype(np.int64)
    v = np.where(nib & 8, -1.0, 1.0) * mag[nib & 7]
    s = np.ldexp(1.0, scales.astype(np.int64) - 127)
    return (v * np.repeat(s, 32)[:v.size]).reshape(R, Cc)


def test_reference_written_pool_places_each_tensor():
    """Each tensor the plan places as gate, up or down decodes to weights
    whose max error against that tensor's source equals the err_max the
    converter recorded for it (computed in float32 as the converter does,
    tools/convert-ds4f.py:1335-1347, :1074-1077) -- and differs for the
    other role of the same shape."""
    meta = json.load(open(os.path.join(REF, "pool-mxfp4.json")))
    L, E = meta["n_layers"], meta["n_experts"]
    H, M = 64, 32
    off, nb = dc.pool_layout_plan(os.path.join(REF, "pool-mxfp4.json"),
                                  dc.FMT_MXFP4, H, M, L, E)
    assert nb == meta["expert_nbytes"] == 3264
    raw = np.fromfile(os.path.join(REF, "pool-mxfp4.bin"), np.uint8)
    src = np.load(os.path.join(REF, "source.npz"))
    # the converter's slot order is the sorted names: down, gate, up
    first = [t["n"].rsplit(".", 2)[-2] for t in meta["tensors"][:3]]
    assert first == ["down_proj", "gate_proj", "up_proj"]
    recorded = {(t["layer"], t["expert"], t["n"].rsplit(".", 2)[-2]): t["err_max"]
                for t in meta["tensors"]}

    def source(l, x, role, R, Cc):
        return (e4m3(src[f"w_{l}_{x}_{role}"]).astype(np.float32).reshape(R, Cc) *
                src[f"s_{l}_{x}_{role}"][:, None])

    for l in range(L):
        for x in range(E):
            for r, role in enumerate(ROLES):
                R, Cc = (H, M) if role == "down_proj" else (M, H)
                vo, so = off[l, x, r]
                dec = mxfp4(raw[vo:vo + R * Cc // 2], raw[so:so + R * Cc // 32],
                            R, Cc).astype(np.float32)
                err = float(np.max(np.abs(dec - source(l, x, role, R, Cc))))
                assert err == recorded[(l, x, role)], (l, x, role, err)
                if role != "down_proj":
                    other = "up_proj" if role == "gate_proj" else "gate_proj"
                    e2 = float(np.max(np.abs(dec - source(l, x, other, R, Cc))))
                    assert e2 != recorded[(l, x, role)]


def _slots(fmt, L, E, H, M, seed):
    nb = sum(sum(pf.tensor_bytes(fmt, *s)) for s in ((M, H), (M, H), (H, M)))
    rng = np.random.default_rng(seed)
    return rng.integers(0, 256, (L, E, nb), dtype=np.uint8)


@pytest.mark.parametrize("fmt,H,M", [(dc.FMT_MXFP4, 64, 32), (dc.FMT_FP8, 256, 128)])
@pytest.mark.parametrize("order,names", [(pf.CONVERTER_ORDER, True),
                                         (pf.ROLES, True),
                                         (("up", "down", "gate"), True),
                                         (pf.ROLES, False)])
def test_plan_reads_any_tensor_order(tmp_path, fmt, H, M, order, names):
    L, E = 2, 3
    slots = _slots(fmt, L, E, H, M, 7)
    b, j = tmp_path / "pool.bin", tmp_path / "pool.json"
    pf.write_pool(b, j, fmt, L, E, H, M, lambda l, x: slots[l, x], order=order, names=names)
    off, nb = dc.pool_layout_plan(j, fmt, H, M, L, E)
    raw = np.fromfile(b, np.uint8)
    for l in range(L):
        for x in range(E):
            parts = pf.split_slot(fmt, H, M, slots[l, x])
            for r, role in enumerate(pf.ROLES):
                v, s = parts[role]
                vo, so = off[l, x, r]
                assert np.array_equal(raw[vo:vo + v.size], v)
                assert np.array_equal(raw[so:so + s.size], s)


def _base(tmp_path, fmt=dc.FMT_MXFP4, H=64, M=32, L=2, E=3):
    slots = _slots(fmt, L, E, H, M, 1)
    b, j = tmp_path / "pool.bin", tmp_path / "pool.json"
    pf.write_pool(b, j, fmt, L, E, H, M, lambda l, x: slots[l, x])
    return json.load(open(j)), j


def _refused(tmp_path, meta, needle, H=64, M=32, L=2, E=3, fmt=dc.FMT_MXFP4, text=None):
    p = tmp_path / "bad.json"
    p.write_text(text if text is not None else json.dumps(meta))
    with pytest.raises(dc.GpuError, match=needle):
        dc.pool_layout_plan(p, fmt, H, M, L, E)


def test_plan_refusals(tmp_path):
    meta, _ = _base(tmp_path)
    m = copy.deepcopy(meta); m["n_layers"] = 3
    _refused(tmp_path, m, "vs model")
    m = copy.deepcopy(meta); del m["tensors"]
    _refused(tmp_path, m, "missing keys")
    m = copy.deepcopy(meta); m["format"] = "fp8-pool-v1"
    _refused(tmp_path, m, "format")
    m = copy.deepcopy(meta); m["tensors"][1]["shape"] = [64, 32]
    _refused(tmp_path, m, "shape")
    m = copy.deepcopy(meta); m["tensors"][0]["v_nbytes"] += 2
    _refused(tmp_path, m, "value")
    m = copy.deepcopy(meta); m["tensors"][4]["v_off"] = 5
    _refused(tmp_path, m, "out of slot bounds")
    m = copy.deepcopy(meta); m["tensors"][2]["s_off"] += meta["expert_nbytes"]
    _refused(tmp_path, m, "out of slot bounds")
    m = copy.deepcopy(meta); m["tensors"][2]["n"] = m["tensors"][1]["n"]
    _refused(tmp_path, m, "twice")
    m = copy.deepcopy(meta); del m["tensors"][5]
    _refused(tmp_path, m, "lacks")
    m = copy.deepcopy(meta); m["tensors"][0]["n"] = "layers.0.ffn.experts.0.w1.weight"
    _refused(tmp_path, m, "not a gate_proj")
    # sizes whose slot offsets 24 + (L E) nb would leave int64, and a
    # negative tensor offset: refused before any arithmetic on them
    for nb in (2 ** 62, 2 ** 63 - 1, (2 ** 63 - 24) // 6 + 1):
        m = copy.deepcopy(meta); m["expert_nbytes"] = nb
        _refused(tmp_path, m, "expert_nbytes")
    m = copy.deepcopy(meta); m["tensors"][3]["v_off"] = -(2 ** 63) + 5
    _refused(tmp_path, m, "negative offset")
    _refused(tmp_path, None, "not parseable", text=json.dumps(meta)[:-40])
    _refused(tmp_path, None, "not parseable", text='{"n_layers": 01}')
    with pytest.raises(dc.GpuError, match="cannot read"):
        dc.pool_layout_plan(tmp_path / "absent.json", dc.FMT_MXFP4, 64, 32, 2, 3)


def test_plan_skips_entries_as_the_engine_does(tmp_path):
    """Entries missing a per-tensor key, or with a layer / expert out of
    range, are ignored (src/moe.c:97-101)."""
    meta, _ = _base(tmp_path)
    m = copy.deepcopy(meta)
    m["tensors"].append({"n": "stray", "layer": 9, "expert": 0, "shape": [1],
                         "v_off": 0, "s_off": 0, "v_nbytes": 0, "s_nbytes": 0})
    m["tensors"].append({"layer": 0, "expert": 0})
    p = tmp_path / "skip.json"
    p.write_text(json.dumps(m))
    dc.pool_layout_plan(p, dc.FMT_MXFP4, 64, 32, 2, 3)


def test_json_reader_corner_cases(tmp_path):
    meta, j = _base(tmp_path)
    # escapes, unicode, nested values, floats, literals and odd spacing
    t0 = meta["tensors"][0]
    t0["n"] = t0["n"].replace("down_proj", "down\\u005fproj")
    body = json.dumps(meta, indent=None).replace("down\\\\u005fproj", "down\\u005fproj")
    assert "down\\u005fproj" in body
    body = body.replace('"tensors":', '"extra": {"a": [1.5e-3, -0.0, true, false, null, "\\u00e9\\ud83d\\ude00"]},\n\t "tensors" :')
    p = tmp_path / "odd.json"
    p.write_text(body)
    off, nb = dc.pool_layout_plan(p, dc.FMT_MXFP4, 64, 32, 2, 3)
    ref, _ = dc.pool_layout_plan(j, dc.FMT_MXFP4, 64, 32, 2, 3)
    assert np.array_equal(off, ref)


# ---- against the reference's own layout loader ------------------------------
# ds4f_pool_layout_load (src/moe.c:51-160) is compiled into oracle/_ref with
# the rest of moe.c; the structures below mirror include/ds4f/moe.h:20-44 and
# include/ds4f/ds4f.h:56-75 (x86-64, LP64).

class _MoETensor(C.Structure):
    _fields_ = [("dims", C.c_long * 4), ("rank", C.c_int), ("rel_v", C.c_long),
                ("rel_s", C.c_long), ("rel_b", C.c_long), ("v_nbytes", C.c_long),
                ("s_nbytes", C.c_long), ("bsize", C.c_int), ("fmt", C.c_int)]


class _ExpertLayout(C.Structure):
    _fields_ = [("n", C.c_int), ("chain", C.c_int), ("t", _MoETensor * 8)]


class _PoolLayout(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("n_experts", C.c_int),
                ("expert_nbytes", C.c_int64), ("max_rc", C.c_int64),
                ("exp", C.POINTER(_ExpertLayout))]


class _Cfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_layers", "n_experts", "topk", "n_shared", "hidden",
                                       "latent", "moe_inter", "n_heads", "n_kv_heads", "qk_rope")] + \
               [(n, C.c_double) for n in ("rope_factor", "rope_beta_fast", "rope_beta_slow",
                                          "rope_max_pos", "rope_theta")] + \
               [("expert_nbytes", C.c_int64), ("n_shards", C.c_int), ("seed", C.c_uint64)]


def _ref_layout(path, L, E):
    """-> (rc, [[(rel_v, rel_s, dims) per entry] per expert]) from the
    reference's loader, or None when oracle/_ref is absent."""
    so = os.path.join(ROOT, "oracle", "_ref", "libds4f_ref.so")
    if not os.path.exists(so):
        return None
    R = C.CDLL(so)
    R.ds4f_pool_layout_load.argtypes = [C.POINTER(_PoolLayout), C.c_char_p, C.POINTER(_Cfg)]
    pl, cfg = _PoolLayout(), _Cfg()
    cfg.n_layers, cfg.n_experts = L, E
    rc = R.ds4f_pool_layout_load(C.byref(pl), str(path).encode(), C.byref(cfg))
    if rc != 0:
        return rc, None
    out = []
    for i in range(L * E):
        el = pl.exp[i]
        out.append([(el.t[k].rel_v, el.t[k].rel_s, list(el.t[k].dims[:el.t[k].rank]))
                    for k in range(el.n)])
    C.CDLL(None).free(C.cast(pl.exp, C.c_void_p))
    return rc, out


def _compare_with_reference(json_path, fmt, H, M, L, E):
    got = _ref_layout(json_path, L, E)
    if got is None:
        pytest.skip("oracle/_ref not built")
    rc, ref = got
    assert rc == 0
    off, nb = dc.pool_layout_plan(json_path, fmt, H, M, L, E)
    meta = json.load(open(json_path))
    entries = {}
    for t in meta["tensors"]:
        entries.setdefault((t["layer"], t["expert"]), []).append(t)
    for l in range(L):
        for x in range(E):
            base = 24 + (l * E + x) * nb
            ents = entries[(l, x)]
            assert len(ref[l * E + x]) == len(ents) == 3
            for k, t in enumerate(ents):
                role = (ROLES.index(t["n"].rsplit(".", 2)[-2]) if "n" in t else k)
                rv, rs, dims = ref[l * E + x][k]
                assert (rv, rs) == (off[l, x, role, 0] - base, off[l, x, role, 1] - base)
                assert dims == t["shape"]


def test_plan_agrees_with_reference_loader_on_converter_pool():
    _compare_with_reference(os.path.join(REF, "pool-mxfp4.json"), dc.FMT_MXFP4, 64, 32, 2, 4)


@pytest.mark.parametrize("order,names", [(pf.CONVERTER_ORDER, True), (pf.ROLES, False),
                                         (("up", "gate", "down"), True)])
def test_plan_agrees_with_reference_loader_on_written_pools(tmp_path, order, names):
    L, E, H, M = 3, 5, 64, 32
    slots = _slots(dc.FMT_MXFP4, L, E, H, M, 9)
    b, j = tmp_path / "pool.bin", tmp_path / "pool.json"
    pf.write_pool(b, j, dc.FMT_MXFP4, L, E, H, M, lambda l, x: slots[l, x], order=order, names=names)
    _compare_with_reference(j, dc.FMT_MXFP4, H, M, L, E)


def test_refusals_shared_with_reference_loader(tmp_path):
    meta, _ = _base(tmp_path)
    for mutate in (lambda m: m.__setitem__("n_layers", 5),
                   lambda m: m["tensors"][4].__setitem__("v_off", 5),
                   lambda m: m.pop("expert_nbytes")):
        m = copy.deepcopy(meta)
        mutate(m)
        p = tmp_path / "bad.json"
        p.write_text(json.dumps(m))
        got = _ref_layout(p, 2, 3)
        if got is None:
            pytest.skip("oracle/_ref not built")
        assert got[0] != 0
        with pytest.raises(dc.GpuError):
            dc.pool_layout_plan(p, dc.FMT_MXFP4, 64, 32, 2, 3)


def test_reader_survives_mutated_files(tmp_path):
    """Seeded byte flips, truncations, insertions and deletions of a valid
    layout file: every one either plans or is refused with an error -- none
    may crash the host process."""
    _, j = _base(tmp_path)
    good = j.read_bytes()
    rng = np.random.default_rng(11)
    p = tmp_path / "m.json"
    planned = refused = 0
    for i in range(1500):
        b = bytearray(good)
        for _ in range(int(rng.integers(1, 4))):
            kind = int(rng.integers(0, 4))
            at = int(rng.integers(0, len(b)))
            if kind == 0:
                b[at] = int(rng.integers(0, 256))
            elif kind == 1:
                del b[at:]
            elif kind == 2:
                b[at:at] = bytes(rng.choice(list(b'{}[]",:-0123456789.eE \\u'), int(rng.integers(1, 6))))
            else:
                del b[at:at + int(rng.integers(1, 8))]
            if not b:
                b = bytearray(b"{")
        p.write_bytes(bytes(b))
        try:
            dc.pool_layout_plan(p, dc.FMT_MXFP4, 64, 32, 2, 3)
            planned += 1
        except dc.GpuError:
            refused += 1
    assert planned + refused == 1500 and refused > 0
