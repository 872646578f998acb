"""ds4f_gpu_pool_load_json: a packed pool with the converter's layout file
(tools/convert-ds4f.py:1321-1393) loaded into HBM, each tensor placed by
name whatever its order in the file slot.

  * a model's own experts written in the converter's order (down, gate, up:
    the order of the pool the reference's converter wrote,
    tests/golden/refpool, on which tests/test_poolfile.py pins the layout
    reader) and loaded into a second model: every expert slot
    byte-identical, every layer step bit-identical; a shard loads its own
    experts;
  * a packed file whose header disagrees with its layout file is refused."""
import importlib.util
import os

import numpy as np
import pytest

from tests._lib import PKG, ds4f_cuda

pytestmark = pytest.mark.gpu
dc = ds4f_cuda()
spec = importlib.util.spec_from_file_location("poolfile", os.path.join(PKG, "poolfile.py"))
pf = importlib.util.module_from_spec(spec)
spec.loader.exec_module(pf)


@pytest.fixture(scope="module", autouse=True)
def gpu():
    dc.init()
    yield


@pytest.mark.parametrize("fmt", [dc.FMT_FP8, dc.FMT_MXFP4])
def test_converter_order_pool_round_trip(tmp_path, fmt):
    L, H, M, E, K = 2, 1024, 256, 16, 8
    r = dc.Model(fmt, L, H, M, E, K)
    r.synth(11 + fmt)
    b, j = tmp_path / "pool.bin", tmp_path / "pool.json"
    pf.write_pool(b, j, fmt, L, E, H, M, r.get_expert)
    m = dc.Model(fmt, L, H, M, E, K)
    for l in range(L):
        m.set_trunk(l, *r.get_trunk(l))
    m.pool_load_json(b, j)
    for l in range(L):
        for x in range(E):
            assert np.array_equal(m.get_expert(l, x), r.get_expert(l, x)), (l, x)
    x = np.random.default_rng(3).standard_normal(H).astype(np.float32)
    for l in range(L):
        xr, ir, wr = r.layer(l, x)
        xm, im, wm = m.layer(l, x)
        assert np.array_equal(ir, im)
        assert np.array_equal(xr.view(np.uint32), xm.view(np.uint32))
        x = xr
    # an expert-parallel shard loads its own experts only
    s = dc.Model(fmt, L, H, M, E, K, expert_first=4, expert_count=8)
    s.pool_load_json(b, j)
    for l in range(L):
        for x in range(4, 12):
            assert np.array_equal(s.get_expert(l, x), r.get_expert(l, x))
    for mm in (s, m, r):
        mm.close()


def test_header_disagreeing_with_layout_is_refused(tmp_path):
    L, H, M, E, K = 1, 1024, 256, 8, 8
    slots = np.zeros((L, E + 1, sum(sum(pf.tensor_bytes(dc.FMT_MXFP4, *s))
                                    for s in ((M, H), (M, H), (H, M)))), np.uint8)
    b, j = tmp_path / "p.bin", tmp_path / "p.json"
    b2, j2 = tmp_path / "q.bin", tmp_path / "q.json"
    pf.write_pool(b, j, dc.FMT_MXFP4, L, E, H, M, lambda l, x: slots[l, x])
    pf.write_pool(b2, j2, dc.FMT_MXFP4, L, E + 1, H, M, lambda l, x: slots[l, x])
    m = dc.Model(dc.FMT_MXFP4, L, H, M, E, K)
    with pytest.raises(dc.GpuError, match="header"):
        m.pool_load_json(b2, j)          # 9-expert file, 8-expert layout
    with pytest.raises(dc.GpuError, match="format"):
        dc.Model(dc.FMT_FP8, L, H, M, E, K).pool_load_json(b, j)
    m.pool_load_json(b, j)
    m.close()
