"""Failure detection of the persistent decode kernel without a GPU fault.

Every wait in k_decode is bounded. The test hook ds4f_gpu_model_inject_stall
makes one CTA withhold its rows of the state at one layer-step (the words are
simply never written, as if that CTA had stalled); with a short wait limit
every other CTA's gather of the state gives up, records the error code and
its CTA, drains its own copies and returns. The call must then report -1
with that code through ds4f_gpu_last_error(), within the limit's time, and
the model must stay usable: the next call, with the hook off, gives exactly
the result of a model that never failed.
"""
import time

import numpy as np
import pytest

from oracle import pyoracle as po
from tests._lib import ds4f_cuda

pytestmark = pytest.mark.gpu
dc = ds4f_cuda()


@pytest.fixture(scope="module", autouse=True)
def gpu():
    dc.init()
    yield


@pytest.mark.parametrize("cta,layer_step", [(5, 1), (0, 2), (100, 0)])
def test_withheld_state_words_time_out_and_recover(cta, layer_step):
    m = dc.Model(dc.FMT_FP8, 4, 1024, 256, 64, 8)
    m.synth(12)
    m.set_path(dc.PATH_PERSISTENT)
    x = po.fill_f32(1024, po.key(12, 0, 4, 0, 0), 1.0)
    want = m.stack(x, 1)                            # a clean step first
    m.set_wait_limit(1 << 14)
    m.inject_stall(cta, layer_step)
    t0 = time.time()
    with pytest.raises(dc.GpuError, match=r"gave up waiting \(code 1 at CTA \d+\)"):
        m.stack(x, 1)
    assert time.time() - t0 < 10.0
    # the error is sticky until the next launch, which clears it
    with pytest.raises(dc.GpuError, match="gave up waiting"):
        m.stats()
    m.inject_stall(-1, 0)
    m.set_wait_limit(0)
    again = m.stack(x, 1)
    assert np.array_equal(again, want)
    m.stats()                                       # no error left
    m.close()


def test_wait_limit_alone_changes_nothing():
    """A short limit that no healthy wait reaches: identical results."""
    m = dc.Model(dc.FMT_MXFP4, 3, 1024, 256, 64, 8)
    m.synth(13)
    m.set_path(dc.PATH_PERSISTENT)
    x = po.fill_f32(1024, po.key(13, 0, 4, 0, 0), 1.0)
    want = m.stack(x, 2)
    m.set_wait_limit(1 << 20)
    assert np.array_equal(m.stack(x, 2), want)
    m.close()

