"""Failure detection on the GPU, without faulting it: a bounded wait that runs
out (ann_selftest_wait, nothing ever arrives on the barrier) gives up after its
limit, reports ANN_DEVERR_WAIT_TIMEOUT through the device error word that every
waiting kernel uses, and leaves the context usable: the next attention call
still matches the oracle."""
import math

import numpy as np
import pytest

import oracle
from tests.helpers import assert_close, normal, rng

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ann():
    from tests.helpers import build_library
    build_library()
    import alpakann_b200
    return alpakann_b200


def test_wait_that_runs_out_is_reported(ann):
    import torch
    from alpakann_b200 import _capi
    queue = ann.Queue()
    assert queue.take_device_error() == 0
    _capi.check(_capi.lib.ann_selftest_wait(queue.handle, 0, 5_000_000))  # 5 ms, nothing arrives
    bits = queue.take_device_error()
    assert bits & _capi.ANN_DEVERR_WAIT_TIMEOUT
    assert queue.take_device_error() == 0  # taking the word clears it
    # the context is still usable: a prefill right after matches the oracle
    g = rng(3)
    q, k, v = (normal(g, (1, 70, 2, 64), np.float32) for _ in range(3))
    o = torch.full((1, 70, 2, 64), float("nan"), device="cuda")
    ann.onHost.nn.attentionPrefill(queue, None, torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(),
                                   torch.from_numpy(v).cuda(), o, 0.125, 1, 0, True)
    torch.cuda.synchronize()
    s = np.empty((1, 2, 70, 70), np.float32)
    oracle.attention_scores(q, k, s, 1, 0)
    oracle.scale(s, np.float32(0.125), s)
    p = np.empty_like(s)
    oracle.causal_softmax(s, p, 3, 2, 3)
    ref = np.empty_like(q)
    oracle.attention_apply(p, v, ref, 1, 0)
    assert_close(o.cpu().numpy(), ref, np.float32, "prefill after a timed-out wait")
    assert queue.take_device_error() == 0


def test_wait_that_completes_reports_nothing(ann):
    from alpakann_b200 import _capi
    queue = ann.Queue()
    _capi.check(_capi.lib.ann_selftest_wait(queue.handle, 1, 5_000_000))
    assert queue.take_device_error() == 0
