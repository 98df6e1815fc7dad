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


def test_signal_barrier_single_rank_and_absent_rank(ann):
    """ann_signal_barrier on one GPU, no multicast, no peer memory: with one
    rank every epoch completes at once; with a second rank that never signals
    (its word is a flag nothing sets) the bounded wait runs out, reports
    ANN_DEVERR_WAIT_TIMEOUT, and the context stays usable."""
    import ctypes

    import torch
    from alpakann_b200 import _capi
    queue = ann.Queue()
    assert queue.take_device_error() == 0
    sig = torch.zeros(2, dtype=torch.int32, device="cuda")
    one = torch.tensor([sig.data_ptr()], dtype=torch.int64, device="cuda")
    for epoch in (1, 2, 3):
        _capi.check(_capi.lib.ann_signal_barrier(queue.handle, ctypes.c_void_p(sig.data_ptr()),
                                                 ctypes.c_void_p(one.data_ptr()), 1, 0, epoch, 1_000_000_000))
    assert queue.take_device_error() == 0
    assert sig[0].item() == 3
    sig.zero_()
    two = torch.tensor([sig.data_ptr(), sig.data_ptr()], dtype=torch.int64, device="cuda")
    _capi.check(_capi.lib.ann_signal_barrier(queue.handle, ctypes.c_void_p(sig.data_ptr()),
                                             ctypes.c_void_p(two.data_ptr()), 2, 0, 1, 20_000_000))  # 20 ms
    assert queue.take_device_error() & _capi.ANN_DEVERR_WAIT_TIMEOUT
    assert sig.tolist() == [1, 0]
    x = torch.randn(1000, device="cuda")
    y = torch.empty_like(x)
    ann.onHost.ops.scale(queue, None, x, 2.0, y)
    assert torch.equal(y, x * 2)
    with pytest.raises(_capi.AnnShapeError):  # epochs start at 1
        _capi.check(_capi.lib.ann_signal_barrier(queue.handle, ctypes.c_void_p(sig.data_ptr()),
                                                 ctypes.c_void_p(one.data_ptr()), 1, 0, 0, 1_000_000))


def test_signal_barrier_dev_epochs_and_graph_replay(ann):
    """ann_signal_barrier_dev keeps the epoch in device memory: it advances with
    every call, also when the call is captured in a CUDA graph and replayed;
    with a second rank that never signals the bounded wait runs out as for
    ann_signal_barrier (no multicast, no peer memory)."""
    import ctypes

    import torch
    from alpakann_b200 import _capi
    lib = _capi.lib
    s = torch.cuda.Stream()
    queue = ann.Queue(s)
    assert queue.take_device_error() == 0
    sig = torch.zeros(2, dtype=torch.int32, device="cuda")
    word = torch.zeros(1, dtype=torch.int32, device="cuda")
    one = torch.tensor([sig.data_ptr()], dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()

    def barrier(peers, nranks, timeout_ns=1_000_000_000):
        _capi.check(lib.ann_signal_barrier_dev(queue.handle, ctypes.c_void_p(sig.data_ptr()),
                                               ctypes.c_void_p(peers.data_ptr()), nranks, 0,
                                               ctypes.c_void_p(word.data_ptr()), timeout_ns))

    for _ in range(2):
        barrier(one, 1)
    s.synchronize()
    assert word.item() == 2 and sig[0].item() == 2
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        barrier(one, 1)
    with torch.cuda.stream(s):
        for _ in range(3):
            g.replay()
    s.synchronize()
    assert word.item() == 5 and sig[0].item() == 5  # captured once, three new epochs
    assert queue.take_device_error() == 0
    del g
    sig.zero_()
    word.zero_()
    two = torch.tensor([sig.data_ptr(), sig.data_ptr()], dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()
    barrier(two, 2, 20_000_000)  # 20 ms
    assert queue.take_device_error() & _capi.ANN_DEVERR_WAIT_TIMEOUT
    assert sig.tolist() == [1, 0] and word.item() == 1
    with pytest.raises(_capi.AnnShapeError):  # an epoch word is required
        _capi.check(lib.ann_signal_barrier_dev(queue.handle, ctypes.c_void_p(sig.data_ptr()),
                                               ctypes.c_void_p(one.data_ptr()), 1, 0, None, 1_000_000))

