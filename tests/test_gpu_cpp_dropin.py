"""Runs the C++ drop-in test program (tests/cpp/test_dropin.cpp): the
reference's hot-path cases called through include/alpakann_b200/onHost.hpp."""
import subprocess

import pytest

pytestmark = pytest.mark.gpu


def test_cpp_dropin_program():
    from tests.cpp import build
    exe = build.build()
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert " 0 failures" in r.stdout


def test_cpp_dropin_builds():
    from tests.cpp import build
    assert build.build()


def test_cpp_decode_step_matches_python_api():
    """tests/cpp/decode_e2e.cpp -- the decode step written against the C++
    header with host buffers (rmsNorm, ropeInPlace, fused decode, copies in and
    out) -- gives the same output and rmsNorm as the same step through the
    Python API on the same inputs (same kernels: bit for bit)."""
    import ctypes
    import math
    import sys

    import numpy as np
    import torch

    import alpakann_b200 as ann
    from tests.cpp import build
    build.build()
    sys.path.insert(0, build.ROOT)
    import bench
    lib = bench.e2e_library()
    assert lib is not None
    B, H, Tk, D = 2, 4, 300, 128
    dm = H * D
    g = torch.Generator().manual_seed(3)
    hq, hk = (torch.randn((B, 1, H, D), generator=g).pin_memory() for _ in range(2))
    hh = torch.randn((B, dm), generator=g).pin_memory()
    hout = torch.empty((B, 1, H, D)).pin_memory()
    k, v = (torch.randn((B, H, Tk, D), generator=g).cuda() for _ in range(2))
    w = (1 + 0.02 * torch.randn((dm,), generator=g)).cuda()
    ang = np.arange(Tk + 1)[:, None] * np.power(1e4, -2.0 * np.arange(D // 2) / D)[None]
    cos, sin = torch.from_numpy(np.cos(ang)).float().cuda(), torch.from_numpy(np.sin(ang)).float().cuda()
    q, kn, hid, nrm, out = (torch.empty_like(t, device="cuda") for t in (hq, hk, hh, hh, hout))
    st = bench.DecodeE2E()
    st.B, st.Hl, st.H, st.Tk, st.D, st.dm = B, H, H, Tk, D, dm
    st.eps, st.scale, st.position = 1e-5, 1.0 / math.sqrt(D), Tk
    st.h_q, st.h_knew, st.h_hidden, st.h_out = hq.data_ptr(), hk.data_ptr(), hh.data_ptr(), hout.data_ptr()
    st.q, st.knew, st.hidden, st.normed = q.data_ptr(), kn.data_ptr(), hid.data_ptr(), nrm.data_ptr()
    st.norm_w, st.cos_t, st.sin_t = w.data_ptr(), cos.data_ptr(), sin.data_ptr()
    kp, vp = (ctypes.c_void_p * 1)(k.data_ptr()), (ctypes.c_void_p * 1)(v.data_ptr())
    st.k_caches, st.v_caches, st.n_caches = ctypes.cast(kp, ctypes.c_void_p), ctypes.cast(vp, ctypes.c_void_p), 1
    st.out, st.head0, st.nranks, st.rank = out.data_ptr(), 0, 1, 0
    ms = ctypes.c_float(0)
    stream = torch.cuda.current_stream()
    assert lib.decode_e2e_run(ctypes.byref(st), 1, ctypes.c_void_p(stream.cuda_stream), ctypes.byref(ms)) == 0, \
        lib.decode_e2e_error()
    torch.cuda.synchronize()
    # the same step through the Python API
    queue = ann.Queue()
    q2, kn2, n2, o2 = hq.cuda(), hk.cuda(), torch.empty((B, dm), device="cuda"), torch.empty((B, 1, H, D), device="cuda")
    ann.onHost.nn.rmsNorm(queue, None, hh.cuda(), w, n2, 1e-5)
    ann.onHost.nn.ropeInPlace(queue, None, q2, kn2, cos, sin, ann.RopeLayout.BTHD, Tk)
    ann.onHost.nn.attentionDecode(queue, None, q2, k, v, o2, 1.0 / math.sqrt(D), 1, ann.AttentionKvLayout.BHTD)
    torch.cuda.synchronize()
    assert torch.equal(hout, o2.cpu())
    assert torch.equal(nrm, n2) and torch.equal(q, q2) and torch.equal(kn, kn2)
    assert ms.value > 0
