"""ann_mlp_static_scratch, the gated MLP that allocates nothing, for callers
that cannot allocate device memory while they run. Checked through the C ABI
against the allocating ann_mlp_f32 / ann_mlp_f64 and against the oracle's
composition of the reference mlp (gemm, swiglu, gemm: onHost/nn/mlp.hpp:307-337):
two calls in a row with different inputs (a stale or shared buffer would show
in the second), each within the MLP tests' tolerance; edge shapes K = 1, F = 1
and F = 0 (an empty hidden layer gives an all-zero output); and, once a first
call has reserved the buffer, that a further call leaves the device's free
memory unchanged. The file name sorts last, so the suite runs it after every
other test; it also passes alone in a fresh process."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def capi():
    from tests.helpers import build_library
    build_library()
    from alpakann_b200 import _capi
    return _capi


@pytest.mark.parametrize("np_t,torch_t,code,tol", [
    (np.float32, torch.float32, 0, dict(rtol=1e-4, atol=1e-5)),
    (np.float64, torch.float64, 1, dict(rtol=1e-11, atol=1e-12))])
def test_static_scratch_matches_allocating_mlp(capi, np_t, torch_t, code, tol):
    sfx = "f32" if np_t == np.float32 else "f64"
    rng = np.random.default_rng(21)
    B, K, F, N = 37, 96, 200, 72  # ragged against the 64 x 64 tiles
    wg = torch.from_numpy((rng.standard_normal((K, F)) / np.sqrt(K)).astype(np_t)).cuda()
    wu = torch.from_numpy((rng.standard_normal((K, F)) / np.sqrt(K)).astype(np_t)).cuda()
    wd = torch.from_numpy((rng.standard_normal((F, N)) / np.sqrt(F)).astype(np_t)).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        x = torch.from_numpy(rng.standard_normal((B, K)).astype(np_t) * (1 + call)).cuda()
        want = torch.empty((B, N), dtype=torch_t, device="cuda")
        got = torch.full((B, N), float("nan"), dtype=torch_t, device="cuda")
        capi.check(getattr(capi.lib, f"ann_mlp_{sfx}")(stream, capi.ref(x), capi.ref(wg), capi.ref(wu),
                                                        capi.ref(wd), capi.ref(want), None, 0))
        capi.check(capi.lib.ann_mlp_static_scratch(stream, code, capi.ref(x), capi.ref(wg), capi.ref(wu),
                                                   capi.ref(wd), capi.ref(got)))
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), **tol, err_msg=f"call {call}")
        ref = oracle.gated_mlp(x.cpu().numpy(), wg.cpu().numpy(), wu.cpu().numpy(), wd.cpu().numpy())
        np.testing.assert_allclose(got.cpu().numpy(), ref, **tol, err_msg=f"call {call} vs oracle")


@pytest.mark.parametrize("B,K,F,N", [(5, 1, 7, 3), (9, 13, 1, 70), (6, 20, 0, 65), (1, 1, 1, 1)])
@pytest.mark.parametrize("np_t,code,tol", [
    (np.float32, 0, dict(rtol=1e-4, atol=1e-5)),
    (np.float64, 1, dict(rtol=1e-11, atol=1e-12))])
def test_static_scratch_edge_shapes_vs_oracle(capi, B, K, F, N, np_t, code, tol):
    """K = 1, F = 1, F = 0 (no hidden units: the output is all zeros, as the
    reference's gemm over an empty inner extent gives) against the oracle."""
    rng = np.random.default_rng(B * 1000 + K * 100 + F * 10 + N)
    x = rng.standard_normal((B, K)).astype(np_t)
    wg = rng.standard_normal((K, F)).astype(np_t)
    wu = rng.standard_normal((K, F)).astype(np_t)
    wd = rng.standard_normal((F, N)).astype(np_t)
    dev = [torch.from_numpy(a).cuda() for a in (x, wg, wu, wd)]
    got = torch.full((B, N), float("nan"), dtype=dev[0].dtype, device="cuda")
    for _ in range(2):
        capi.check(capi.lib.ann_mlp_static_scratch(None, code, *(capi.ref(d) for d in dev), capi.ref(got)))
        torch.cuda.synchronize()
        ref = oracle.gated_mlp(x, wg, wu, wd) if F > 0 else np.zeros((B, N), np_t)
        np.testing.assert_allclose(got.cpu().numpy(), ref, **tol)
    if F == 0:
        assert not got.cpu().numpy().any()


def test_static_scratch_second_call_reserves_nothing(capi):
    """The buffer is reserved when the first call loads the code on this
    device; a further call must leave the device's free memory unchanged."""
    rng = np.random.default_rng(5)
    x, wg, wu = (torch.from_numpy(rng.standard_normal(s).astype(np.float32)).cuda()
                 for s in ((64, 128), (128, 256), (128, 256)))
    wd = torch.from_numpy(rng.standard_normal((256, 96)).astype(np.float32)).cuda()
    out = torch.empty((64, 96), device="cuda")
    args = (capi.ref(x), capi.ref(wg), capi.ref(wu), capi.ref(wd), capi.ref(out))
    capi.check(capi.lib.ann_mlp_static_scratch(None, 0, *args))  # may reserve the buffer
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        capi.check(capi.lib.ann_mlp_static_scratch(None, 0, *args))
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before


def test_static_scratch_rejects_oversize(capi):
    """batch * hidden * 4 above 8 MiB: a clear error, nothing launched."""
    x = torch.zeros((1024, 8), device="cuda")
    wg = torch.zeros((8, 4096), device="cuda")
    wd = torch.zeros((4096, 8), device="cuda")
    out = torch.zeros((1024, 8), device="cuda")
    rc = capi.lib.ann_mlp_static_scratch(None, 0, capi.ref(x), capi.ref(wg), capi.ref(wg), capi.ref(wd),
                                         capi.ref(out))
    assert rc == capi.ANN_EINVAL
    assert "static scratch" in capi.lib.ann_last_error().decode()
