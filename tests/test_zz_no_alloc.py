"""ann_mlp_static_scratch, the gated MLP that allocates nothing, against the
allocating ann_mlp_f32 / ann_mlp_f64 through the C ABI: two calls in a row
with different inputs (a stale or shared buffer would show in the second),
each within the MLP tests' tolerance of the existing entry point. The file
name sorts last, so the suite runs it after every other test; it also passes
alone in a fresh process."""
import numpy as np
import pytest
import torch

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
