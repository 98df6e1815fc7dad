"""Full-size decode configurations on one GPU, checked on sampled rows
against the oracle pipeline and through size-independent properties."""
import math

import numpy as np
import pytest

import oracle
from tests.helpers import assert_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ann():
    import alpakann_b200
    return alpakann_b200


def _sample_check(q, k, v, out, rows, scale, g, T):
    """Oracle pipeline on the sampled rows only, from host copies of the
    heads those rows read."""
    for b, t, h in rows:
        kvh = h // g
        qh = q[b:b + 1, t:t + 1, h:h + 1].cpu().numpy()
        kh = k[b:b + 1, kvh:kvh + 1].cpu().numpy()
        vh = v[b:b + 1, kvh:kvh + 1].cpu().numpy()
        ref = oracle.attention_rows(qh, kh, vh, np.array([[0, 0, 0]], np.int64), T(scale), 1, 1, False)[0]
        assert_close(out[b, t, h].cpu().numpy(), ref, T, f"row {(b, t, h)}")


@pytest.mark.parametrize("cfg", [
    # c5 on one GPU: batch 16, cache 32768, 64 heads x 128, fp32 (32 GiB of K+V)
    dict(B=16, Tk=32768, H=64, D=128, T=np.float32, seed=5),
    # c2 again at full size with the KV cache generated on the device
    dict(B=8, Tk=2048, H=32, D=128, T=np.float32, seed=2),
], ids=["c5_1gpu", "c2"])
def test_decode_full_size(ann, cfg):
    import torch
    B, Tk, H, D, T = cfg["B"], cfg["Tk"], cfg["H"], cfg["D"], cfg["T"]
    dt = torch.float32 if T == np.float32 else torch.float64
    gen = torch.Generator(device="cuda").manual_seed(cfg["seed"])
    k = torch.randn((B, H, Tk, D), generator=gen, dtype=dt, device="cuda")
    v = torch.randn((B, H, Tk, D), generator=gen, dtype=dt, device="cuda")
    q = torch.randn((B, 1, H, D), generator=gen, dtype=dt, device="cuda")
    out = torch.full((B, 1, H, D), float("nan"), dtype=dt, device="cuda")
    scale = 1.0 / math.sqrt(D)
    queue = ann.Queue()
    ann.onHost.nn.attentionDecode(queue, None, q, k, v, out, scale, 1, ann.AttentionKvLayout.BHTD)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    rng = np.random.default_rng(cfg["seed"])
    rows = [(int(rng.integers(B)), 0, int(rng.integers(H))) for _ in range(6)] + [(0, 0, 0), (B - 1, 0, H - 1)]
    _sample_check(q, k, v, out, rows, scale, 1, T)
    # property: the output is a convex combination of V rows -> within [min V, max V] per dim
    vmin = v.amin(dim=2).unsqueeze(1)
    vmax = v.amax(dim=2).unsqueeze(1)
    assert bool(((out >= vmin - 1e-5) & (out <= vmax + 1e-5)).all())
    # property: a constant V gives that constant back exactly up to rounding
    v.fill_(0.5)
    ann.onHost.nn.attentionDecode(queue, None, q, k, v, out, scale, 1, ann.AttentionKvLayout.BHTD)
    torch.cuda.synchronize()
    assert float((out - 0.5).abs().max()) < 1e-5
    assert queue.take_device_error() == 0
    del k, v
    torch.cuda.empty_cache()
