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


def _fp64_attention(q, k, v, scale, causal, kv_bhtd):
    """Every output row of q [B,Tq,H,D] against k / v ([B,H,Tk,D] when kv_bhtd,
    else [B,Tk,H,D]) recomputed in fp64 on the device, one (batch, head) at a
    time: scores, scale, (top-left causal) softmax, apply."""
    import torch
    B, Tq, H, D = q.shape
    out = torch.empty(q.shape, dtype=torch.float64, device=q.device)
    for b in range(B):
        for h in range(H):
            qh = q[b, :, h].double()
            kh = (k[b, h] if kv_bhtd else k[b, :, h]).double()
            vh = (v[b, h] if kv_bhtd else v[b, :, h]).double()
            s = (qh @ kh.T) * scale
            if causal:
                s.masked_fill_(torch.ones_like(s, dtype=torch.bool).triu(1), float("-inf"))
            out[b, :, h] = torch.softmax(s, dim=-1) @ vh
    return out


def _assert_full(got, ref, T, what):
    import torch
    rtol, atol = (1e-4, 1e-5) if T == np.float32 else (1e-11, 1e-12)
    err = (got.double() - ref).abs()
    bound = rtol * ref.abs() + atol
    worst = float((err / bound).max())
    assert worst <= 1.0, f"{what}: worst error {worst:.3f} of the tolerance, {int((err > bound).sum())} bad"
    assert bool(torch.isfinite(got).all())


@pytest.mark.parametrize("cfg", [
    dict(B=4, T=4096, H=32, D=128, T_=np.float32, name="c3"),
    dict(B=2, T=1024, H=16, D=64, T_=np.float64, name="c4"),
], ids=["c3", "c4"])
def test_prefill_full_output_vs_fp64(ann, cfg):
    """The WHOLE c3 (fp32) / c4 (fp64) prefill output, every tile edge and
    every split merge, against an fp64 recomputation on the device."""
    import torch
    B, Tt, H, D, T = cfg["B"], cfg["T"], cfg["H"], cfg["D"], cfg["T_"]
    dt = torch.float32 if T == np.float32 else torch.float64
    gen = torch.Generator(device="cuda").manual_seed(31)
    q, k, v = (torch.randn((B, Tt, H, D), generator=gen, dtype=dt, device="cuda") for _ in range(3))
    out = torch.full_like(q, float("nan"))
    scale = 1.0 / math.sqrt(D)
    queue = ann.Queue()
    ann.onHost.nn.attentionPrefill(queue, None, q, k, v, out, scale, 1, ann.AttentionKvLayout.BTHD, True)
    torch.cuda.synchronize()
    assert queue.take_device_error() == 0
    _assert_full(out, _fp64_attention(q, k, v, scale, True, False), T, cfg["name"])


def test_decode_c5_full_output_vs_fp64(ann):
    """The WHOLE c5 decode output (batch 16, cache 32768, 64 heads x 128, fp32,
    32 GiB of K+V) against an fp64 recomputation on the device."""
    import torch
    B, Tk, H, D = 16, 32768, 64, 128
    gen = torch.Generator(device="cuda").manual_seed(11)
    k = torch.randn((B, H, Tk, D), generator=gen, device="cuda")
    v = torch.randn((B, H, Tk, D), generator=gen, device="cuda")
    q = torch.randn((B, 1, H, D), generator=gen, device="cuda")
    out = torch.full_like(q, float("nan"))
    scale = 1.0 / math.sqrt(D)
    queue = ann.Queue()
    ann.onHost.nn.attentionDecode(queue, None, q, k, v, out, scale, 1, ann.AttentionKvLayout.BHTD)
    torch.cuda.synchronize()
    assert queue.take_device_error() == 0
    ref = torch.empty((B, 1, H, D), dtype=torch.float64, device="cuda")
    for b in range(B):  # one sequence at a time: its K / V in fp64 is 2 x 2 GiB
        s = torch.einsum("hd,htd->ht", q[b, 0].double(), k[b].double()) * scale
        ref[b, 0] = torch.einsum("ht,htd->hd", torch.softmax(s, -1), v[b].double())
    _assert_full(out, ref, np.float32, "c5")
    del k, v
    torch.cuda.empty_cache()
