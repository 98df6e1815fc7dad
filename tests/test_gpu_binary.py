"""loadBinaryTensor on the GPU (onHost/core/binary.hpp:234-323): payload
bytes land on the device bit for bit, across staging chunks, for whole
tensors and for per-rank boxes of a row-major weight. The oracle is the file
itself, read with numpy."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def core():
    from tests.helpers import build_library
    build_library()
    from alpakann_b200.onHost import core
    return core


def make_file(tmp_path, name, prefix_bytes, arr):
    p = tmp_path / name
    with open(p, "wb") as f:
        f.write(b"\xab" * prefix_bytes)
        f.write(arr.tobytes())
    return str(p)


@pytest.mark.parametrize("dtype,np_t", [(torch.float32, np.float32), (torch.float64, np.float64)])
def test_roundtrip_reference_case(core, tmp_path, dtype, np_t):
    # test/unit/core/binary.cpp:70-102: 6 values behind a 64-byte poison prefix
    values = (np.arange(6, dtype=np_t) * np_t(0.5) - np_t(1.25))
    path = make_file(tmp_path, "rt.bin", 64, values)
    spec = core.TensorSpec("t", 64, 6, (2, 3))
    sha = core.sha256File(path)
    t = core.loadBinaryTensor(None, path, spec, sha, dtype=dtype)
    torch.cuda.synchronize()
    assert t.shape == (6,) and t.dtype == dtype
    assert np.array_equal(t.cpu().numpy(), values)


def test_multichunk_on_side_stream(core, tmp_path):
    """40 MiB + 3 floats (three staging chunks, a ragged last one) at a
    non-zero offset, loaded on a side stream; then a second load right away,
    which must wait for the first one's staging buffers."""
    rng = np.random.default_rng(11)
    n = (40 << 20) // 4 + 3
    a = rng.standard_normal(n).astype(np.float32)
    b = rng.standard_normal(1 << 20).astype(np.float32)
    path = make_file(tmp_path, "mc.bin", 128, np.concatenate([a, np.zeros(13, np.float32), b]))
    off_b = 128 + (n + 13) * 4
    assert off_b % 64 == 0
    s = torch.cuda.Stream()
    ta = core.loadBinaryTensor(s, path, core.TensorSpec("a", 128, n))
    tb = core.loadBinaryTensor(s, path, core.TensorSpec("b", off_b, b.size, (1024, 1024)))
    s.synchronize()
    assert np.array_equal(ta.cpu().numpy(), a)
    assert np.array_equal(tb.cpu().numpy(), b)


@pytest.mark.parametrize("rows,cols", [((0, 4096), (1000, 1000)),     # column shard, two row chunks
                                       ((1024, 1024), (0, 3000)),     # row shard: contiguous run
                                       ((7, 13), (2999, 1)),          # one column
                                       ((0, 4096), (0, 3000))])       # everything
def test_box_matches_numpy_slice(core, tmp_path, rows, cols):
    rng = np.random.default_rng(3)
    w = rng.standard_normal((4096, 3000))
    path = make_file(tmp_path, "w.bin", 64, w)
    spec = core.TensorSpec("w", 64, w.size, w.shape)
    t = core.loadBinaryTensorBox(None, path, spec, rows, cols, dtype=torch.float64)
    torch.cuda.synchronize()
    r0, nr = rows
    c0, nc = cols
    assert np.array_equal(t.cpu().numpy(), w[r0:r0 + nr, c0:c0 + nc])


def test_box_into_pitched_destination(core, tmp_path):
    """Through the C ABI: rows land out_row_pitch_bytes apart; the padding
    between them is left untouched."""
    from alpakann_b200 import _capi
    rng = np.random.default_rng(5)
    w = rng.standard_normal((300, 512)).astype(np.float32)
    path = make_file(tmp_path, "p.bin", 0, w)
    s, keep = core._spec(core.TensorSpec("w", 0, w.size, w.shape))
    dst = torch.full((100, 80), -7.0, device="cuda")
    rc = _capi.lib.ann_load_binary_tensor_box(torch.cuda.current_stream().cuda_stream, path.encode(),
                                              ctypes.byref(s), 4, b"", 100, 100, 256, 64, dst.data_ptr(), 80 * 4)
    assert rc == 0, _capi.lib.ann_last_error()
    got = dst.cpu().numpy()
    assert np.array_equal(got[:, :64], w[100:200, 256:320])
    assert np.all(got[:, 64:] == -7.0)


def test_sharded_weights_reassemble(core, tmp_path):
    """Four column-parallel shards of one [in, out] weight, as four ranks
    would load them, concatenate to the whole weight."""
    rng = np.random.default_rng(9)
    w = rng.standard_normal((256, 512)).astype(np.float32)
    path = make_file(tmp_path, "wq.bin", 64, w)
    spec = core.TensorSpec("Wq", 64, w.size, w.shape)
    sha = core.sha256File(path)
    parts = [core.loadBinaryTensorBox(None, path, spec, (0, 256), (r * 128, 128), sha) for r in range(4)]
    whole = core.loadBinaryTensor(None, path, spec, sha)
    torch.cuda.synchronize()
    assert torch.equal(torch.cat(parts, dim=1), whole.view(256, 512))
    assert np.array_equal(whole.cpu().numpy().reshape(256, 512), w)
