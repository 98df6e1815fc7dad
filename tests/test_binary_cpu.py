"""Model-artifact loader checks that need no GPU (onHost/core/binary.hpp).

sha256File against the known vectors of the reference's test
(test/unit/core/binary.cpp:139-159) and against hashlib on every length
around the 64-byte block and padding edges, on both compression paths (x86
SHA extensions and the scalar recurrence). Then every layout the reference's
loader rejects (test/unit/core/binary.cpp:182-235): each raises before
anything touches a device, so no GPU is needed.
"""
import hashlib
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def core():
    from tests.helpers import build_library
    build_library()
    from alpakann_b200.onHost import core
    return core


def write(tmp_path, name, data: bytes):
    p = tmp_path / name
    p.write_bytes(data)
    return str(p)


def test_sha256_known_vectors(core, tmp_path):
    # test/unit/core/binary.cpp:143-152
    assert core.sha256File(write(tmp_path, "e.bin", b"")) == \
        "e3b0c44298fc1c149afbf4c8996fb92427ae41e4649b934ca495991b7852b855"
    assert core.sha256File(write(tmp_path, "abc.bin", b"abc")) == \
        "ba7816bf8f01cfea414140de5dae2223b00361a396177a9cb410ff61f20015ad"
    # :154-159, 1000 bytes i & 0xff; the reference only checks the length
    long = bytes(i & 0xFF for i in range(1000))
    got = core.sha256File(write(tmp_path, "long.bin", long))
    assert len(got) == 64 and got == hashlib.sha256(long).hexdigest()


def test_sha256_block_edges_match_hashlib(core):
    rng = np.random.default_rng(0x5EED)
    data = rng.integers(0, 256, 4096, dtype=np.uint8).tobytes()
    for n in list(range(0, 200)) + [447, 448, 511, 512, 513, 1023, 1024, 4095, 4096]:
        assert core.sha256Bytes(data[:n]) == hashlib.sha256(data[:n]).hexdigest(), n


def test_sha256_large_file_chunks(core, tmp_path):
    # crosses the 4 MiB read chunks of the file hash at an odd length
    rng = np.random.default_rng(7)
    data = rng.integers(0, 256, (9 << 20) + 37, dtype=np.uint8).tobytes()
    assert core.sha256File(write(tmp_path, "big.bin", data)) == hashlib.sha256(data).hexdigest()


def test_sha256_scalar_path_matches(tmp_path):
    """ANN_SHA256_SCALAR=1 forces the scalar recurrence (read once per
    process, hence the child process)."""
    data = bytes((i * 131 + 7) & 0xFF for i in range(100_003))
    p = write(tmp_path, "s.bin", data)
    code = ("import sys; sys.path.insert(0, %r); from alpakann_b200.onHost import core; "
            "print(core.sha256File(%r))" % (ROOT, p))
    for env in ("1", "0"):
        out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, check=True,
                             env={**os.environ, "ANN_SHA256_SCALAR": env}).stdout.strip()
        assert out == hashlib.sha256(data).hexdigest(), env


def test_sha256_missing_file(core, tmp_path):
    from alpakann_b200._capi import AnnIOError
    with pytest.raises(AnnIOError, match="sha256File: cannot open"):
        core.sha256File(str(tmp_path / "nope.bin"))
    with pytest.raises(RuntimeError):
        core.sha256File(str(tmp_path))  # a directory cannot be read


@pytest.fixture()
def payload(tmp_path):
    # test/unit/core/binary.cpp:193-197: 16 floats of 1.0
    return write(tmp_path, "reject.bin", np.ones(16, np.float32).tobytes())


def spec(core, offset, count, shape=()):
    return core.TensorSpec("spec", offset, count, tuple(shape))


def test_rejects_unaligned_offset(core, payload):
    with pytest.raises(ValueError, match="is not 64-byte aligned"):
        core.loadBinaryTensor(None, payload, spec(core, 8, 4))


def test_rejects_shape_product(core, payload):
    with pytest.raises(ValueError, match="shape product 8 of tensor 'spec' does not match count 6"):
        core.loadBinaryTensor(None, payload, spec(core, 0, 6, (2, 4)))


def test_rejects_truncated(core, payload):
    with pytest.raises(ValueError, match="exceeds file size 64"):
        core.loadBinaryTensor(None, payload, spec(core, 0, 1000))


def test_rejects_byte_overflow(core, payload):
    huge = (2 ** 64 - 1) // 4 + 1
    with pytest.raises(ValueError, match="overflows"):
        core.loadBinaryTensor(None, payload, spec(core, 0, huge))


def test_rejects_shape_overflow(core, payload):
    with pytest.raises(ValueError, match="overflows"):
        core.loadBinaryTensor(None, payload, spec(core, 0, 4, (2 ** 40, 2 ** 40)))


def test_rejects_zero_elements(core, payload):
    with pytest.raises(ValueError, match="has zero elements"):
        core.loadBinaryTensor(None, payload, spec(core, 0, 0))


def test_rejects_corrupt_sha(core, payload):
    from alpakann_b200._capi import AnnIOError
    with pytest.raises(AnnIOError, match="SHA-256 mismatch"):
        core.loadBinaryTensor(None, payload, spec(core, 0, 4), "0" * 64)


def test_rejects_missing_file(core, tmp_path):
    from alpakann_b200._capi import AnnIOError
    with pytest.raises(AnnIOError, match="cannot stat"):
        core.loadBinaryTensor(None, str(tmp_path / "alpakann_does_not_exist.bin"), spec(core, 0, 4))


def test_rejects_non_float_types(core, payload):
    import torch
    with pytest.raises(TypeError):
        core.loadBinaryTensor(None, payload, spec(core, 0, 4), dtype=torch.int32)


def test_check_order_matches_reference(core, tmp_path):
    """Zero count is reported before a missing file, a missing file before an
    unaligned offset (binary.hpp:263-296)."""
    from alpakann_b200._capi import AnnIOError
    missing = str(tmp_path / "missing.bin")
    with pytest.raises(ValueError, match="zero elements"):
        core.loadBinaryTensor(None, missing, spec(core, 8, 0))
    with pytest.raises(AnnIOError):
        core.loadBinaryTensor(None, missing, spec(core, 8, 4))


def test_sha_is_case_insensitive_and_validation_only_call(core, tmp_path):
    """A matching digest in upper case passes every check; with no device
    buffer the C ABI stops after the checks (validation-only call)."""
    import ctypes
    from alpakann_b200 import _capi
    data = np.arange(32, dtype=np.float32).tobytes()
    p = write(tmp_path, "ok.bin", data)
    s, keep = core._spec(spec(core, 64, 16, (4, 4)))
    sha = hashlib.sha256(data).hexdigest().upper().encode()
    assert _capi.lib.ann_load_binary_tensor(None, p.encode(), ctypes.byref(s), 4, sha, None) == 0
    assert _capi.lib.ann_load_binary_tensor_box(None, p.encode(), ctypes.byref(s), 4, sha, 1, 2, 1, 3, None, 12) == 0


@pytest.mark.parametrize("rows,cols,pitch,msg", [
    ((3, 2), (0, 4), 16, "outside"), ((0, 4), (2, 3), 12, "outside"), ((0, 0), (0, 4), 16, "outside"),
    ((-1, 2), (0, 4), 16, "outside"), ((0, 2), (0, 4), 12, "row pitch"), ((0, 2), (0, 4), 18, "row pitch")])
def test_box_rejects(core, tmp_path, rows, cols, pitch, msg):
    import ctypes
    from alpakann_b200 import _capi
    p = write(tmp_path, "box.bin", np.zeros(16, np.float32).tobytes())
    s, keep = core._spec(spec(core, 0, 16, (4, 4)))
    rc = _capi.lib.ann_load_binary_tensor_box(None, p.encode(), ctypes.byref(s), 4, b"", rows[0], rows[1], cols[0],
                                              cols[1], None, pitch)
    assert rc == _capi.ANN_EINVAL and msg in _capi.lib.ann_last_error().decode()


def test_box_needs_shape(core, tmp_path):
    p = write(tmp_path, "box.bin", np.zeros(16, np.float32).tobytes())
    with pytest.raises(ValueError, match="needs the tensor's shape"):
        core.loadBinaryTensorBox(None, p, spec(core, 0, 16), (0, 1), (0, 1))
