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
