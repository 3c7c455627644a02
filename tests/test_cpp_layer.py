"""The C++20 drop-in layer (cppinf_b200/cpp: cppinf::tensors / cppinf::ops / cppinf::nn with device storage) through
its own test binary, whose cases follow the reference's tests/ops/ops_test.cpp, tests/nn/rope_test.cpp and
tests/tensors/tensor_test.cpp. Host-only cases (metadata, views, validation) run without a GPU."""

from __future__ import annotations

import subprocess
from pathlib import Path

import pytest

PACKAGE = Path(__file__).resolve().parent.parent / "cppinf_b200"
BINARY = PACKAGE / "_lib" / "cppinf_ops_tests"


def _run(*args: str) -> subprocess.CompletedProcess:
    # The binary is a build output (not in the repository): make brings it up to date with its sources first.
    build = subprocess.run(["make", "-C", str(PACKAGE), "_lib/cppinf_ops_tests"], capture_output=True, text=True,
                           timeout=900)
    assert build.returncode == 0 and BINARY.exists(), f"building {BINARY} failed:\n{build.stdout}{build.stderr}"
    return subprocess.run([str(BINARY), *args], capture_output=True, text=True, timeout=600)


def test_cpp_drop_in_host_only_cases():
    proc = _run("--host-only")
    assert proc.returncode == 0, proc.stdout + proc.stderr
    assert " 0 failed" in proc.stdout


@pytest.mark.gpu
def test_cpp_drop_in_all_cases_on_gpu(cuda):
    proc = _run()
    assert proc.returncode == 0, proc.stdout + proc.stderr
    assert "FAILED" not in proc.stdout
