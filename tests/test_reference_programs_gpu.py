"""The reference's own test programs, compiled unchanged, pass against this build.

`make -C oracle ref_tests` (run by `__graft_entry__.build()` where the
reference sources exist) compiles the reference's tests/*.cpp -- the page
pool, CPU reference, sparse CUDA, device page pool, continuous batching and
dense CUDA tests -- without modification against this repository's drop-in
headers (include/dsd) and libraries (libdsd_host.so over libdsd_b200.so), into
oracle/_ref/tests/.  Each program prints "... passed" on success and
"... skipped" when it sees no GPU; on a B200 every one must pass.
"""
import os
import subprocess

import pytest

from conftest import ROOT

TESTS = os.path.join(ROOT, "oracle", "_ref", "tests")
CPU_PROGRAMS = ["test_page_pool", "test_reference"]
GPU_PROGRAMS = ["test_sparse_cuda", "test_device_page_pool", "test_continuous_batching",
                "test_dense_cuda"]


def run(name):
    exe = os.path.join(TESTS, name)
    if not os.path.exists(exe):
        pytest.skip("reference test programs were not built (no reference sources here)")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout


@pytest.mark.parametrize("name", CPU_PROGRAMS)
def test_reference_cpu_program(name):
    assert "passed" in run(name)


@pytest.mark.gpu
@pytest.mark.parametrize("name", GPU_PROGRAMS)
def test_reference_gpu_program(name):
    out = run(name)
    assert "skipped" not in out, out
    assert "passed" in out, out
