"""Builds and runs the C++ test programs of the drop-in API (tests/cpp)."""
import os
import subprocess

import pytest

from conftest import ROOT

PKG = os.path.join(ROOT, "15-618_dynamic_sparse_decode_b200")
CPP = os.path.join(ROOT, "tests", "cpp")


def build_and_run(name, tmp_path):
    import importlib.util
    spec = importlib.util.spec_from_file_location("_b", os.path.join(PKG, "build.py"))
    b = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b)
    if not os.path.exists(b.HOST_LIB):
        b.build()
    exe = str(tmp_path / name)
    subprocess.run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", f"-I{ROOT}/include",
                    f"-I{CPP}", "-o", exe, os.path.join(CPP, name + ".cpp"), f"-L{PKG}",
                    "-ldsd_host", "-ldsd_b200", f"-Wl,-rpath,{PKG}"], check=True)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout


def test_host_cache_cpp(tmp_path):
    assert "passed" in build_and_run("test_host_cache", tmp_path)


@pytest.mark.gpu
def test_sparse_gpu_cpp(tmp_path):
    assert "passed" in build_and_run("test_sparse_gpu", tmp_path)


@pytest.mark.gpu
def test_cli_dsd_bench_config2():
    exe = os.path.join(PKG, "bin", "dsd_bench")
    r = subprocess.run([exe, "8", "16", "512", "2048", "7", "2", "1", "32", "128", "16"],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    assert "sparse_gpu_selection_exact=1" in r.stdout
    line = [l for l in r.stdout.splitlines() if l.startswith("avg_max_abs_diff_sparse_gpu_vs_sparse_cpu")]
    assert float(line[0].split("=")[1]) <= 1e-4


@pytest.mark.gpu
def test_cli_continuous_small():
    exe = os.path.join(PKG, "bin", "dsd_continuous_bench")
    r = subprocess.run([exe, "12", "4", "8", "40", "120", "3", "9", "7", "4", "16", "8", "3"],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    kv = dict(l.split("=", 1) for l in r.stdout.splitlines() if "=" in l)
    assert int(kv["total_generated_tokens"]) > 0
    assert float(kv["continuous_sparse_tokens_per_second"]) > 0
    assert float(kv["continuous_vs_serial_speedup"]) > 0


@pytest.mark.gpu
def test_cli_continuous_dense_mode():
    exe = os.path.join(PKG, "bin", "dsd_continuous_bench")
    r = subprocess.run([exe, "8", "4", "8", "40", "120", "3", "9", "7", "4", "16", "8", "3", "1",
                        "0", "0", "0", "0", "1", "1", "1"], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr
    kv = dict(l.split("=", 1) for l in r.stdout.splitlines() if "=" in l)
    assert kv["continuous_dense_gpu_available"] == "1"
    assert float(kv["continuous_dense_gpu_tokens_per_second"]) > 0
