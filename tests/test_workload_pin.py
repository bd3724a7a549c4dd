"""The continuous workload generator is pinned to the reference (CPU only).

Every config-4/5 input -- request arrivals, prompt and decode lengths, prompt
payloads, initial queries and per-step tokens -- comes from the reference's
BuildSyntheticContinuousWorkload (src/continuous_batching.cpp:336-381) and
DeterministicTokenVector (:44-59).  This file checks both restatements -- the
oracle's (oracle/dsd_oracle.cpp) and this build's C++ API
(csrc/host/continuous_batching.cpp, through tests/cpp/dump_workload.cpp) --
against fixtures the reference's own code produced
(tests/golden/continuous_workload.npz, made by tests/golden/make_golden.py),
and against the reference library itself where oracle/_ref was built.
"""
import hashlib
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT
from oracle import oracle as o

G = np.load(os.path.join(ROOT, "tests", "golden", "continuous_workload.npz"))
SPEC_FIELDS = ["request_ids", "arrival_steps", "prompt_tokens", "decode_steps"]
PAYLOAD_FIELDS = ["prompt_keys", "prompt_values", "initial_queries"]
FULL_CASES = ["cont_small", "cont_mid"]
PKG = os.path.join(ROOT, "15-618_dynamic_sparse_decode_b200")


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def check_against_golden(name, w, payloads=True):
    for f in SPEC_FIELDS:
        assert np.array_equal(w[f], G[f"{name}_{f}"]), f"{name}: {f} differs"
    if payloads:
        for f in PAYLOAD_FIELDS:
            assert sha(w[f]) == str(G[f"{name}_sha256_{f}"]), f"{name}: {f} differs"


@pytest.mark.parametrize("name", FULL_CASES)
def test_oracle_workload_matches_reference_golden(name):
    cfg = [int(x) for x in G[f"{name}_config"]]
    check_against_golden(name, o.continuous_workload(*cfg, with_payloads=True))


def test_oracle_config4_specs_match_reference_golden():
    """BASELINE config 4's arrivals and lengths (the payload draws are made and
    discarded, so the stream stays aligned)."""
    cfg = [int(x) for x in G["cont_cfg4_config"]]
    check_against_golden("cont_cfg4", o.continuous_workload(*cfg, with_payloads=False),
                         payloads=False)


def test_oracle_token_vectors_match_reference_golden():
    for case, want in zip(G["tokens_cases"], G["tokens_sha256"]):
        assert sha(o.deterministic_token_vector(*[int(x) for x in case])) == str(want), case


@pytest.fixture(scope="module")
def dump_exe(tmp_path_factory):
    import importlib.util
    spec = importlib.util.spec_from_file_location("_b", os.path.join(PKG, "build.py"))
    b = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b)
    if not os.path.exists(b.HOST_LIB):
        b.build()
    exe = str(tmp_path_factory.mktemp("dump") / "dump_workload")
    subprocess.run(["g++", "-O2", "-std=c++17", f"-I{ROOT}/include", "-o", exe,
                    os.path.join(ROOT, "tests", "cpp", "dump_workload.cpp"), f"-L{PKG}",
                    "-ldsd_host", "-ldsd_b200", f"-Wl,-rpath,{PKG}"], check=True)
    return exe


def host_workload(exe, tmp_path, cfg, mode="specs"):
    out = str(tmp_path / "w.bin")
    subprocess.run([exe, mode, *map(str, cfg), out], check=True)
    raw = np.fromfile(out, np.uint8)
    n, e = cfg[2], cfg[0] * cfg[1]
    ints = raw[: 16 * n].view(np.int32).reshape(4, n)
    w = dict(zip(SPEC_FIELDS, ints))
    floats = raw[16 * n:].view(np.float32)
    t = int(w["prompt_tokens"].sum()) if mode == "specs" else 0
    w["prompt_keys"] = floats[: t * e].reshape(t, e)
    w["prompt_values"] = floats[t * e: 2 * t * e].reshape(t, e)
    w["initial_queries"] = floats[2 * t * e:].reshape(n, e)
    return w


@pytest.mark.parametrize("name", FULL_CASES)
def test_cpp_api_workload_matches_reference_golden(dump_exe, tmp_path, name):
    cfg = [int(x) for x in G[f"{name}_config"]]
    check_against_golden(name, host_workload(dump_exe, tmp_path, cfg))


def test_cpp_api_token_vectors_match_reference_golden(dump_exe, tmp_path):
    out = str(tmp_path / "t.bin")
    for case, want in zip(G["tokens_cases"], G["tokens_sha256"]):
        subprocess.run([dump_exe, "tokens", *[str(int(x)) for x in case], out], check=True)
        assert sha(np.fromfile(out, np.float32)) == str(want), case


@pytest.mark.skipif(not o.ref_available(), reason="reference sources were not built here")
@pytest.mark.parametrize("cfg", [(2, 4, 33, 0, 0, 5, 0, 3, 1), (8, 2, 17, 40, 1, 30, 5, 9, 99),
                                 (1, 16, 64, 7, 2, 11, 1, 1, 2024)])
def test_oracle_workload_matches_reference_library(cfg):
    """Extra shapes straight against the reference (zero-length prompts and
    decodes, an empty arrival window, many arrival ties)."""
    a = o.continuous_workload(*cfg, with_payloads=True)
    b = o.ref_continuous_workload(*cfg, with_payloads=True)
    for f in SPEC_FIELDS + PAYLOAD_FIELDS:
        assert np.array_equal(a[f].view(np.uint8), b[f].view(np.uint8)), f
    for t in [(64, 0, 0, 0), (100, 9, 3, 2), (4096, 2047, 300, 1)]:
        assert np.array_equal(o.deterministic_token_vector(*t).view(np.uint32),
                              o.ref_deterministic_token_vector(*t).view(np.uint32))


@pytest.mark.parametrize("cfg", [(32, 128, 96, 16, 256, 1536, 8, 24, 11),
                                 (2, 4, 50, 0, 0, 7, 0, 3, 5)])
def test_cpp_specs_without_payloads_match_oracle(dump_exe, tmp_path, cfg):
    """This build's lengths-only generator (config 5's specs; no reference
    counterpart) against the oracle's restatement, initial queries included."""
    w = host_workload(dump_exe, tmp_path, cfg, mode="specs_only")
    s = o.continuous_specs_only(*cfg[2:])
    for f in SPEC_FIELDS:
        assert np.array_equal(w[f], s[f]), f
    assert w["prompt_keys"].size == 0 and w["prompt_values"].size == 0
    e = cfg[0] * cfg[1]
    for i, r in enumerate(s["request_ids"]):
        q = o.deterministic_token_vector(e, int(r), 0, 0)
        assert np.array_equal(w["initial_queries"][i].view(np.uint32), q.view(np.uint32))
