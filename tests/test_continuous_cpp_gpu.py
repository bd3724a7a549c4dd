"""The C++ serving loop (RunContinuousSparseDecode, the dsd_continuous_bench
path) checked step by step against the oracle (GPU).

tests/cpp/trace_continuous.cpp runs the loop with a step observer and writes
every step: the batch in launch order (request id, context tokens, page list,
the query the host handed over) and the step's result (selected ids, scores,
outputs).  This test replays the trace on the host: it regenerates each
request's prompt and decode tokens from the reference's generators (restated
in the oracle), rebuilds the content of every page the step can read from
(prompt pages, then decode pages opened by the first decoded token, summaries
by the reference's formulas), checks the query against the one the reference
loop would use, and decodes the step with the oracle: selected ids equal in
order, scores bit for bit, outputs <= 1e-4.  This covers what the Python-driven
continuous tests do not: the C++ loop's admission options, worker-pool query
packing and page bookkeeping at batch 32-64.
"""
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT
from oracle import oracle as o

pytestmark = pytest.mark.gpu

PKG = os.path.join(ROOT, "15-618_dynamic_sparse_decode_b200")


@pytest.fixture(scope="module")
def trace_exe(tmp_path_factory):
    exe = str(tmp_path_factory.mktemp("trace") / "trace_continuous")
    subprocess.run(["g++", "-O2", "-std=c++17", f"-I{ROOT}/include", "-o", exe,
                    os.path.join(ROOT, "tests", "cpp", "trace_continuous.cpp"), f"-L{PKG}",
                    "-ldsd_host", "-ldsd_b200", f"-Wl,-rpath,{PKG}"], check=True)
    return exe


def read_trace(path, E):
    raw = np.fromfile(path, np.uint8)
    pos = 0

    def ints(n):
        nonlocal pos
        v = raw[pos:pos + 4 * n].view(np.int32)
        pos += 4 * n
        return v

    def floats(n):
        nonlocal pos
        v = raw[pos:pos + 4 * n].view(np.float32)
        pos += 4 * n
        return v

    steps = []
    while True:
        b = int(ints(1)[0])
        if b < 0:
            break
        reqs = []
        for _ in range(b):
            rid, ctx_tok, n = (int(x) for x in ints(3))
            pages = ints(n).copy()
            q = floats(E).copy()
            ns = int(ints(1)[0])
            sel = ints(ns).copy()
            sc = floats(n).copy()
            out = floats(E).copy()
            reqs.append(dict(rid=rid, ctx=ctx_tok, pages=pages, query=q, sel=sel, scores=sc,
                             out=out))
        steps.append(reqs)
    generated = int(ints(1)[0])
    assert pos == raw.size
    return steps, generated


def replay(steps, w, H, D, P, K, synthetic_prefill, gpu_append, kv_format):
    """Checks every traced step against the oracle; returns the steps checked."""
    E = H * D
    rnd = o.stored_round(kv_format)
    index = {int(r): i for i, r in enumerate(w["request_ids"])}
    pt = w["prompt_tokens"]
    offs = np.concatenate([[0], np.cumsum(pt)])
    cap = 1 + max(int(r["pages"].max()) for s in steps for r in s if r["pages"].size)
    kp = np.zeros((cap, P, E), np.float32)
    vp = np.zeros((cap, P, E), np.float32)
    summ = np.zeros((cap, E), np.float32)
    tc = np.zeros(cap, np.int32)
    owner = [None] * cap        # (request, kind, index) whose content the slot holds

    def decode_token(rid, t, stream):
        return (o.synthetic_decode(rid, t, E, stream) if gpu_append
                else o.deterministic_token_vector(E, rid, t, stream))

    for si, reqs in enumerate(steps):
        queries, cand = [], []
        for r in reqs:
            rid, i = r["rid"], index[r["rid"]]
            n_prompt = int(pt[i])
            d = r["ctx"] - n_prompt                      # tokens decoded before this step
            n_pp = (n_prompt + P - 1) // P
            pages = r["pages"]
            assert len(pages) == n_pp + (d + P - 1) // P, (si, rid, "page count")
            for j in range(n_pp):
                pid = int(pages[j])
                if owner[pid] == (rid, "p", j):
                    continue
                n = min(P, n_prompt - j * P)
                if synthetic_prefill:
                    k = o.synthetic_prompt(rid, j, n, E, 1)
                    v = o.synthetic_prompt(rid, j, n, E, 2)
                else:
                    k = w["prompt_keys"][offs[i] + j * P: offs[i] + j * P + n]
                    v = w["prompt_values"][offs[i] + j * P: offs[i] + j * P + n]
                kp[pid, :n], vp[pid, :n] = rnd(k), rnd(v)
                summ[pid] = rnd(o.page_summary(kp[pid, :n]))
                tc[pid] = n
                owner[pid] = (rid, "p", j)
            for m, pid in enumerate(pages[n_pp:]):
                pid = int(pid)
                want = min(P, d - m * P)
                if owner[pid] != (rid, "d", m):
                    owner[pid] = (rid, "d", m)
                    tc[pid] = 0
                    summ[pid] = 0
                while tc[pid] < want:
                    t = m * P + int(tc[pid])
                    key = rnd(decode_token(rid, t, 1))
                    kp[pid, tc[pid]] = key
                    vp[pid, tc[pid]] = rnd(decode_token(rid, t, 2))
                    summ[pid] = rnd(o.running_mean_append(summ[pid], key, int(tc[pid])))
                    tc[pid] += 1
            q = (w["initial_queries"][i] if d == 0
                 else o.deterministic_token_vector(E, rid, d, 0))
            assert np.array_equal(r["query"].view(np.uint32), q.view(np.uint32)), (si, rid)
            queries.append(q)
            cand.append(pages)
        b = o.Batch(H, D, P, K, kp, vp, summ, tc, np.stack(queries),
                    np.concatenate([[0], np.cumsum([len(c) for c in cand])]).astype(np.int32),
                    np.concatenate(cand).astype(np.int32))
        sel, so, out, scores = o.sparse_decode(b)
        for j, r in enumerate(reqs):
            c0, c1 = int(b.cand_offsets[j]), int(b.cand_offsets[j + 1])
            assert np.array_equal(r["scores"].view(np.uint32), scores[c0:c1].view(np.uint32)), \
                (si, r["rid"], "scores")
            assert np.array_equal(r["sel"], sel[so[j]:so[j + 1]]), (si, r["rid"], "selected")
            diff = float(np.abs(r["out"] - out[j]).max())
            assert diff <= 1e-4, (si, r["rid"], diff)
    return len(steps)


def run(trace_exe, tmp_path, n, max_active, window, pmin, pmax, dmin, dmax, seed, H, D, P, K,
        admission, preadmit, precompute, gpu_append, lazy, kv_format=0):
    path = str(tmp_path / "trace.bin")
    argv = [n, max_active, window, pmin, pmax, dmin, dmax, seed, H, D, P, K, admission,
            preadmit, precompute, gpu_append, lazy, kv_format]
    r = subprocess.run([trace_exe, path, *map(str, argv)], capture_output=True, text=True,
                       timeout=1200)
    assert r.returncode == 0, r.stdout + r.stderr
    steps, generated = read_trace(path, H * D)
    synthetic = admission == 2
    if synthetic:
        w = host_specs_without_payloads(H, D, n, window, pmin, pmax, dmin, dmax, seed)
    else:
        w = o.continuous_workload(H, D, n, window, pmin, pmax, dmin, dmax, seed)
    assert generated == int(w["decode_steps"].sum())
    assert sum(len(s) for s in steps) == generated
    return replay(steps, w, H, D, P, K, synthetic, bool(gpu_append), kv_format)


def host_specs_without_payloads(H, D, n, window, pmin, pmax, dmin, dmax, seed):
    """BuildSyntheticContinuousSpecs: mt19937(seed), per request arrival,
    prompt and decode lengths only, sorted by (arrival, id); the initial query
    from mt19937(MixSeed(r, 0, 0)) (tests/test_workload_pin.py pins both)."""
    spec = o.continuous_specs_only(n, window, pmin, pmax, dmin, dmax, seed)
    spec["initial_queries"] = np.stack([o.deterministic_token_vector(H * D, int(r), 0, 0)
                                        for r in spec["request_ids"]])
    return spec


def test_cpp_loop_config4_published_options(trace_exe, tmp_path):
    """Config 4's shape and the options of the reference's published run:
    direct GPU upload of the generator's payloads, preadmitted prompts,
    precomputed decode payloads, GPU synthetic append, lazy release; 64
    requests at most 32 active, shorter prompts so the replay stays small."""
    assert run(trace_exe, tmp_path, 64, 32, 16, 256, 1024, 8, 40, 7, 32, 128, 16, 8,
               1, 1, 1, 1, 1) > 30


def test_cpp_loop_config4_runtime_admission(trace_exe, tmp_path):
    """The reference CLI's default options: runtime admission by direct
    upload, host-generated decode tokens appended through the pool."""
    assert run(trace_exe, tmp_path, 48, 32, 16, 256, 1024, 8, 32, 7, 32, 128, 16, 8,
               1, 0, 0, 0, 0) > 30


@pytest.mark.parametrize("kv_format", [0, 1], ids=["f32", "bf16"])
def test_cpp_loop_config5_modes(trace_exe, tmp_path, kv_format):
    """Config 5's modes: synthetic GPU prefill, GPU synthetic append, P32 k32,
    at most 64 active of 96 requests, shorter prompts."""
    assert run(trace_exe, tmp_path, 96, 64, 16, 256, 1536, 8, 24, 11, 32, 128, 32, 32,
               2, 0, 0, 1, 0, kv_format) > 20
