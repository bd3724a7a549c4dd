"""The opt-in bf16 and fp8 e4m3 page formats vs the oracle (GPU).

Such a context stores K, V and summaries rounded to nearest even in the
format (fp8 saturating) and computes in fp32.  The checker is the fp32
oracle run over what the context must store (oracle.stored_batch /
stored_round): stored values bit for bit, selected ids equal in order,
scores bit for bit, outputs <= 1e-4 max-abs.  The fp32 format stays the
default and the reference-parity path; nothing here changes it.
"""
import numpy as np
import pytest

from oracle import oracle as o
from test_continuous_gpu import run_continuous
from test_shapes_gpu import random_batch

pytestmark = pytest.mark.gpu

FORMATS = {"bf16": 1, "fp8": 2}     # DSD_KV_BF16, DSD_KV_FP8


@pytest.fixture(params=sorted(FORMATS))
def fmt(request):
    return FORMATS[request.param]


def narrow_ctx(dsd, b, fmt, top_k=None, **kw):
    k = b.top_k if top_k is None else top_k
    n = np.diff(b.cand_offsets)
    opts = dict(capacity_pages=b.capacity, max_batch=max(1, b.batch),
                max_candidates=max(1, int(n.sum())),
                max_selected=max(1, int(np.minimum(n, k).sum())), kv_format=fmt)
    opts.update(kw)
    return dsd.SparseDecodeContext(b.num_heads, b.head_dim, b.page_size, k, **opts)


def check(res, ref, tol=1e-4):
    sel, so, out, scores = o.sparse_decode(ref)
    assert np.array_equal(res["scores"].view(np.uint32), scores.view(np.uint32))
    assert np.array_equal(res["selected"], sel)
    assert float(np.abs(res["outputs"] - out).max()) <= tol


CASES = [
    ("ragged", (4, 16, 16, 3, 4, 33, 97, 7)),
    ("wide", (2, 64, 8, 4, 2, 17, 45, 17)),
    ("larger_candidates", (2, 16, 8, 8, 2, 160, 184, 123)),
    ("cfg2", (32, 128, 16, 8, 16, 512, 2048, 7)),
]


@pytest.mark.parametrize("name,cfg", CASES, ids=[c[0] for c in CASES])
def test_decode_matches_oracle_on_stored_values(dsd, fmt, name, cfg):
    b = o.synthetic_batch(*cfg)
    ref = o.stored_batch(b, o.stored_round(fmt))
    with narrow_ctx(dsd, b, fmt) as ctx:
        assert ctx.lib.dsd_ctx_kv_format(ctx.h) == fmt
        ctx.upload_pool(b.key_pool, b.value_pool, b.token_counts)
        for p in range(0, b.capacity, max(1, b.capacity // 16)):
            k, v, s, n = ctx.download_page(p)
            assert n == ref.token_counts[p]
            assert np.array_equal(k[:n].view(np.uint32), ref.key_pool[p, :n].view(np.uint32))
            assert np.array_equal(v[:n].view(np.uint32), ref.value_pool[p, :n].view(np.uint32))
            assert np.array_equal(s.view(np.uint32), ref.summaries[p].view(np.uint32)), p
        check(ctx.decode_batch(b.queries, b.cand_offsets, b.cand_ids), ref)


def test_dense_mode(dsd, fmt):
    b = o.synthetic_batch(8, 32, 16, 4, 6, 40, 300, 3)
    ref = o.stored_batch(b, o.stored_round(fmt))
    with narrow_ctx(dsd, b, fmt, max_selected=len(b.cand_ids)) as ctx:
        ctx.upload_pool(b.key_pool, b.value_pool, b.token_counts)
        ctx.set_dense(True)
        res = ctx.decode_batch(b.queries, b.cand_offsets, b.cand_ids)
        assert float(np.abs(res["outputs"] - o.dense_decode(ref)).max()) <= 1e-4


@pytest.mark.parametrize("H,D,P", [(4, 8, 16), (16, 16, 4), (64, 128, 2), (8, 64, 32), (3, 32, 1)],
                         ids=["d8", "d16", "e8192", "p32", "p1_h3"])
def test_head_and_page_shapes(dsd, fmt, H, D, P):
    if fmt == FORMATS["fp8"] and D < 16:
        pytest.skip("fp8 pages need head_dim >= 16")
    rng = np.random.default_rng(H * 1000 + D * 10 + P)
    b = random_batch(rng, H, D, P, 5, [3, 17, 40, 9])
    with narrow_ctx(dsd, b, fmt) as ctx:
        ctx.upload_pool(b.key_pool, b.value_pool, b.token_counts)
        check(ctx.decode_batch(b.queries, b.cand_offsets, b.cand_ids),
              o.stored_batch(b, o.stored_round(fmt)))


def test_rejects_small_head_dim(dsd):
    with pytest.raises(dsd.InvalidArgument):
        dsd.SparseDecodeContext(4, 4, 8, 2, 8, 1, 8, 2, kv_format=FORMATS["bf16"])
    with pytest.raises(dsd.InvalidArgument):
        dsd.SparseDecodeContext(4, 8, 8, 2, 8, 1, 8, 2, kv_format=FORMATS["fp8"])


def test_generators_round_on_store(dsd, fmt):
    E, P = 64, 8
    rnd = o.stored_round(fmt)
    summary = lambda keys: rnd(o.page_summary(rnd(keys)))
    with dsd.SparseDecodeContext(4, 16, P, 3, 16, 4, 64, 12, kv_format=fmt) as ctx:
        ctx.prefill_synthetic([5, 6, 7], [8, 8, 3], request_id=11)
        ctx.generate_normal([3, 4], [8, 5], [2, 2], [0, 8], seed=9)
        for i, (pid, n) in enumerate([(5, 8), (6, 8), (7, 3)]):
            k, v, s, cnt = ctx.download_page(pid)
            ek = o.synthetic_prompt(11, i, n, E, 1)
            assert cnt == n
            assert np.array_equal(k[:n], rnd(ek))
            assert np.array_equal(v[:n], rnd(o.synthetic_prompt(11, i, n, E, 2)))
            assert np.array_equal(s.view(np.uint32), summary(ek).view(np.uint32))
        for pid, first, n in ((3, 0, 8), (4, 8, 5)):
            k, v, s, cnt = ctx.download_page(pid)
            ek = o.normal_fill(9, 1, (2 << 40) + first * E, n * E).reshape(n, E)
            assert np.array_equal(k[:n], rnd(ek))
            assert np.array_equal(s.view(np.uint32), summary(ek).view(np.uint32))
        # synthetic decode tokens: running mean over the stored mean
        ctx.append_tokens_synthetic([7, 7], [3, 4], [11, 11], [0, 1])
        k, v, s, cnt = ctx.download_page(7)
        summ = summary(o.synthetic_prompt(11, 2, 3, E, 1))
        for off, step in ((3, 0), (4, 1)):
            key = o.synthetic_decode(11, step, E, 1)
            assert np.array_equal(k[off], rnd(key))
            summ = rnd(o.running_mean_append(summ, rnd(key), off))
        assert cnt == 5 and np.array_equal(s.view(np.uint32), summ.view(np.uint32))
        ctx.free_pages([7])
        _, _, s, _ = ctx.download_page(7)
        assert not s.any()


@pytest.mark.parametrize("split_step,depth", [(False, 1), (True, 2)],
                         ids=["sync_step", "two_steps_in_flight"])
def test_continuous_serving(dsd, fmt, split_step, depth):
    assert run_continuous(dsd, 4, 16, 8, 3, 10, 4, 6, 20, 60, 3, 10, 7, split_step, depth,
                          kv_format=fmt) > 5


def test_continuous_config4_shape(dsd, fmt):
    assert run_continuous(dsd, 32, 128, 16, 8, 12, 6, 8, 1024, 4096, 4, 10, 7,
                          kv_format=fmt) > 5


@pytest.mark.parametrize("admission", ["0", "1", "2"], ids=["cpu_cache", "direct", "synthetic"])
def test_continuous_cli_serves_the_same_tokens(admission):
    """dsd_continuous_bench with kv_format 1 or 2 (argv 26) serves the workload
    with the same token accounting as the fp32 pool, in every admission mode."""
    import os
    import subprocess
    from conftest import ROOT
    exe = os.path.join(ROOT, "15-618_dynamic_sparse_decode_b200", "bin", "dsd_continuous_bench")
    base = ["10", "4", "8", "40", "120", "3", "9", "7", "4", "16", "8", "3", admission,
            "0", "0", "0", "0", "1", "1", "0", "1", "1", "1", "0", "1"]

    def run(fmt):
        out = subprocess.run([exe, *base, fmt], capture_output=True, text=True, timeout=600)
        assert out.returncode == 0, out.stderr
        return dict(l.split("=", 1) for l in out.stdout.splitlines() if "=" in l)

    f32 = run("0")
    assert f32["kv_format"] == "fp32" and int(f32["total_generated_tokens"]) > 0
    for code, name in (("1", "bf16"), ("2", "fp8")):
        r = run(code)
        assert r["kv_format"] == name
        assert int(r["total_generated_tokens"]) == int(f32["total_generated_tokens"])
        assert float(r["continuous_sparse_tokens_per_second"]) > 0


def test_fp8_every_code_widens_exactly(dsd):
    """Every finite e4m3 code (the 126 positive and 126 negative normals and
    subnormals, and +-0) appears in the keys and values of a page set, so the
    device's widening of each code is exercised: scores must equal the
    oracle's bit for bit and outputs be within 1e-4."""
    import torch
    codes = np.array([c for c in range(256) if c & 0x7F != 0x7F], np.uint8)
    vals = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    H, D, P = 2, 16, 8
    E = H * D
    rng = np.random.default_rng(8)
    cap = 12
    flat_k = np.resize(rng.permutation(vals), cap * P * E).astype(np.float32)
    flat_v = np.resize(rng.permutation(vals), cap * P * E).astype(np.float32)
    kp = flat_k.reshape(cap, P, E)
    vp = flat_v.reshape(cap, P, E) / np.float32(64.0)   # keep the softmax outputs moderate
    tc = np.full(cap, P, np.int32)
    summ = np.stack([o.page_summary(kp[p]) for p in range(cap)])
    q = rng.standard_normal((3, E)).astype(np.float32) * np.float32(0.05)
    offs = np.array([0, 4, 9, 12], np.int32)
    ids = rng.permutation(cap).astype(np.int32)
    b = o.Batch(H, D, P, 3, kp, vp, summ, tc, q, offs, ids)
    ref = o.stored_batch(b, o.stored_round(2))
    assert np.array_equal(ref.key_pool, kp)          # every key is an exact e4m3 value
    with narrow_ctx(dsd, b, 2) as ctx:
        ctx.upload_pool(kp, vp, tc)
        check(ctx.decode_batch(q, offs, ids), ref)
