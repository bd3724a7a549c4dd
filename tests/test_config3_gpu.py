"""BASELINE config 3 at full size on one GPU (64 requests, 16k-32k context, k=64).

The whole batch runs on the device.  With fp32 pages (the reference's
format) EVERY one of the 64 requests is re-generated on the host with the
oracle's restatement of the workload generator and decoded by the oracle:
ids equal in order, scores bit for bit, outputs <= 1e-4.  The bf16- and
fp8-page contexts run the same check, against the oracle over the rounded
values, on 8 requests: both sides of the production step's two-range split
(31, 32), the first and last request and four spread between.
Size-independent properties cover every request in every format: each
selects exactly min(k, n) distinct pages of its own, in (score desc, id asc)
order of the device's scores.
"""
import numpy as np
import pytest

import bench
from oracle import oracle as o

pytestmark = pytest.mark.gpu

# the step graph splits the 64 requests into ranges [0, 32) and [32, 64)
SAMPLED = [0, 9, 20, 31, 32, 45, 54, 63]


@pytest.fixture(scope="module", params=[0, 1, 2], ids=["f32", "bf16", "fp8"])
def cfg3(dsd, request):
    fmt = request.param
    ctx_lens = bench.workload_contexts()
    ctx, cap, ids, counts = bench.build_workload(dsd, ctx_lens, 0, fmt)
    q = bench.queries_host(dsd)
    res = ctx.decode_step(np.arange(bench.BATCH), q, output_mode=dsd.OUTPUT_DEBUG)
    rnd = o.stored_round(fmt)
    yield dict(fmt=fmt, ctx=ctx, ctx_lens=ctx_lens, cap=cap, ids=ids, counts=counts, q=q, res=res, rnd=rnd)
    ctx.close()


def request_pages(ctx_lens, cap, r):
    pages = (ctx_lens + bench.P - 1) // bench.P
    first = cap - 1 - int(pages[:r].sum())
    return np.arange(first, first - pages[r], -1, dtype=np.int32)


def test_selection_properties(cfg3):
    res, ctx_lens, cap = cfg3["res"], cfg3["ctx_lens"], cfg3["cap"]
    pages = (ctx_lens + bench.P - 1) // bench.P
    sel = res["selected"]
    assert sel.size == bench.BATCH * bench.K_TOP
    for r in range(bench.BATCH):
        s = sel[r * bench.K_TOP:(r + 1) * bench.K_TOP]
        own = request_pages(ctx_lens, cap, r)
        assert len(set(s.tolist())) == bench.K_TOP
        assert set(s.tolist()) <= set(own.tolist())
        # scores in candidate order; selected are the best by (score desc, id asc)
        off = int(pages[:r].sum())
        sc = res["scores"][off:off + pages[r]]
        order = sorted(range(len(own)), key=lambda i: (-sc[i], own[i]))
        assert [int(own[i]) for i in order[:bench.K_TOP]] == s.tolist()


def test_requests_match_oracle(cfg3):
    """fp32 pages: all 64 requests; bf16/fp8 pages: the sampled 8."""
    for r in (range(bench.BATCH) if cfg3["fmt"] == 0 else SAMPLED):
        check_request_against_oracle(cfg3, r)


def check_request_against_oracle(cfg3, r):
    E, P = bench.E, bench.P
    ctx_lens, cap, res = cfg3["ctx_lens"], cfg3["cap"], cfg3["res"]
    n_tok = int(ctx_lens[r])
    own = request_pages(ctx_lens, cap, r)
    n_pages = len(own)
    base = int(own.min())
    rnd = cfg3["rnd"]   # the stored format's rounding (identity for fp32 pages)
    keys = rnd(o.normal_fill(bench.SEED, 1, (r << 40), n_tok * E).reshape(n_tok, E))
    vals = rnd(o.normal_fill(bench.SEED, 2, (r << 40), n_tok * E).reshape(n_tok, E))
    kp = np.zeros((n_pages, P, E), np.float32)
    vp = np.zeros((n_pages, P, E), np.float32)
    tc = np.zeros(n_pages, np.int32)
    summ = np.zeros((n_pages, E), np.float32)
    for j, pid in enumerate(own):
        loc = int(pid) - base
        t0, t1 = j * P, min(n_tok, (j + 1) * P)
        kp[loc, :t1 - t0] = keys[t0:t1]
        vp[loc, :t1 - t0] = vals[t0:t1]
        tc[loc] = t1 - t0
        summ[loc] = rnd(o.page_summary(keys[t0:t1]))
    # device summaries of a few pages are the oracle's, bit for bit
    for j in (0, n_pages // 2, n_pages - 1):
        _, _, s, n = cfg3["ctx"].download_page(int(own[j]))
        assert n == tc[int(own[j]) - base]
        assert np.array_equal(s.view(np.uint32), summ[int(own[j]) - base].view(np.uint32))
    b = o.Batch(bench.H, bench.D, P, bench.K_TOP, kp, vp, summ, tc, cfg3["q"][r:r + 1],
                np.array([0, n_pages], np.int32), (own - base).astype(np.int32))
    sel, _, out, scores = o.sparse_decode(b)
    pages = (ctx_lens + P - 1) // P
    off = int(pages[:r].sum())
    assert np.array_equal(res["scores"][off:off + n_pages].view(np.uint32),
                          scores.view(np.uint32)), f"request {r}: scores differ"
    got = res["selected"][r * bench.K_TOP:(r + 1) * bench.K_TOP]
    assert np.array_equal(got, sel + base), f"request {r}: selected pages differ"
    diff = float(np.abs(res["outputs"][r] - out[0]).max())
    assert diff <= 1e-4, f"request {r}: output max abs diff {diff}"
