"""GPU parity of the decode step against the CPU oracle (sparse_cpu restated).

Bar (per the reference's own tests, tests/test_sparse_cuda.cpp:23-84):
selected page ids equal IN ORDER; outputs within the case tolerance max-abs
(<= 1e-4 everywhere, the reference's per-case 1e-5..5e-5 where it has one);
scores bit-identical (the score kernel follows ScorePagesCpu's operation order).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def make_ctx(dsd, b, top_k=None, tables=False, **kw):
    k = b.top_k if top_k is None else top_k
    n = np.diff(b.cand_offsets)
    opts = dict(capacity_pages=b.capacity, max_batch=max(1, b.batch),
                max_candidates=max(1, int(n.sum())),
                max_selected=max(1, int(np.minimum(n, k).sum())))
    if tables:
        opts.update(max_requests=max(1, b.batch), max_pages_per_request=max(1, int(n.max())))
    opts.update(kw)
    return dsd.SparseDecodeContext(b.num_heads, b.head_dim, b.page_size, k, **opts)


def check_against_oracle(orc, b, res, tol, top_k=None):
    sel, so, out, scores = orc.sparse_decode(b, top_k)
    assert np.array_equal(res["scores"].view(np.uint32), scores.view(np.uint32)), \
        "scores differ from ScorePagesCpu bit for bit"
    for r in range(b.batch):
        got = res["selected"][so[r]:so[r + 1]]
        exp = sel[so[r]:so[r + 1]]
        assert np.array_equal(got, exp), f"request {r}: selected {got} != {exp}"
    diff = float(np.abs(res["outputs"] - out).max()) if out.size else 0.0
    assert diff <= tol, f"max abs diff {diff} > {tol}"
    return diff


# tests/test_sparse_cuda.cpp:217-251 and :120-132 (shape, seed, tolerance)
REFERENCE_CASES = [
    ("small", (2, 8, 4, 2, 3, 5, 19, 11), 1e-5),
    ("ragged", (4, 16, 16, 3, 4, 33, 97, 7), 2e-5),
    ("wide", (2, 64, 8, 4, 2, 17, 45, 17), 5e-5),
    ("larger_candidates", (2, 16, 8, 8, 2, 160, 184, 123), 3e-5),
]


@pytest.mark.parametrize("name,cfg,tol", REFERENCE_CASES, ids=[c[0] for c in REFERENCE_CASES])
def test_reference_synthetic_cases(dsd, orc, name, cfg, tol):
    b = orc.synthetic_batch(*cfg)
    with make_ctx(dsd, b) as ctx:
        ctx.upload_pool(b.key_pool, b.value_pool, b.token_counts)
        res = ctx.decode_batch(b.queries, b.cand_offsets, b.cand_ids, timing=True)
        check_against_oracle(orc, b, res, tol)
        assert res["timing"]["total_ms"] > 0.0


@pytest.mark.parametrize("cfg", [
    (8, 16, 16, 8, 1, 1024, 1024, 7),      # config 1 as dsd_bench runs it (H=8, D=16)
    (32, 128, 16, 8, 1, 1024, 1024, 7),    # config 1 at the BASELINE shape
    (32, 128, 16, 8, 16, 512, 2048, 7),    # config 2
], ids=["cfg1_h8d16", "cfg1_h32d128", "cfg2"])
def test_baseline_configs(dsd, orc, cfg):
    b = orc.synthetic_batch(*cfg)
    with make_ctx(dsd, b) as ctx:
        ctx.upload_pool(b.key_pool, b.value_pool, b.token_counts)
        res = ctx.decode_batch(b.queries, b.cand_offsets, b.cand_ids)
        check_against_oracle(orc, b, res, 1e-4)


def test_device_summaries_bitwise(dsd, orc):
    b = orc.synthetic_batch(32, 128, 16, 8, 4, 100, 300, 5)
    with make_ctx(dsd, b) as ctx:
        ctx.upload_pool(b.key_pool, b.value_pool, b.token_counts)
        for p in range(b.capacity):
            k, v, s, n = ctx.download_page(p)
            assert n == b.token_counts[p]
            assert np.array_equal(k[:n], b.key_pool[p, :n])
            assert np.array_equal(v[:n], b.value_pool[p, :n])
            assert np.array_equal(s.view(np.uint32), b.summaries[p].view(np.uint32)), p


def test_top_k_zero_gives_zero_output(dsd, orc):
    # tests/test_sparse_cuda.cpp:86-118
    b = orc.synthetic_batch(2, 8, 4, 0, 3, 5, 19, 11)
    with make_ctx(dsd, b, top_k=0) as ctx:
        ctx.upload_pool(b.key_pool, b.value_pool, b.token_counts)
        res = ctx.decode_batch(b.queries, b.cand_offsets, b.cand_ids)
        assert res["selected"].size == 0
        assert not res["outputs"].any()


def test_tie_break_lower_page_id(dsd, orc):
    # tests/test_sparse_cuda.cpp:134-169: 4 pages of zero keys, candidates [3,2,1,0], k=2
    H, D, P = 2, 8, 4
    E = H * D
    cap = 4
    kp = np.zeros((cap, P, E), np.float32)
    vp = np.random.default_rng(0).uniform(-1, 1, (cap, P, E)).astype(np.float32)
    tc = np.full(cap, P, np.int32)
    q = np.random.default_rng(1).uniform(-1, 1, (1, E)).astype(np.float32)
    b = orc.Batch(H, D, P, 2, kp, vp, np.zeros((cap, E), np.float32), tc, q,
                  np.array([0, 4], np.int32), np.array([3, 2, 1, 0], np.int32))
    with make_ctx(dsd, b) as ctx:
        ctx.upload_pool(kp, vp, tc)
        res = ctx.decode_batch(q, b.cand_offsets, b.cand_ids)
        assert list(res["selected"]) == [0, 1]
        check_against_oracle(orc, b, res, 1e-5)


@pytest.mark.parametrize("k", [1, 8, 16, 17, 32, 64])
def test_forced_ties_and_signed_zero(dsd, orc, k):
    """Duplicated page contents, all-zero pages (score +0/-0) and ragged pages."""
    rng = np.random.default_rng(k)
    H, D, P = 4, 32, 8
    E = H * D
    cap = 160
    kp = rng.standard_normal((cap, P, E)).astype(np.float32)
    vp = rng.standard_normal((cap, P, E)).astype(np.float32)
    tc = rng.integers(1, P + 1, cap).astype(np.int32)
    # groups of identical pages -> identical summaries -> exact score ties
    for g in range(0, 60, 4):
        kp[g + 1:g + 4] = kp[g]
        tc[g + 1:g + 4] = tc[g]
    kp[60:80] = 0.0                                   # zero summaries -> score 0
    kp[80:90] = -0.0
    kp[90:95] = 1e-30                                 # tiny: product underflows to +-0
    summ = np.zeros((cap, E), np.float32)
    for p in range(cap):
        summ[p] = orc.page_summary(kp[p, :tc[p]])
    B = 5
    q = rng.standard_normal((B, E)).astype(np.float32)
    q[4] = 0.0                                        # every score is +-0 for request 4
    perm = rng.permutation(cap)
    offs = np.array([0, 40, 70, 120, 130, 160], np.int32)
    b = orc.Batch(H, D, P, k, kp, vp, summ, tc, q, offs, perm.astype(np.int32))
    with make_ctx(dsd, b) as ctx:
        ctx.upload_pool(kp, vp, tc)
        res = ctx.decode_batch(q, offs, b.cand_ids)
        check_against_oracle(orc, b, res, 1e-4)


def test_sparse_equals_dense_when_k_covers_all_pages(dsd, orc):
    # tests/test_reference.cpp:270-290 (H2 D8 P4 k64, B3 ctx 12, seed 123, 1e-5)
    b = orc.synthetic_batch(2, 8, 4, 64, 3, 12, 12, 123)
    with make_ctx(dsd, b) as ctx:
        ctx.upload_pool(b.key_pool, b.value_pool, b.token_counts)
        res = ctx.decode_batch(b.queries, b.cand_offsets, b.cand_ids)
        dense = orc.dense_decode(b)
        assert float(np.abs(res["outputs"] - dense).max()) <= 1e-5


def test_empty_and_ragged_requests(dsd, orc):
    """Requests with no candidates mix with normal ones; outputs for them are zero."""
    b = orc.synthetic_batch(4, 16, 8, 3, 4, 1, 40, 3)
    offs = b.cand_offsets
    # rebuild the CSR with request 1 and 3 emptied
    segs = [b.cand_ids[offs[r]:offs[r + 1]] for r in range(b.batch)]
    segs[1] = segs[1][:0]
    segs[3] = segs[3][:0]
    new_offs = np.concatenate([[0], np.cumsum([len(s) for s in segs])]).astype(np.int32)
    b2 = orc.Batch(b.num_heads, b.head_dim, b.page_size, b.top_k, b.key_pool, b.value_pool,
                   b.summaries, b.token_counts, b.queries, new_offs,
                   np.concatenate(segs).astype(np.int32))
    with make_ctx(dsd, b2) as ctx:
        ctx.upload_pool(b.key_pool, b.value_pool, b.token_counts)
        res = ctx.decode_batch(b2.queries, b2.cand_offsets, b2.cand_ids)
        check_against_oracle(orc, b2, res, 1e-5)
        assert not res["outputs"][1].any() and not res["outputs"][3].any()


def test_capacity_errors_raise_invalid_argument(dsd, orc):
    # sparse_batched_attention.cu:600-608 throws std::invalid_argument
    b = orc.synthetic_batch(2, 8, 4, 2, 3, 5, 19, 11)
    with make_ctx(dsd, b, max_batch=2) as ctx:
        ctx.upload_pool(b.key_pool, b.value_pool, b.token_counts)
        with pytest.raises(dsd.InvalidArgument):
            ctx.decode_batch(b.queries, b.cand_offsets, b.cand_ids)
    with make_ctx(dsd, b) as ctx:
        bad = b.cand_ids.copy()
        bad[0] = b.capacity + 5
        with pytest.raises(dsd.OutOfRange):
            ctx.decode_batch(b.queries, b.cand_offsets, bad)


def test_page_table_step_matches_csr_step(dsd, orc):
    b = orc.synthetic_batch(32, 128, 16, 8, 16, 512, 2048, 9)
    with make_ctx(dsd, b, tables=True) as ctx:
        ctx.upload_pool(b.key_pool, b.value_pool, b.token_counts)
        for r in range(b.batch):
            ctx.set_request_pages(r, b.cand_ids[b.cand_offsets[r]:b.cand_offsets[r + 1]])
        a = ctx.decode_batch(b.queries, b.cand_offsets, b.cand_ids)
        s = ctx.decode_step(np.arange(b.batch), b.queries)
        assert np.array_equal(a["selected"], s["selected"])
        assert np.array_equal(a["scores"].view(np.uint32), s["scores"].view(np.uint32))
        assert np.array_equal(a["outputs"], s["outputs"])
        check_against_oracle(orc, b, s, 1e-4)
        # a subset in another order
        order = np.array([5, 2, 11], np.int32)
        sub = ctx.decode_step(order, b.queries[order])
        assert np.array_equal(sub["outputs"], a["outputs"][order])


def test_bound_graph_step_matches_host_step(dsd, orc):
    torch = pytest.importorskip("torch")
    b = orc.synthetic_batch(32, 128, 16, 8, 8, 300, 900, 21)
    with make_ctx(dsd, b, tables=True) as ctx:
        ctx.upload_pool(b.key_pool, b.value_pool, b.token_counts)
        for r in range(b.batch):
            ctx.set_request_pages(r, b.cand_ids[b.cand_offsets[r]:b.cand_offsets[r + 1]])
        host = ctx.decode_step(np.arange(b.batch), b.queries)
        dq = torch.from_numpy(b.queries).cuda()
        do = torch.zeros_like(dq)
        ctx.bind_requests(np.arange(b.batch))
        ctx.decode_bound(dq.data_ptr(), do.data_ptr())
        torch.cuda.synchronize()
        assert np.array_equal(do.cpu().numpy(), host["outputs"])
        do.zero_()
        t = ctx.decode_bound_timed(dq.data_ptr(), do.data_ptr())
        assert np.array_equal(do.cpu().numpy(), host["outputs"])
        assert t["score_ms"] > 0 and t["attention_ms"] > 0


def test_pinned_host_buffers_match_pageable(dsd, orc):
    """Pinned caller buffers are DMA'd directly; results equal the staged path."""
    torch = pytest.importorskip("torch")
    b = orc.synthetic_batch(32, 128, 16, 8, 8, 300, 900, 23)
    with make_ctx(dsd, b, tables=True) as ctx:
        ctx.upload_pool(b.key_pool, b.value_pool, b.token_counts)
        for r in range(b.batch):
            ctx.set_request_pages(r, b.cand_ids[b.cand_offsets[r]:b.cand_offsets[r + 1]])
        ref = ctx.decode_step(np.arange(b.batch), b.queries, output_mode=dsd.OUTPUT_OUTPUTS)
        q_pin = torch.empty(b.queries.shape, dtype=torch.float32, pin_memory=True).numpy()
        q_pin[:] = b.queries
        o_pin = torch.zeros(b.queries.shape, dtype=torch.float32, pin_memory=True).numpy()
        got = ctx.decode_step(np.arange(b.batch), q_pin, output_mode=dsd.OUTPUT_OUTPUTS, out=o_pin)
        assert got["outputs"] is o_pin
        assert np.array_equal(o_pin, ref["outputs"])
        res = ctx.decode_batch(q_pin, b.cand_offsets, b.cand_ids)
        check_against_oracle(orc, b, res, 1e-4)


# tests/test_dense_cuda.cpp:96-156: dense_gpu vs dense_cpu on the reference's
# five shapes (head_dim 80 is stored padded to 128), plus config-3 width and
# head_dim 256 (the top of the reference dense path's range)
DENSE_CASES = [((2, 8, 4, 8, 3, 5, 19, 11), 1e-5), ((4, 16, 16, 8, 5, 33, 97, 7), 2e-5),
               ((2, 64, 8, 16, 4, 17, 45, 17), 5e-5), ((2, 80, 8, 16, 4, 17, 45, 19), 5e-5),
               ((2, 128, 8, 16, 2, 9, 25, 29), 1e-4), ((32, 128, 16, 8, 4, 256, 1024, 7), 1e-4),
               ((2, 256, 8, 16, 2, 9, 25, 3), 1e-4)]


@pytest.mark.parametrize("cfg,tol", DENSE_CASES, ids=[f"dense{i}" for i in range(len(DENSE_CASES))])
def test_dense_baseline_matches_dense_cpu(dsd, orc, cfg, tol):
    b = orc.synthetic_batch(*cfg)
    n = np.diff(b.cand_offsets)
    with dsd.SparseDecodeContext(b.num_heads, b.head_dim, b.page_size, b.top_k, b.capacity,
                                 b.batch, int(n.sum()), int(n.sum())) as ctx:
        ctx.upload_pool(b.key_pool, b.value_pool, b.token_counts)
        ctx.set_dense(True)
        res = ctx.decode_batch(b.queries, b.cand_offsets, b.cand_ids)
        assert np.array_equal(res["selected"], b.cand_ids)      # every page, candidate order
        assert float(np.abs(res["outputs"] - orc.dense_decode(b)).max()) <= tol
        ctx.set_dense(False)                                    # back to the sparse path
        check_against_oracle(orc, b, ctx.decode_batch(b.queries, b.cand_offsets, b.cand_ids), 1e-4)


@pytest.mark.parametrize("batch", [1, 2, 3, 7, 8, 17, 64])
def test_step_io_split_by_request_range(dsd, orc, batch):
    """Untimed page-table steps upload the second request range's queries and
    download the first range's outputs on a copy stream; every batch size,
    pinned or pageable, two steps in flight included, equals the oracle."""
    torch = pytest.importorskip("torch")
    b = orc.synthetic_batch(8, 32, 16, 4, batch, 100, 400, 31 + batch)
    with make_ctx(dsd, b, tables=True) as ctx:
        ctx.upload_pool(b.key_pool, b.value_pool, b.token_counts)
        for r in range(b.batch):
            ctx.set_request_pages(r, b.cand_ids[b.cand_offsets[r]:b.cand_offsets[r + 1]])
        reqs = np.arange(b.batch)
        check_against_oracle(orc, b, ctx.decode_step(reqs, b.queries), 1e-4)
        _, _, out, _ = orc.sparse_decode(b)
        q_pin = torch.empty(b.queries.shape, dtype=torch.float32, pin_memory=True).numpy()
        q_pin[:] = b.queries
        o_pin = torch.zeros(b.queries.shape, dtype=torch.float32, pin_memory=True).numpy()
        ctx.reset_transfer_stats()
        ctx.decode_step(reqs, q_pin, output_mode=dsd.OUTPUT_OUTPUTS, out=o_pin)
        assert float(np.abs(o_pin - out).max()) <= 1e-4
        # the outputs reach the host whether copied or written by the kernels
        st = ctx.transfer_stats()
        assert st["d2h_bytes"] >= o_pin.nbytes and st["h2d_bytes"] >= q_pin.nbytes
        if batch == 17:
            # page-locked result buffers are written by the kernels directly (one
            # step graph per buffer, at most 16 kept): cycle through more than that
            for i in range(18):
                o_i = torch.full(b.queries.shape, float("nan"), dtype=torch.float32,
                                 pin_memory=True).numpy()
                ctx.decode_step(reqs, q_pin, output_mode=dsd.OUTPUT_OUTPUTS, out=o_i)
                assert float(np.abs(o_i - out).max()) <= 1e-4, i
        ctx.decode_step_begin(reqs, q_pin)
        ctx.decode_step_begin(reqs, b.queries)
        for _ in range(2):
            assert float(np.abs(ctx.decode_step_end()["outputs"] - out).max()) <= 1e-4
        # a result buffer too small or of the wrong type is refused before any copy
        with pytest.raises(dsd.InvalidArgument):
            ctx.decode_step(reqs, q_pin, output_mode=dsd.OUTPUT_OUTPUTS,
                            out=np.zeros((batch, b.ept - 1), np.float32))
        with pytest.raises(dsd.InvalidArgument):
            ctx.decode_step(reqs, q_pin, output_mode=dsd.OUTPUT_OUTPUTS,
                            out=np.zeros((batch, b.ept), np.float64))
