"""Failure detection and the device-side input generators (GPU).

* A device wait that can never complete gives up after its budget, the call
  returns DSD_ETIMEOUT and the context stays usable (nothing faults or hangs).
* Bad inputs are rejected on the host before any launch, and the context keeps
  working afterwards.
* Synthetic prefill / append (the reference's admission mode 2 hash) and the
  normal workload generator write exactly what the oracle restatements compute;
  summaries follow the CPU formulas bit for bit.
"""
import numpy as np
import pytest

from oracle import oracle as o

pytestmark = pytest.mark.gpu


def small_ctx(dsd, cap=16, tables=True, H=4, D=16):
    return dsd.SparseDecodeContext(H, D, 8, 3, cap, 4, cap, 12,
                                   max_requests=4 if tables else 0, max_pages_per_request=cap)


# (H, D): the stored layout; a head_dim that is not a power of two >= 4 is
# stored padded (5 -> 8, 80 -> 128, 3 -> 4) and must read back unchanged
HEAD_SHAPES = pytest.mark.parametrize("H,D", [(4, 16), (3, 5), (2, 80), (5, 3)],
                                      ids=["h4d16", "h3d5_padded", "h2d80_padded", "h5d3_padded"])


def decode_checks(dsd, ctx):
    rng = np.random.default_rng(3)
    E, P = 64, 8
    k = rng.standard_normal((4 * P, E)).astype(np.float32)
    v = rng.standard_normal((4 * P, E)).astype(np.float32)
    ctx.upload_pages([0, 1, 2, 3], [P] * 4, k, v)
    q = rng.standard_normal((1, E)).astype(np.float32)
    res = ctx.decode_batch(q, [0, 4], [0, 1, 2, 3])
    kp = np.zeros((16, P, E), np.float32); kp[:4] = k.reshape(4, P, E)
    vp = np.zeros((16, P, E), np.float32); vp[:4] = v.reshape(4, P, E)
    tc = np.zeros(16, np.int32); tc[:4] = P
    summ = np.zeros((16, E), np.float32)
    for p in range(4):
        summ[p] = o.page_summary(kp[p])
    b = o.Batch(4, 16, P, 3, kp, vp, summ, tc, q, np.array([0, 4], np.int32),
                np.array([0, 1, 2, 3], np.int32))
    sel, _, out, _ = o.sparse_decode(b)
    assert np.array_equal(res["selected"], sel)
    assert float(np.abs(res["outputs"] - out).max()) <= 1e-5


def test_bounded_wait_times_out_and_context_survives(dsd):
    with small_ctx(dsd) as ctx:
        rc = ctx.lib.dsd_selftest_bounded_wait(ctx.h, 2_000_000)
        assert rc == dsd.DSD_ETIMEOUT, ctx.lib.dsd_last_error()
        assert b"budget" in ctx.lib.dsd_last_error()
        decode_checks(dsd, ctx)                     # the context is still usable


def test_bad_inputs_rejected_before_launch(dsd):
    with small_ctx(dsd) as ctx:
        with pytest.raises(dsd.OutOfRange):
            ctx.upload_pages([99], [8], np.zeros((8, 64), np.float32), np.zeros((8, 64), np.float32))
        with pytest.raises(dsd.InvalidArgument):
            ctx.upload_pages([1], [9], np.zeros((9, 64), np.float32), np.zeros((9, 64), np.float32))
        with pytest.raises(dsd.InvalidArgument):
            ctx.decode_step(np.array([42]), np.zeros((1, 64), np.float32))   # unknown request
        with pytest.raises(dsd.InvalidArgument):
            ctx.decode_batch(np.zeros((5, 64), np.float32), [0, 1, 2, 3, 4, 5], [0, 1, 2, 3, 4])
        with pytest.raises(dsd.OutOfRange):
            ctx.append_tokens([0], [8], np.zeros((1, 64), np.float32), np.zeros((1, 64), np.float32))
        decode_checks(dsd, ctx)


@HEAD_SHAPES
def test_synthetic_prefill_and_append_match_reference_hash(dsd, H, D):
    E, P = H * D, 8
    with small_ctx(dsd, H=H, D=D) as ctx:
        ctx.prefill_synthetic([5, 6, 7], [8, 8, 3], request_id=11)
        for i, (pid, n) in enumerate([(5, 8), (6, 8), (7, 3)]):
            k, v, s, cnt = ctx.download_page(pid)
            assert cnt == n
            ek = o.synthetic_prompt(11, i, n, E, 1)
            ev = o.synthetic_prompt(11, i, n, E, 2)
            assert np.array_equal(k[:n], ek) and np.array_equal(v[:n], ev)
            assert np.array_equal(s.view(np.uint32), o.page_summary(ek).view(np.uint32))
        # decode tokens into page 7 (offsets 3, 4) then a fresh page 8
        ctx.append_tokens_synthetic([7, 7, 8], [3, 4, 0], [11, 11, 11], [0, 1, 2])
        k, v, s, cnt = ctx.download_page(7)
        assert cnt == 5
        summ = o.page_summary(o.synthetic_prompt(11, 2, 3, E, 1))
        for off, step in ((3, 0), (4, 1)):
            key = o.synthetic_decode(11, step, E, 1)
            assert np.array_equal(k[off], key)
            assert np.array_equal(v[off], o.synthetic_decode(11, step, E, 2))
            summ = o.running_mean_append(summ, key, off)
        assert np.array_equal(s.view(np.uint32), summ.view(np.uint32))
        k8, _, s8, cnt8 = ctx.download_page(8)
        assert cnt8 == 1 and np.array_equal(s8, o.synthetic_decode(11, 2, E, 1))


@HEAD_SHAPES
def test_normal_generator_pages_match_oracle(dsd, H, D):
    E, P = H * D, 8
    with small_ctx(dsd, H=H, D=D) as ctx:
        ctx.generate_normal([3, 4], [8, 5], [2, 2], [0, 8], seed=9)
        for pid, first, n in ((3, 0, 8), (4, 8, 5)):
            k, v, s, cnt = ctx.download_page(pid)
            assert cnt == n
            ek = o.normal_fill(9, 1, (2 << 40) + first * E, n * E).reshape(n, E)
            ev = o.normal_fill(9, 2, (2 << 40) + first * E, n * E).reshape(n, E)
            assert np.array_equal(k[:n], ek) and np.array_equal(v[:n], ev)
            assert np.array_equal(s.view(np.uint32), o.page_summary(ek).view(np.uint32))


def test_free_pages_clear_metadata(dsd):
    with small_ctx(dsd) as ctx:
        ctx.prefill_synthetic([0, 1], [8, 2], request_id=1)
        ctx.free_pages([1])
        tc, live = ctx.download_metadata()
        assert tc[0] == 8 and tc[1] == 0 and live[0] == 1 and live[1] == 0
        _, _, s, _ = ctx.download_page(1)
        assert not s.any()


@HEAD_SHAPES
def test_upload_append_download_round_trip(dsd, H, D):
    """Rows go in and come back in the caller's layout whatever the stored
    head width; summaries follow the CPU formulas bit for bit."""
    E, P = H * D, 8
    rng = np.random.default_rng(H * 100 + D)
    k = rng.standard_normal((P + 3, E)).astype(np.float32)
    v = rng.standard_normal((P + 3, E)).astype(np.float32)
    with small_ctx(dsd, H=H, D=D) as ctx:
        ctx.upload_pages([2, 9], [P, 3], k, v)
        k9, v9, s9, n9 = ctx.download_page(9)
        assert n9 == 3 and np.array_equal(k9[:3], k[P:]) and np.array_equal(v9[:3], v[P:])
        assert np.array_equal(s9.view(np.uint32), o.page_summary(k[P:]).view(np.uint32))
        nk = rng.standard_normal((2, E)).astype(np.float32)
        nv = rng.standard_normal((2, E)).astype(np.float32)
        ctx.append_tokens([9, 9], [3, 4], nk, nv)
        k9, v9, s9, n9 = ctx.download_page(9)
        assert n9 == 5 and np.array_equal(k9[3:5], nk) and np.array_equal(v9[3:5], nv)
        summ = o.page_summary(k[P:])
        for off in (3, 4):
            summ = o.running_mean_append(summ, nk[off - 3], off)
        assert np.array_equal(s9.view(np.uint32), summ.view(np.uint32))


def test_append_pages_multi_is_all_or_nothing(dsd):
    """dsd_request_append_pages_multi: pages join their requests' tables in
    order; a call that would overflow one table is refused before any change."""
    with small_ctx(dsd, cap=16) as ctx:   # 4 page-table slots of 16 pages
        ctx.set_request_pages(7, [0, 1])
        ctx.append_request_pages_multi([7, 9, 7], [2, 3, 4])
        assert ctx.request_num_pages(7) == 4 and ctx.request_num_pages(9) == 1
        with pytest.raises(dsd.InvalidArgument):
            # request 9 holds 1 page: 16 more would exceed its 16-entry table
            ctx.append_request_pages_multi([11] + [9] * 16, [0] + list(range(16)))
        assert ctx.request_num_pages(9) == 1 and ctx.request_num_pages(11) == 0
        # no slot was taken by the refused call: two of the four are still free
        ctx.set_request_pages(12, [5])
        ctx.set_request_pages(13, [6])
        with pytest.raises(dsd.DsdError):
            ctx.set_request_pages(14, [8])
