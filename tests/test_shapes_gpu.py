"""Shape and size edges of the CUDA path vs the oracle (GPU).

Covers the kernel variants the config tests do not reach: head_dim 4 and 8
(1 and 2 float4 per lane), H*D = 8192 (two register slots), head_dim that is
not a power of two (1, 3, 5, 80, 100, 127, 200: stored padded to the next
power of two; the reference accepts any head_dim in (0, 128], and up to 256 on
its dense path), head_dim 256, page sizes 1, 32 and 64, a request with more than 8192 candidates (select reads the keys from
global memory), k large enough for long bitonic sorts, and batches at the
1024-request limit.
"""
import numpy as np
import pytest

from oracle import oracle as o

pytestmark = pytest.mark.gpu


def random_batch(rng, H, D, P, k, n_per_req, cap_extra=0, zero_frac=0.0):
    E = H * D
    B = len(n_per_req)
    cap = int(sum(n_per_req)) + cap_extra
    kp = rng.standard_normal((cap, P, E)).astype(np.float32)
    vp = rng.standard_normal((cap, P, E)).astype(np.float32)
    tc = rng.integers(1, P + 1, cap).astype(np.int32)
    if zero_frac:
        kp[rng.random(cap) < zero_frac] = 0.0
    summ = np.zeros((cap, E), np.float32)
    for p in range(cap):
        summ[p] = o.page_summary(kp[p, :tc[p]])
    ids = rng.permutation(cap)[: sum(n_per_req)].astype(np.int32)
    offs = np.concatenate([[0], np.cumsum(n_per_req)]).astype(np.int32)
    q = rng.standard_normal((B, E)).astype(np.float32)
    return o.Batch(H, D, P, k, kp, vp, summ, tc, q, offs, ids)


def run_and_check(dsd, b, tol=1e-4, kv_format=0):
    n = np.diff(b.cand_offsets)
    with dsd.SparseDecodeContext(b.num_heads, b.head_dim, b.page_size, b.top_k, b.capacity,
                                 b.batch, int(n.sum()), max(1, int(np.minimum(n, b.top_k).sum())),
                                 kv_format=kv_format) as ctx:
        ctx.upload_pool(b.key_pool, b.value_pool, b.token_counts)
        res = ctx.decode_batch(b.queries, b.cand_offsets, b.cand_ids)
    sel, so, out, scores = o.sparse_decode(b)
    assert np.array_equal(res["scores"].view(np.uint32), scores.view(np.uint32))
    assert np.array_equal(res["selected"], sel)
    assert float(np.abs(res["outputs"] - out).max()) <= tol


@pytest.mark.parametrize("H,D,P", [(2, 4, 4), (16, 4, 8), (4, 8, 16), (64, 128, 2),
                                   (8, 64, 32), (4, 32, 64), (3, 16, 1),
                                   (3, 1, 4), (5, 3, 8), (4, 5, 4), (2, 80, 8), (4, 100, 16),
                                   (2, 127, 4), (48, 96, 16), (4, 256, 8), (3, 200, 4),
                                   (32, 256, 2)],
                         ids=["d4", "d4_h16", "d8", "e8192", "p32", "p64", "p1_h3",
                              "d1", "d3", "d5", "d80", "d100", "d127", "h48_d96", "d256",
                              "d200", "d256_e8192"])
def test_head_and_page_shapes(dsd, H, D, P):
    rng = np.random.default_rng(H * 1000 + D * 10 + P)
    run_and_check(dsd, random_batch(rng, H, D, P, 5, [3, 17, 40, 9]))


def test_request_with_more_than_8192_candidates(dsd):
    rng = np.random.default_rng(11)
    run_and_check(dsd, random_batch(rng, 2, 8, 2, 64, [9000, 300], zero_frac=0.05))


@pytest.mark.parametrize("k", [511, 1024, 4096])
def test_large_k(dsd, k):
    rng = np.random.default_rng(k)
    run_and_check(dsd, random_batch(rng, 2, 8, 4, k, [5000, 1200, 7]))


def test_batch_at_the_limit(dsd):
    rng = np.random.default_rng(5)
    n = rng.integers(0, 6, 1024)
    run_and_check(dsd, random_batch(rng, 2, 16, 4, 3, list(n)))


@pytest.mark.parametrize("kv_format,H,D", [(1, 4, 5), (1, 2, 80), (2, 3, 12), (2, 2, 100),
                                           (1, 4, 256), (2, 2, 256)],
                         ids=["bf16_d5", "bf16_d80", "fp8_d12", "fp8_d100", "bf16_d256",
                              "fp8_d256"])
def test_padded_head_dim_narrow_pages(dsd, kv_format, H, D):
    """bf16 / fp8 pages with a padded head width, against the oracle on the
    rounded values."""
    rng = np.random.default_rng(kv_format * 1000 + D)
    b = o.stored_batch(random_batch(rng, H, D, 8, 4, [6, 20, 11]), o.stored_round(kv_format))
    run_and_check(dsd, b, kv_format=kv_format)
