"""The allocation-free decode entry point agrees with the regular one (GPU).

dsd_decode_batch_noalloc is for callers that may not allocate device memory
themselves or through this library -- for example code embedded in a host
framework that owns every allocation through its own allocator or a fixed
memory budget.  It keeps its working memory in one static device array, so
these tests call it through the C ABI on two calls in a row (the second call
must not see the first call's leftovers) and compare it with dsd_decode_batch
and with the oracle, on a small batch and on one that reaches its limit of
8192 selected pages; a page id outside the pool is rejected on the device
before anything is read.  The file is named to be collected last.
"""
import ctypes

import numpy as np
import pytest

from oracle import oracle as o

pytestmark = pytest.mark.gpu


def noalloc(dsd, lib, b, ctx, d_ids, d_q, d_out, torch):
    kptr, vptr, sptr, cptr = ctx.device_pointers()
    cfg = dsd.ModelConfig(b.num_heads, b.head_dim, b.page_size, b.top_k)
    offs = np.ascontiguousarray(b.cand_offsets, np.int32)
    torch.cuda.synchronize()
    return lib.dsd_decode_batch_noalloc(
        0, ctypes.byref(cfg), b.capacity, b.batch, offs.ctypes.data_as(dsd._I32P),
        ctypes.c_void_p(d_ids.data_ptr()), ctypes.c_void_p(d_q.data_ptr()),
        ctypes.c_void_p(sptr), ctypes.c_void_p(kptr), ctypes.c_void_p(vptr),
        ctypes.c_void_p(cptr), ctypes.c_void_p(d_out.data_ptr()), None)


@pytest.mark.parametrize("shape", [(32, 128, 16, 8, 12, 200, 1500, 31),
                                   # 256 requests x k=32 = 8192 selected pages (the limit)
                                   (4, 64, 16, 32, 256, 528, 1024, 5)],
                         ids=["batch12", "selected_limit"])
def test_noalloc_matches_context_step_and_oracle_twice(dsd, shape):
    torch = pytest.importorskip("torch")
    lib = dsd.load_library()
    b = o.synthetic_batch(*shape)
    n = np.diff(b.cand_offsets)
    with dsd.SparseDecodeContext(b.num_heads, b.head_dim, b.page_size, b.top_k, b.capacity,
                                 b.batch, int(n.sum()), int(np.minimum(n, b.top_k).sum())) as ctx:
        ctx.upload_pool(b.key_pool, b.value_pool, b.token_counts)
        d_ids = torch.from_numpy(b.cand_ids.astype(np.int32)).cuda()
        rng = np.random.default_rng(5)
        queries = [b.queries, rng.uniform(-1, 1, b.queries.shape).astype(np.float32)]
        for q in queries:
            expected = ctx.decode_batch(q, b.cand_offsets, b.cand_ids)["outputs"]
            b.queries = q
            _, _, want, _ = o.sparse_decode(b)
            d_q = torch.from_numpy(q).cuda()
            d_out = torch.full_like(d_q, float("nan"))
            rc = noalloc(dsd, lib, b, ctx, d_ids, d_q, d_out, torch)
            assert rc == dsd.DSD_OK, lib.dsd_last_error().decode()
            got = d_out.cpu().numpy()
            assert float(np.abs(got - expected).max()) <= 1e-4
            assert float(np.abs(got - want).max()) <= 1e-4


def test_noalloc_rejects_out_of_range_page_id_on_device(dsd):
    """An id beyond the pool is caught by the first kernel: DSD_EINVAL, zero
    outputs, nothing loaded; the next valid call is unaffected."""
    torch = pytest.importorskip("torch")
    lib = dsd.load_library()
    b = o.synthetic_batch(8, 32, 16, 4, 3, 40, 120, 9)
    n = np.diff(b.cand_offsets)
    with dsd.SparseDecodeContext(b.num_heads, b.head_dim, b.page_size, b.top_k, b.capacity,
                                 b.batch, int(n.sum()), int(np.minimum(n, b.top_k).sum())) as ctx:
        ctx.upload_pool(b.key_pool, b.value_pool, b.token_counts)
        d_q = torch.from_numpy(b.queries).cuda()
        for bad in (b.capacity, 1 << 30, -1):
            ids = b.cand_ids.astype(np.int32).copy()
            ids[len(ids) // 2] = bad
            d_out = torch.full_like(d_q, float("nan"))
            rc = noalloc(dsd, lib, b, ctx, torch.from_numpy(ids).cuda(), d_q, d_out, torch)
            assert rc == dsd.DSD_EINVAL
            assert "capacity" in lib.dsd_last_error().decode()
            assert not bool(d_out.abs().sum().item())
        d_out = torch.full_like(d_q, float("nan"))
        rc = noalloc(dsd, lib, b, ctx, torch.from_numpy(b.cand_ids.astype(np.int32)).cuda(),
                     d_q, d_out, torch)
        assert rc == dsd.DSD_OK, lib.dsd_last_error().decode()
        _, _, want, _ = o.sparse_decode(b)
        assert float(np.abs(d_out.cpu().numpy() - want).max()) <= 1e-4


def test_noalloc_rejects_sizes_beyond_its_limit(dsd):
    lib = dsd.load_library()
    cfg = dsd.ModelConfig(32, 128, 16, 8)
    offs = np.zeros(258, np.int32)
    rc = lib.dsd_decode_batch_noalloc(0, ctypes.byref(cfg), 100, 257,
                                      offs.ctypes.data_as(dsd._I32P), *([None] * 8))
    assert rc == dsd.DSD_EINVAL
    assert "256" in lib.dsd_last_error().decode()
