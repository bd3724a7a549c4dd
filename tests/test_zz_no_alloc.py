"""The allocation-free decode entry point agrees with the regular one (GPU).

dsd_decode_batch_noalloc is for callers that may not allocate device memory
themselves or through this library -- for example code embedded in a host
framework that owns every allocation through its own allocator or a fixed
memory budget.  It keeps its working memory in one static device array, so
this test checks it through the C ABI against dsd_decode_batch on two calls in
a row (the second call must not see the first call's leftovers).  The file is
named to be collected last.
"""
import ctypes

import numpy as np
import pytest

from oracle import oracle as o

pytestmark = pytest.mark.gpu


def test_noalloc_matches_context_step_twice(dsd):
    torch = pytest.importorskip("torch")
    lib = dsd.load_library()
    b = o.synthetic_batch(32, 128, 16, 8, 12, 200, 1500, 31)
    n = np.diff(b.cand_offsets)
    with dsd.SparseDecodeContext(b.num_heads, b.head_dim, b.page_size, b.top_k, b.capacity,
                                 b.batch, int(n.sum()), int(np.minimum(n, b.top_k).sum())) as ctx:
        ctx.upload_pool(b.key_pool, b.value_pool, b.token_counts)
        kptr, vptr, sptr, cptr = ctx.device_pointers()
        cfg = dsd.ModelConfig(b.num_heads, b.head_dim, b.page_size, b.top_k)
        offs = np.ascontiguousarray(b.cand_offsets, np.int32)
        d_ids = torch.from_numpy(b.cand_ids.astype(np.int32)).cuda()
        rng = np.random.default_rng(5)
        queries = [b.queries, rng.uniform(-1, 1, b.queries.shape).astype(np.float32)]
        for q in queries:
            expected = ctx.decode_batch(q, b.cand_offsets, b.cand_ids)["outputs"]
            d_q = torch.from_numpy(q).cuda()
            d_out = torch.full_like(d_q, float("nan"))
            torch.cuda.synchronize()
            rc = lib.dsd_decode_batch_noalloc(
                0, ctypes.byref(cfg), b.batch, offs.ctypes.data_as(dsd._I32P),
                ctypes.c_void_p(d_ids.data_ptr()), ctypes.c_void_p(d_q.data_ptr()),
                ctypes.c_void_p(sptr), ctypes.c_void_p(kptr), ctypes.c_void_p(vptr),
                ctypes.c_void_p(cptr), ctypes.c_void_p(d_out.data_ptr()), None)
            assert rc == dsd.DSD_OK, lib.dsd_last_error().decode()
            got = d_out.cpu().numpy()
            assert float(np.abs(got - expected).max()) <= 1e-4


def test_noalloc_rejects_sizes_beyond_its_limit(dsd):
    lib = dsd.load_library()
    cfg = dsd.ModelConfig(32, 128, 16, 8)
    offs = np.zeros(258, np.int32)
    rc = lib.dsd_decode_batch_noalloc(0, ctypes.byref(cfg), 257,
                                      offs.ctypes.data_as(dsd._I32P), *([None] * 8))
    assert rc == dsd.DSD_EINVAL
    assert "256" in lib.dsd_last_error().decode()
