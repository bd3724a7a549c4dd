"""CUDA path vs the reference's own outputs stored in tests/golden (GPU)."""
import glob
import os

import numpy as np
import pytest

from oracle import oracle as o

pytestmark = pytest.mark.gpu

GOLDEN = sorted(p for p in glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz"))
                if not os.path.basename(p).startswith("continuous"))
TOL = {"small": 1e-5, "ragged": 2e-5, "wide": 5e-5, "larger_candidates": 3e-5,
       "sparse_eq_dense": 1e-5}


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_cuda_matches_reference_golden(dsd, path):
    name = os.path.basename(path)[:-4]
    g = np.load(path)
    b = o.synthetic_batch(*tuple(int(x) for x in g["config"]))
    n = np.diff(b.cand_offsets)
    ctx = dsd.SparseDecodeContext(b.num_heads, b.head_dim, b.page_size, b.top_k, b.capacity,
                                  b.batch, int(n.sum()), int(np.minimum(n, b.top_k).sum()))
    with ctx:
        ctx.upload_pool(b.key_pool, b.value_pool, b.token_counts)
        res = ctx.decode_batch(b.queries, b.cand_offsets, b.cand_ids)
    assert np.array_equal(res["selected"], g["selected"])
    assert np.array_equal(res["scores"].view(np.uint32), g["scores"].view(np.uint32))
    tol = TOL.get(name, 1e-4)
    assert float(np.abs(res["outputs"] - g["outputs"]).max()) <= tol
