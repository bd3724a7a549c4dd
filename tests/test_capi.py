"""The C-ABI library loads and exports every symbol include/dsd_b200.h declares (CPU)."""
import os
import re

import pytest

from conftest import ROOT, load_pkg

HEADER = os.path.join(ROOT, "include", "dsd_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(dsd_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in ["dsd_ctx_create", "dsd_ctx_destroy", "dsd_pool_upload_pages",
                     "dsd_pool_prefill_synthetic", "dsd_append_tokens", "dsd_pool_free_pages",
                     "dsd_decode_batch", "dsd_decode_step", "dsd_download_page",
                     "dsd_download_metadata", "dsd_get_transfer_stats", "dsd_last_error"]:
        assert required in names


def test_library_exports_every_declared_symbol():
    dsd = load_pkg()
    lib = dsd.load_library()
    for name in declared_functions():
        assert hasattr(lib, name), name
    bound = {n for n, _, _ in dsd.SIGNATURES}
    assert set(declared_functions()) <= bound


def test_no_gpu_is_reported_cleanly():
    dsd = load_pkg()
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    assert dsd.available() is False
    with pytest.raises(dsd.DsdError):
        dsd.SparseDecodeContext(4, 16, 16, 4, 8, 2, 8, 8)


def test_host_normal_generator_matches_oracle():
    from oracle import oracle as o
    import numpy as np
    dsd = load_pkg()
    idx = dsd.normal_index(5, 1234, 4096, 17)
    a = dsd.generate_normal_host(7, 1, idx, 5000)
    b = o.normal_fill(7, 1, idx, 5000)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
