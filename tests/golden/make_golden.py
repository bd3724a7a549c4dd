"""Regenerates the golden fixtures from the UNMODIFIED reference CPU code.

Run in a container that has the reference sources (oracle/_ref is built from
them by `make -C oracle ref`):

    python tests/golden/make_golden.py

For every case it runs the reference's BuildSyntheticBatch and
DecodePipeline::RunNaiveSparseStep / RunDenseStep (through oracle/ref_shim.cpp)
and stores the selected ids, scores, outputs and a SHA-256 of every input
array.  Tests regenerate the inputs with the oracle's restated generator,
check the hashes, and compare the CUDA path against these outputs -- so the
fixtures pin both the restatement and the GPU result without the reference
being present.
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as o  # noqa: E402

# (name, (num_heads, head_dim, page_size, top_k, batch, min_ctx, max_ctx, seed))
CASES = [
    # tests/test_sparse_cuda.cpp:217-251, :120-132
    ("small", (2, 8, 4, 2, 3, 5, 19, 11)),
    ("ragged", (4, 16, 16, 3, 4, 33, 97, 7)),
    ("wide", (2, 64, 8, 4, 2, 17, 45, 17)),
    ("larger_candidates", (2, 16, 8, 8, 2, 160, 184, 123)),
    # tests/test_reference.cpp:270-290 (sparse == dense when k >= pages)
    ("sparse_eq_dense", (2, 8, 4, 64, 3, 12, 12, 123)),
    # BASELINE config 1 as `dsd_bench 8 1 1024 1024 7 10 2` runs it, and at 32x128
    ("cfg1_h8d16", (8, 16, 16, 8, 1, 1024, 1024, 7)),
    ("cfg1_h32d128", (32, 128, 16, 8, 1, 1024, 1024, 7)),
    # BASELINE config 2 (`dsd_bench 8 16 512 2048 7 10 2 32 128 16`)
    ("cfg2", (32, 128, 16, 8, 16, 512, 2048, 7)),
    # larger k through the reference's k > 16 regime, CPU rule
    ("k32", (4, 32, 8, 32, 6, 100, 400, 5)),
]

INPUT_FIELDS = ["key_pool", "value_pool", "summaries", "token_counts", "queries",
                "cand_offsets", "cand_ids"]


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# Continuous workload generator (src/continuous_batching.cpp:44-59, :336-381):
# (name, (num_heads, head_dim, requests, arrival_window, min_prompt, max_prompt,
#         min_decode, max_decode, seed), payload hashes?)
CONTINUOUS_CASES = [
    ("cont_small", (2, 4, 20, 10, 3, 9, 1, 4, 7), True),
    ("cont_mid", (4, 8, 48, 16, 17, 80, 2, 12, 11), True),
    # BASELINE config 4 (`dsd_continuous_bench 128 32 64 1024 4096 16 64 7 32 128 16 8`):
    # the spec arrays only (the payloads are ~10.7 GB)
    ("cont_cfg4", (32, 128, 128, 64, 1024, 4096, 16, 64, 7), False),
]
# DeterministicTokenVector(count, request, decode_step, stream)
TOKEN_CASES = [(4096, 0, 1, 0), (4096, 5, 0, 1), (4096, 127, 63, 2), (128, 3, 7, 0),
               (4096, 1000, 255, 1)]
SPEC_FIELDS = ["request_ids", "arrival_steps", "prompt_tokens", "decode_steps"]
PAYLOAD_FIELDS = ["prompt_keys", "prompt_values", "initial_queries"]


def make_continuous():
    out = {}
    for name, cfg, payloads in CONTINUOUS_CASES:
        w = o.ref_continuous_workload(*cfg, with_payloads=payloads)
        out[f"{name}_config"] = np.array(cfg, np.int64)
        for f in SPEC_FIELDS:
            out[f"{name}_{f}"] = w[f]
        if payloads:
            for f in PAYLOAD_FIELDS:
                out[f"{name}_sha256_{f}"] = np.array(digest(w[f]))
        print(f"{name}: {len(w['request_ids'])} requests, "
              f"{int(w['prompt_tokens'].sum())} prompt tokens")
    out["tokens_cases"] = np.array(TOKEN_CASES, np.int64)
    out["tokens_sha256"] = np.array([digest(o.ref_deterministic_token_vector(*t))
                                     for t in TOKEN_CASES])
    np.savez_compressed(os.path.join(HERE, "continuous_workload.npz"), **out)


def main():
    if not o.ref_available():
        o.build(with_reference=True)
    make_continuous()
    for name, cfg in CASES:
        rb = o.RefBatch(*cfg)
        b = rb.export()
        sel, so, out, scores = rb.sparse_cpu()
        dense = rb.dense_cpu()
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            config=np.array(cfg, np.int64), selected=sel, selected_offsets=so, outputs=out,
            scores=scores, dense_outputs=dense,
            **{f"sha256_{f}": np.array(digest(getattr(b, f))) for f in INPUT_FIELDS})
        rb.close()
        print(f"{name}: pages={b.capacity} candidates={len(b.cand_ids)} selected={len(sel)}")


if __name__ == "__main__":
    main()
