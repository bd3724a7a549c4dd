"""The CLIs print what the reference's experiment scripts parse (GPU).

experiment/common.sh builds its CSVs with three lookups on the raw logs:
`kv_from_file` (a `key=value` line), `token_kv_from_file` (a `key=value`
token anywhere on a line) and `section_table_value_from_file` (column N of a
row inside a `== Section ==` block).  They are restated here and applied to
every field the reference's decode and continuous CSV rows read.
"""
import os
import subprocess

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu
BIN = os.path.join(ROOT, "15-618_dynamic_sparse_decode_b200", "bin")


def kv(text, key):
    for line in text.splitlines():
        k, sep, v = line.partition("=")
        if sep and k == key:
            return v
    return None


def token_kv(text, key):
    for line in text.splitlines():
        for tok in line.split():
            k, sep, v = tok.partition("=")
            if sep and k == key:
                return v
    return None


def section_value(text, section, row, col):
    inside = False
    for line in text.splitlines():
        if line == section:
            inside = True
            continue
        if inside and line.startswith("== "):
            return None
        f = line.split()
        if inside and f and f[0] == row:
            return f[col - 1] if len(f) >= col else None
    return None


def is_number(s):
    try:
        float(s)
        return True
    except (TypeError, ValueError):
        return False


def test_dsd_bench_fields_parse():
    out = subprocess.run([os.path.join(BIN, "dsd_bench"), "4", "4", "64", "256", "7", "2", "1",
                          "8", "32", "16"], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr
    t = out.stdout
    for key in ["top_k_pages", "batch_size", "min_ctx", "max_ctx", "seed", "iterations", "warmup",
                "num_heads", "head_dim", "page_size", "total_pages", "total_context_tokens",
                "total_candidate_pages", "total_selected_tokens",
                "sparse_current_over_dense_bytes", "sparse_target_over_dense_bytes"]:
        assert is_number(token_kv(t, key)), key
    for section, row, col in [("== End-to-End ==", "dense_cpu", 2), ("== End-to-End ==", "sparse_cpu", 2),
                              ("== End-to-End ==", "dense_gpu", 2), ("== End-to-End ==", "sparse_gpu", 2),
                              ("== End-to-End ==", "sparse_gpu", 3),
                              ("== Stage / Kernel Breakdown ==", "dense_gpu", 6),
                              ("== Stage / Kernel Breakdown ==", "sparse_gpu", 6),
                              ("== Stage / Kernel Breakdown ==", "sparse_gpu", 2),
                              ("== Stage / Kernel Breakdown ==", "sparse_gpu", 3),
                              ("== Stage / Kernel Breakdown ==", "sparse_gpu", 5),
                              ("== Runtime Overheads ==", "sparse_gpu", 9),
                              ("== Runtime Overheads ==", "sparse_gpu", 8)]:
        assert is_number(section_value(t, section, row, col)), (section, row, col)
    assert float(section_value(t, "== End-to-End ==", "sparse_gpu", 2)) > 0
    assert is_number(kv(t, "avg_max_abs_diff_sparse_gpu_vs_dense_cpu"))
    assert kv(t, "sparse_gpu_selection_exact") == "1"


def test_dsd_continuous_bench_fields_parse():
    out = subprocess.run([os.path.join(BIN, "dsd_continuous_bench"), "10", "4", "8", "40", "120", "3",
                          "9", "7", "4", "16", "8", "3", "1", "0", "0", "0", "0", "1", "1"],
                         capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr
    t = out.stdout
    for key in ["num_requests", "max_active_requests", "arrival_window", "min_prompt_tokens",
                "max_prompt_tokens", "min_decode_steps", "max_decode_steps", "seed", "num_heads",
                "head_dim", "page_size", "top_k_pages", "total_generated_tokens",
                "continuous_vs_serial_speedup"]:
        assert is_number(kv(t, key)), key
    for key in ["admission_mode", "run_batch_output_mode", "run_batch_timing_mode"]:
        assert kv(t, key), key
    for prefix in ["continuous_sparse", "serial_sparse"]:
        for field in ["tokens_per_second", "avg_active_batch_size", "avg_step_ms", "p95_step_ms",
                      "total_ms", "measured_end_to_end_ms", "decode_payload_prep_ms",
                      "prompt_preadmit_ms", "runtime_admission_ms", "run_batch_wall_ms",
                      "append_sync_ms", "release_sync_ms", "serving_loop_other_ms",
                      "outside_run_batch_ms", "admission_ms", "avg_score_ms", "avg_topk_ms",
                      "avg_gather_ms", "avg_attention_ms", "avg_kernel_ms", "avg_h2d_ms",
                      "avg_d2h_ms", "avg_launch_ms", "avg_sync_ms", "avg_prepare_sparse_layout_ms"]:
            assert is_number(kv(t, f"{prefix}_{field}")), f"{prefix}_{field}"
