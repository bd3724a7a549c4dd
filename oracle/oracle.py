"""ctypes front end for the CPU checkers (test infrastructure only).

* ``liboracle.so`` -- the restatement of the reference algorithm
  (``oracle/dsd_oracle.cpp``); always available once ``make -C oracle`` ran.
* ``_ref/libdsd_ref.so`` -- the unmodified reference CPU sources plus a flat
  shim (``oracle/ref_shim.cpp``); present where the reference sources were
  available at build time.

Everything here is numpy in / numpy out; nothing touches a GPU.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libdsd_ref.so")

_F = ctypes.POINTER(ctypes.c_float)
_I = ctypes.POINTER(ctypes.c_int)


def reference_root() -> str | None:
    """Where the reference sources are: $REF_ROOT, else the ``reference_path``
    recorded in the repository's BASELINE.json; None when neither exists."""
    root = os.environ.get("REF_ROOT")
    if not root:
        try:
            import json
            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
                root = json.load(f).get("reference_path")
        except (OSError, ValueError):
            root = None
    return root if root and os.path.isdir(os.path.join(root, "src")) else None


def build(with_reference: bool | None = None) -> None:
    """Compile the restatement (and, when the reference sources exist, _ref)."""
    targets = ["oracle"]
    ref_root = reference_root()
    if with_reference is None:
        with_reference = ref_root is not None
    if with_reference:
        if ref_root is None:
            raise RuntimeError("reference sources not found: set REF_ROOT")
        targets += ["ref", "ref_tests"]
    extra = [f"REF_ROOT={ref_root}"] if ref_root else []
    subprocess.run(["make", "-s", "-C", HERE, *extra, *targets], check=True)


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build(with_reference=False)
        L = ctypes.CDLL(LIB_PATH)
        L.orc_page_summary.argtypes = [_F, ctypes.c_int, ctypes.c_int, _F]
        L.orc_running_mean_append.argtypes = [_F, _F, ctypes.c_int, ctypes.c_int]
        L.orc_sparse_decode.argtypes = [ctypes.c_int] * 4 + [_F, _F, _F, _I, ctypes.c_int, _F,
                                                             _I, _I, _I, _F, _F, ctypes.c_int]
        L.orc_dense_decode.argtypes = [ctypes.c_int] * 3 + [_F, _F, _I, ctypes.c_int, _F, _I, _I, _F]
        L.orc_synthetic_batch_contexts.argtypes = [ctypes.c_int] * 5 + [_I]
        L.orc_synthetic_batch_contexts.restype = ctypes.c_int
        L.orc_synthetic_batch_fill.argtypes = [ctypes.c_int] * 7 + [_F, _F, _F, _I, _F, _I, _I]
        L.orc_deterministic_token_vector.argtypes = [ctypes.c_int] * 4 + [_F]
        L.orc_continuous_workload.argtypes = [ctypes.c_int] * 9 + [_I, _I, _I, _I, _F, _F, _F]
        L.orc_continuous_specs_only.argtypes = [ctypes.c_int] * 7 + [_I, _I, _I, _I]
        L.orc_normal_value.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_uint64]
        L.orc_normal_value.restype = ctypes.c_float
        L.orc_normal_fill.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_uint64,
                                      ctypes.c_longlong, _F]
        L.orc_synthetic_prompt_fill.argtypes = [ctypes.c_int] * 5 + [_F]
        L.orc_synthetic_decode_fill.argtypes = [ctypes.c_int] * 4 + [_F]
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_LIB_PATH)


def ref():
    global _ref
    if _ref is None:
        R = ctypes.CDLL(REF_LIB_PATH)
        R.ref_batch_create.argtypes = [ctypes.c_int] * 8
        R.ref_batch_create.restype = ctypes.c_void_p
        R.ref_batch_destroy.argtypes = [ctypes.c_void_p]
        R.ref_batch_capacity.argtypes = [ctypes.c_void_p]
        R.ref_batch_total_candidates.argtypes = [ctypes.c_void_p]
        R.ref_batch_export.argtypes = [ctypes.c_void_p, _F, _F, _F, _I, _F, _I, _I]
        R.ref_batch_sparse_cpu.argtypes = [ctypes.c_void_p, _I, _F, _F]
        R.ref_batch_dense_cpu.argtypes = [ctypes.c_void_p, _F]
        R.ref_batch_time_cpu.argtypes = [ctypes.c_void_p] + [ctypes.c_int] * 3
        R.ref_batch_time_cpu.restype = ctypes.c_double
        R.ref_deterministic_token_vector.argtypes = [ctypes.c_int] * 4 + [_F]
        R.ref_continuous_workload.argtypes = [ctypes.c_int] * 9 + [_I, _I, _I, _I, _F, _F, _F]
        _ref = R
    return _ref


def fp(a):
    return a.ctypes.data_as(_F)


def ip(a):
    return a.ctypes.data_as(_I)


@dataclass
class Batch:
    """A decode batch in the flat layout shared by the oracle and the CUDA path."""
    num_heads: int
    head_dim: int
    page_size: int
    top_k: int
    key_pool: np.ndarray      # [capacity, page_size, E] float32
    value_pool: np.ndarray    # [capacity, page_size, E] float32
    summaries: np.ndarray     # [capacity, E] float32
    token_counts: np.ndarray  # [capacity] int32
    queries: np.ndarray       # [B, E] float32
    cand_offsets: np.ndarray  # [B+1] int32
    cand_ids: np.ndarray      # [C] int32

    @property
    def ept(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def capacity(self) -> int:
        return int(self.token_counts.shape[0])

    @property
    def batch(self) -> int:
        return int(self.queries.shape[0])

    def selected_offsets(self, top_k: int | None = None) -> np.ndarray:
        k = self.top_k if top_k is None else top_k
        n = np.diff(self.cand_offsets)
        return np.concatenate([[0], np.cumsum(np.clip(np.minimum(n, k), 0, None))]).astype(np.int32)


def _empty_batch(h, d, p, k, capacity, batch, total_cand):
    e = h * d
    return Batch(h, d, p, k,
                 np.zeros((capacity, p, e), np.float32), np.zeros((capacity, p, e), np.float32),
                 np.zeros((capacity, e), np.float32), np.zeros(capacity, np.int32),
                 np.zeros((batch, e), np.float32), np.zeros(batch + 1, np.int32),
                 np.zeros(total_cand, np.int32))


def synthetic_batch(num_heads, head_dim, page_size, top_k, batch, min_ctx, max_ctx, seed) -> Batch:
    """BuildSyntheticBatch restated (mt19937 U(-1,1), LIFO page ids)."""
    L = lib()
    ctx = np.zeros(batch, np.int32)
    cap = L.orc_synthetic_batch_contexts(page_size, batch, min_ctx, max_ctx, seed, ip(ctx))
    b = _empty_batch(num_heads, head_dim, page_size, top_k, cap, batch, cap)
    L.orc_synthetic_batch_fill(num_heads, head_dim, page_size, batch, min_ctx, max_ctx, seed,
                               fp(b.key_pool), fp(b.value_pool), fp(b.summaries),
                               ip(b.token_counts), fp(b.queries), ip(b.cand_offsets),
                               ip(b.cand_ids))
    return b


def sparse_decode(b: Batch, top_k: int | None = None, n_threads: int = 1):
    """sparse_cpu over a flat batch.  Returns (selected, sel_offsets, outputs, scores)."""
    k = b.top_k if top_k is None else top_k
    so = b.selected_offsets(k)
    sel = np.zeros(max(1, int(so[-1])), np.int32)
    out = np.zeros((b.batch, b.ept), np.float32)
    scores = np.zeros(max(1, len(b.cand_ids)), np.float32)
    lib().orc_sparse_decode(b.num_heads, b.head_dim, b.page_size, k, fp(b.key_pool),
                            fp(b.value_pool), fp(b.summaries), ip(b.token_counts), b.batch,
                            fp(b.queries), ip(b.cand_offsets), ip(b.cand_ids), ip(sel), fp(out),
                            fp(scores), n_threads)
    return sel[: so[-1]], so, out, scores[: len(b.cand_ids)]


def dense_decode(b: Batch):
    out = np.zeros((b.batch, b.ept), np.float32)
    lib().orc_dense_decode(b.num_heads, b.head_dim, b.page_size, fp(b.key_pool), fp(b.value_pool),
                           ip(b.token_counts), b.batch, fp(b.queries), ip(b.cand_offsets),
                           ip(b.cand_ids), fp(out))
    return out


def page_summary(keys: np.ndarray) -> np.ndarray:
    keys = np.ascontiguousarray(keys, np.float32)
    out = np.zeros(keys.shape[-1], np.float32)
    lib().orc_page_summary(fp(keys), keys.shape[0], keys.shape[-1], fp(out))
    return out


def running_mean_append(summary: np.ndarray, key: np.ndarray, old_count: int) -> np.ndarray:
    s = np.array(summary, np.float32, copy=True)
    key = np.ascontiguousarray(key, np.float32)
    lib().orc_running_mean_append(fp(s), fp(key), old_count, s.shape[0])
    return s


# ---------------------------------------------------------------- bf16 / fp8 page formats
# The opt-in bf16 and fp8 e4m3 page formats have no reference counterpart (the
# reference pool is fp32 only).  Their contract is stated here so the fp32
# oracle can check it: every stored K, V and summary element is the fp32 value
# rounded to nearest even in the format (fp8 saturating at +-448); a page
# summary is AppendPage's fp32 mean of the ROUNDED keys, rounded once; a
# running-mean update applies AppendToken's fp32 formula to the stored mean
# and the rounded key, then rounds.  Scoring and
# attention are the fp32 oracle run over those stored values.

def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even), as float32."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32).reshape(np.shape(a))


def fp8_round(a: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest fp8 e4m3 value (ties to even,
    saturating at +-448; 3 mantissa bits, exponents -6..8, subnormal quantum
    2^-9), as float32."""
    x = np.ascontiguousarray(a, np.float32).astype(np.float64)
    mag = np.abs(x)
    _, e2 = np.frexp(mag)                      # mag = m * 2^e2, m in [0.5, 1)
    q = np.exp2(np.maximum(e2 - 1, -6) - 3)    # spacing of e4m3 values near mag
    r = np.minimum(np.rint(mag / q) * q, 448.0)
    r[mag == 0] = 0.0
    return np.copysign(r, x).astype(np.float32).reshape(np.shape(a))


def stored_round(kv_format: int):
    """The rounding a page format applies on store (0 fp32, 1 bf16, 2 fp8 e4m3)."""
    return {0: lambda v: np.asarray(v, np.float32), 1: bf16_round, 2: fp8_round}[kv_format]


def stored_batch(b: Batch, rnd) -> Batch:
    """The batch as a context with rounding `rnd` on store holds it (pools
    rounded, summaries recomputed from the rounded keys and rounded)."""
    kp = rnd(b.key_pool)
    vp = rnd(b.value_pool)
    summ = np.zeros_like(b.summaries)
    for p in range(b.capacity):
        n = int(b.token_counts[p])
        if n > 0:
            summ[p] = rnd(page_summary(kp[p, :n]))
    return Batch(b.num_heads, b.head_dim, b.page_size, b.top_k, kp, vp, summ,
                 b.token_counts.copy(), b.queries, b.cand_offsets, b.cand_ids)


def page_summary_bf16(keys: np.ndarray) -> np.ndarray:
    return bf16_round(page_summary(bf16_round(keys)))


def running_mean_append_bf16(summary: np.ndarray, key: np.ndarray, old_count: int) -> np.ndarray:
    return bf16_round(running_mean_append(summary, bf16_round(key), old_count))


def bf16_batch(b: Batch) -> Batch:
    """The batch as a bf16-page context stores it; queries and candidates unchanged."""
    return stored_batch(b, bf16_round)


def deterministic_token_vector(count, request_id, decode_step, stream, fn=None) -> np.ndarray:
    """DeterministicTokenVector (src/continuous_batching.cpp:52-59) restated;
    ``fn`` swaps in another implementation with the same C signature."""
    out = np.zeros(count, np.float32)
    (fn or lib().orc_deterministic_token_vector)(count, request_id, decode_step, stream, fp(out))
    return out


def ref_deterministic_token_vector(count, request_id, decode_step, stream) -> np.ndarray:
    """The reference's own DeterministicTokenVector (needs _ref)."""
    return deterministic_token_vector(count, request_id, decode_step, stream,
                                      ref().ref_deterministic_token_vector)


def synthetic_prompt(request, page_idx, n, ept, stream) -> np.ndarray:
    out = np.zeros((n, ept), np.float32)
    lib().orc_synthetic_prompt_fill(request, page_idx, n, ept, stream, fp(out))
    return out


def synthetic_decode(request, step, ept, stream) -> np.ndarray:
    out = np.zeros(ept, np.float32)
    lib().orc_synthetic_decode_fill(request, step, ept, stream, fp(out))
    return out


def normal_fill(seed: int, kind: int, first_index: int, count: int) -> np.ndarray:
    out = np.zeros(count, np.float32)
    lib().orc_normal_fill(seed, kind, first_index, count, fp(out))
    return out


def continuous_workload(num_heads, head_dim, num_requests, arrival_window, min_prompt,
                        max_prompt, min_decode, max_decode, seed, with_payloads=True, fn=None):
    """BuildSyntheticContinuousWorkload (src/continuous_batching.cpp:336-381)
    restated; specs in (arrival, id) order.  ``fn`` swaps in another
    implementation with the same C signature (the reference's, for pinning)."""
    call = fn or lib().orc_continuous_workload
    ids, arr, pt, ds = (np.zeros(num_requests, np.int32) for _ in range(4))
    args = (num_heads, head_dim, num_requests, arrival_window, min_prompt, max_prompt,
            min_decode, max_decode, seed, ip(ids), ip(arr), ip(pt), ip(ds))
    call(*args, None, None, None)    # sizes first
    if not with_payloads:
        return dict(request_ids=ids, arrival_steps=arr, prompt_tokens=pt, decode_steps=ds)
    e = num_heads * head_dim
    total = int(pt.sum())
    pk = np.zeros((total, e), np.float32)
    pv = np.zeros((total, e), np.float32)
    q = np.zeros((num_requests, e), np.float32)
    call(*args, fp(pk), fp(pv), fp(q))
    return dict(request_ids=ids, arrival_steps=arr, prompt_tokens=pt, decode_steps=ds,
                prompt_keys=pk, prompt_values=pv, initial_queries=q)


def continuous_specs_only(num_requests, arrival_window, min_prompt, max_prompt, min_decode,
                          max_decode, seed):
    """The lengths-only spec draws (this build's BuildSyntheticContinuousSpecs)."""
    ids, arr, pt, ds = (np.zeros(num_requests, np.int32) for _ in range(4))
    lib().orc_continuous_specs_only(num_requests, arrival_window, min_prompt, max_prompt,
                                    min_decode, max_decode, seed, ip(ids), ip(arr), ip(pt), ip(ds))
    return dict(request_ids=ids, arrival_steps=arr, prompt_tokens=pt, decode_steps=ds)


def ref_continuous_workload(*args, **kw):
    """The reference's own BuildSyntheticContinuousWorkload (needs _ref)."""
    return continuous_workload(*args, fn=ref().ref_continuous_workload, **kw)


class RefBatch:
    """The reference's own BuildSyntheticBatch + sparse_cpu (needs _ref)."""

    def __init__(self, num_heads, head_dim, page_size, top_k, batch, min_ctx, max_ctx, seed):
        self.R = ref()
        self.h = self.R.ref_batch_create(num_heads, head_dim, page_size, top_k, batch, min_ctx,
                                         max_ctx, seed)
        self.cfg = (num_heads, head_dim, page_size, top_k)
        self.batch = batch

    def close(self):
        if self.h:
            self.R.ref_batch_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def export(self) -> Batch:
        h, d, p, k = self.cfg
        cap = self.R.ref_batch_capacity(self.h)
        c = self.R.ref_batch_total_candidates(self.h)
        b = _empty_batch(h, d, p, k, cap, self.batch, c)
        self.R.ref_batch_export(self.h, fp(b.key_pool), fp(b.value_pool), fp(b.summaries),
                                ip(b.token_counts), fp(b.queries), ip(b.cand_offsets),
                                ip(b.cand_ids))
        return b

    def sparse_cpu(self):
        b = self.export()
        so = b.selected_offsets()
        sel = np.zeros(max(1, int(so[-1])), np.int32)
        out = np.zeros((b.batch, b.ept), np.float32)
        scores = np.zeros(max(1, len(b.cand_ids)), np.float32)
        self.R.ref_batch_sparse_cpu(self.h, ip(sel), fp(out), fp(scores))
        return sel[: so[-1]], so, out, scores[: len(b.cand_ids)]

    def dense_cpu(self):
        out = np.zeros((self.batch, self.cfg[0] * self.cfg[1]), np.float32)
        self.R.ref_batch_dense_cpu(self.h, fp(out))
        return out

    def time_cpu(self, items: int, n_threads: int, dense: bool = False) -> float:
        """Wall ms of `items` reference steps (request i % batch) on n_threads."""
        return self.R.ref_batch_time_cpu(self.h, items, n_threads, int(dense))
