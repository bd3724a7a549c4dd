"""B200-native batched page-level dynamic sparse decode.

The product is the C ABI in ``include/dsd_b200.h`` (``libdsd_b200.so``, built
from ``csrc/``) and the C++ drop-in host API over it.  This module is the
ctypes binding the tests and ``bench.py`` use.  It loads the in-tree library
and fails loudly when it is missing: there is no CPU fallback.

The directory name is not a Python identifier, so import it with
``importlib.import_module("15-618_dynamic_sparse_decode_b200")`` after
putting the repository root on ``sys.path``.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libdsd_b200.so")

DSD_OK, DSD_EINVAL, DSD_ERANGE, DSD_ENOMEM, DSD_ECUDA, DSD_ETIMEOUT, DSD_EUNAVAILABLE = range(7)
OUTPUT_NONE, OUTPUT_OUTPUTS, OUTPUT_DEBUG = 0, 1, 2
KV_F32, KV_BF16, KV_FP8 = 0, 1, 2

_I32P = ctypes.POINTER(ctypes.c_int32)
_F32P = ctypes.POINTER(ctypes.c_float)
_VP = ctypes.c_void_p


class ModelConfig(ctypes.Structure):
    """dsd_model_config == the reference's ModelConfig (include/dsd/config.h:5-10)."""
    _fields_ = [("num_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("page_size", ctypes.c_int32), ("top_k_pages", ctypes.c_int32)]


class CtxOptions(ctypes.Structure):
    _fields_ = [("capacity_pages", ctypes.c_int32), ("max_batch", ctypes.c_int32),
                ("max_candidates", ctypes.c_int32), ("max_selected", ctypes.c_int32),
                ("max_requests", ctypes.c_int32), ("max_pages_per_request", ctypes.c_int32)]


class StepTiming(ctypes.Structure):
    _fields_ = [("score_ms", ctypes.c_float), ("topk_ms", ctypes.c_float),
                ("attention_ms", ctypes.c_float), ("total_ms", ctypes.c_float)]


class TransferStats(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in
                ("h2d_bytes", "d2h_bytes", "h2d_calls", "d2h_calls", "h2d_large_calls",
                 "d2h_large_calls")]


# (name, restype, argtypes) of every exported entry point, in header order.
SIGNATURES = [
    ("dsd_last_error", ctypes.c_char_p, []),
    ("dsd_available", ctypes.c_int, []),
    ("dsd_ctx_create", ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ModelConfig),
                                      ctypes.POINTER(CtxOptions), ctypes.POINTER(_VP)]),
    ("dsd_ctx_destroy", ctypes.c_int, [_VP]),
    ("dsd_ctx_create_ex", ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ModelConfig),
                                         ctypes.POINTER(CtxOptions), ctypes.c_int,
                                         ctypes.POINTER(_VP)]),
    ("dsd_ctx_kv_format", ctypes.c_int, [_VP]),
    ("dsd_ctx_device_pointers", ctypes.c_int, [_VP, ctypes.POINTER(_VP), ctypes.POINTER(_VP),
                                               ctypes.POINTER(_VP), ctypes.POINTER(_VP)]),
    ("dsd_ctx_stream", _VP, [_VP]),
    ("dsd_step_host_buffers", ctypes.c_int, [_VP, ctypes.POINTER(_VP), ctypes.POINTER(_VP)]),
    ("dsd_step_staging_wait", ctypes.c_int, [_VP]),
    ("dsd_pool_reset", ctypes.c_int, [_VP]),
    ("dsd_pool_upload_pages", ctypes.c_int, [_VP, _I32P, _I32P, ctypes.c_int, _F32P, _F32P,
                                             ctypes.c_int]),
    ("dsd_pool_upload_summaries", ctypes.c_int, [_VP, _I32P, ctypes.c_int, _F32P]),
    ("dsd_pool_prefill_synthetic", ctypes.c_int, [_VP, _I32P, _I32P, ctypes.c_int, ctypes.c_int]),
    ("dsd_pool_generate_normal", ctypes.c_int, [_VP, _I32P, _I32P, _I32P, _I32P, ctypes.c_int,
                                                ctypes.c_uint64]),
    ("dsd_generate_normal_host", None, [ctypes.c_uint64, ctypes.c_int, ctypes.c_uint64,
                                        ctypes.c_int64, _F32P]),
    ("dsd_append_tokens", ctypes.c_int, [_VP, _I32P, _I32P, _I32P, ctypes.c_int, _F32P, _F32P]),
    ("dsd_append_tokens_synthetic", ctypes.c_int, [_VP, _I32P, _I32P, _I32P, _I32P,
                                                   ctypes.c_int]),
    ("dsd_pool_free_pages", ctypes.c_int, [_VP, _I32P, ctypes.c_int]),
    ("dsd_download_page", ctypes.c_int, [_VP, ctypes.c_int, _F32P, _F32P, _F32P, _I32P]),
    ("dsd_download_metadata", ctypes.c_int, [_VP, _I32P, ctypes.POINTER(ctypes.c_uint8)]),
    ("dsd_get_transfer_stats", ctypes.c_int, [_VP, ctypes.POINTER(TransferStats)]),
    ("dsd_reset_transfer_stats", ctypes.c_int, [_VP]),
    ("dsd_decode_batch", ctypes.c_int, [_VP, ctypes.c_int, _F32P, _I32P, _I32P, ctypes.c_int,
                                        ctypes.c_int, _F32P, _F32P, _I32P,
                                        ctypes.POINTER(StepTiming)]),
    ("dsd_request_set_pages", ctypes.c_int, [_VP, ctypes.c_int, _I32P, ctypes.c_int]),
    ("dsd_request_append_pages", ctypes.c_int, [_VP, ctypes.c_int, _I32P, ctypes.c_int]),
    ("dsd_request_append_pages_multi", ctypes.c_int, [_VP, _I32P, _I32P, ctypes.c_int]),
    ("dsd_request_release", ctypes.c_int, [_VP, ctypes.c_int, ctypes.c_int]),
    ("dsd_request_num_pages", ctypes.c_int, [_VP, ctypes.c_int]),
    ("dsd_decode_step", ctypes.c_int, [_VP, _I32P, ctypes.c_int, _F32P, ctypes.c_int,
                                       ctypes.c_int, _F32P, _F32P, _I32P,
                                       ctypes.POINTER(StepTiming)]),
    ("dsd_decode_step_begin", ctypes.c_int, [_VP, _I32P, ctypes.c_int, _F32P, ctypes.c_int,
                                             ctypes.c_int]),
    ("dsd_decode_step_end", ctypes.c_int, [_VP, _F32P, _F32P, _I32P, ctypes.POINTER(StepTiming)]),
    ("dsd_bind_requests", ctypes.c_int, [_VP, _I32P, ctypes.c_int]),
    ("dsd_decode_bound", ctypes.c_int, [_VP, _VP, _VP]),
    ("dsd_decode_bound_timed", ctypes.c_int, [_VP, _VP, _VP, ctypes.POINTER(StepTiming)]),
    ("dsd_read_step_timing", ctypes.c_int, [_VP, ctypes.POINTER(StepTiming)]),
    ("dsd_set_attention_mode", ctypes.c_int, [_VP, ctypes.c_int]),
    ("dsd_kernels_per_step", ctypes.c_int, []),
    ("dsd_selftest_bounded_wait", ctypes.c_int, [_VP, ctypes.c_int64]),
    ("dsd_decode_batch_noalloc", ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ModelConfig),
                                                ctypes.c_int, ctypes.c_int, _I32P, _VP, _VP,
                                                _VP, _VP, _VP, _VP, _VP, _VP]),
]

_lib = None


def load_library(path: str = LIB_PATH):
    """Loads libdsd_b200.so.  Raises if it has not been built: no fallback."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(
            f"{path} is missing; build it with `python {PKG_DIR}/build.py` "
            "(the sparse decode path has no CPU fallback)")
    lib = ctypes.CDLL(path)
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class DsdError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class InvalidArgument(DsdError, ValueError):
    """std::invalid_argument in the reference."""


class OutOfRange(DsdError, IndexError):
    """std::out_of_range in the reference."""


def _check(rc: int) -> None:
    if rc == DSD_OK:
        return
    msg = _lib.dsd_last_error().decode()
    if rc == DSD_EINVAL:
        raise InvalidArgument(rc, msg)
    if rc == DSD_ERANGE:
        raise OutOfRange(rc, msg)
    raise DsdError(rc, msg)


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _ip(a):
    return None if a is None else a.ctypes.data_as(_I32P)


def _fp(a):
    return None if a is None else a.ctypes.data_as(_F32P)


def _out_buffer(out, rows, cols):
    """A caller-supplied result buffer: C-contiguous float32 with room for
    rows x cols values (the library writes exactly that many)."""
    if not (isinstance(out, np.ndarray) and out.dtype == np.float32 and
            out.flags["C_CONTIGUOUS"] and out.size >= rows * cols):
        raise InvalidArgument(int(DSD_EINVAL),
                              f"out must be a C-contiguous float32 array of at least "
                              f"{rows}x{cols} values")
    return out


def available() -> bool:
    return bool(load_library().dsd_available())


def generate_normal_host(seed: int, kind: int, first_index: int, count: int) -> np.ndarray:
    out = np.empty(count, np.float32)
    load_library().dsd_generate_normal_host(seed, kind, first_index, count, _fp(out))
    return out


def normal_index(request: int, token: int, ept: int, element: int = 0) -> int:
    return (request << 40) + token * ept + element


class SparseDecodeContext:
    """One GPU's page pool + decode step (SparseCudaContext over the C ABI)."""

    def __init__(self, num_heads, head_dim, page_size, top_k_pages, capacity_pages, max_batch,
                 max_candidates, max_selected, max_requests=0, max_pages_per_request=0,
                 device=0, kv_format=KV_F32):
        """kv_format: KV_F32 (the reference's fp32 pages), KV_BF16 or KV_FP8
        (pages and summaries stored as bf16 / fp8 e4m3, arithmetic in fp32;
        payloads in and downloads out stay float32 arrays)."""
        self.lib = load_library()
        self.cfg = ModelConfig(num_heads, head_dim, page_size, top_k_pages)
        self.opt = CtxOptions(capacity_pages, max_batch, max_candidates, max_selected,
                              max_requests, max_pages_per_request)
        self.ept = num_heads * head_dim
        h = _VP()
        _check(self.lib.dsd_ctx_create_ex(device, ctypes.byref(self.cfg), ctypes.byref(self.opt),
                                          int(kv_format), ctypes.byref(h)))
        self.h = h
        self.kv_format = int(kv_format)

    def close(self):
        if getattr(self, "h", None):
            self.lib.dsd_ctx_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- pool
    def device_pointers(self):
        k, v, s, c = _VP(), _VP(), _VP(), _VP()
        _check(self.lib.dsd_ctx_device_pointers(self.h, ctypes.byref(k), ctypes.byref(v),
                                                ctypes.byref(s), ctypes.byref(c)))
        return k.value, v.value, s.value, c.value

    def stream(self) -> int:
        return self.lib.dsd_ctx_stream(self.h)

    def reset(self):
        _check(self.lib.dsd_pool_reset(self.h))

    def upload_pages(self, page_ids, token_counts, keys, values, compute_summary=True):
        ids, cnt = _i32(page_ids), _i32(token_counts)
        k, v = _f32(keys), _f32(values)
        _check(self.lib.dsd_pool_upload_pages(self.h, _ip(ids), _ip(cnt), len(ids), _fp(k), _fp(v),
                                              int(compute_summary)))

    def upload_pool(self, key_pool, value_pool, token_counts, pages=None):
        """Uploads pages of flat [cap][P][E] host pools (every page with tokens by default)."""
        tc = np.asarray(token_counts)
        pages = np.nonzero(tc > 0)[0] if pages is None else np.asarray(pages)
        if len(pages) == 0:
            return
        keys = np.concatenate([key_pool[p, : tc[p]] for p in pages])
        vals = np.concatenate([value_pool[p, : tc[p]] for p in pages])
        self.upload_pages(pages, tc[pages], keys, vals)

    def upload_summaries(self, page_ids, summaries):
        ids, s = _i32(page_ids), _f32(summaries)
        _check(self.lib.dsd_pool_upload_summaries(self.h, _ip(ids), len(ids), _fp(s)))

    def prefill_synthetic(self, page_ids, token_counts, request_id):
        ids, cnt = _i32(page_ids), _i32(token_counts)
        _check(self.lib.dsd_pool_prefill_synthetic(self.h, _ip(ids), _ip(cnt), len(ids),
                                                   request_id))

    def generate_normal(self, page_ids, token_counts, request_ids, first_token, seed):
        a = [_i32(x) for x in (page_ids, token_counts, request_ids, first_token)]
        _check(self.lib.dsd_pool_generate_normal(self.h, *[_ip(x) for x in a], len(a[0]), seed))

    def append_tokens(self, page_ids, token_offsets, keys, values, request_ids=None):
        ids, off = _i32(page_ids), _i32(token_offsets)
        req = None if request_ids is None else _i32(request_ids)
        k, v = _f32(keys), _f32(values)
        _check(self.lib.dsd_append_tokens(self.h, _ip(ids), _ip(off), _ip(req), len(ids), _fp(k),
                                          _fp(v)))

    def append_tokens_synthetic(self, page_ids, token_offsets, request_ids, decode_steps):
        a = [_i32(x) for x in (page_ids, token_offsets, request_ids, decode_steps)]
        _check(self.lib.dsd_append_tokens_synthetic(self.h, *[_ip(x) for x in a], len(a[0])))

    def free_pages(self, page_ids):
        ids = _i32(page_ids)
        _check(self.lib.dsd_pool_free_pages(self.h, _ip(ids), len(ids)))

    def download_page(self, page_id):
        P, E = self.cfg.page_size, self.ept
        k = np.empty((P, E), np.float32)
        v = np.empty((P, E), np.float32)
        s = np.empty(E, np.float32)
        n = np.zeros(1, np.int32)
        _check(self.lib.dsd_download_page(self.h, page_id, _fp(k), _fp(v), _fp(s), _ip(n)))
        return k, v, s, int(n[0])

    def download_metadata(self):
        cap = self.opt.capacity_pages
        tc = np.empty(cap, np.int32)
        live = np.empty(cap, np.uint8)
        _check(self.lib.dsd_download_metadata(self.h, _ip(tc),
                                              live.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8))))
        return tc, live

    def transfer_stats(self) -> dict:
        st = TransferStats()
        _check(self.lib.dsd_get_transfer_stats(self.h, ctypes.byref(st)))
        return {n: getattr(st, n) for n, _ in TransferStats._fields_}

    def reset_transfer_stats(self):
        _check(self.lib.dsd_reset_transfer_stats(self.h))

    # ---- decode
    def _results(self, batch, total_cand, total_sel, output_mode, alloc_out=True):
        out = np.zeros((batch, self.ept), np.float32) if alloc_out else None
        scores = np.zeros(max(1, total_cand), np.float32) if output_mode == OUTPUT_DEBUG else None
        sel = np.zeros(max(1, total_sel), np.int32) if output_mode == OUTPUT_DEBUG else None
        return out, scores, sel

    def set_dense(self, dense: bool):
        """Dense baseline: later steps attend over every candidate page."""
        _check(self.lib.dsd_set_attention_mode(self.h, int(dense)))
        self.dense = bool(dense)

    def decode_batch(self, queries, cand_offsets, cand_ids, output_mode=OUTPUT_DEBUG, timing=False):
        """RunBatch with explicit candidates.  Returns dict(outputs, scores, selected, timing)."""
        q = _f32(queries)
        offs, ids = _i32(cand_offsets), _i32(cand_ids)
        B = len(offs) - 1
        n = np.diff(offs)
        total_sel = int(n.sum() if getattr(self, "dense", False)
                        else np.minimum(n, self.cfg.top_k_pages).clip(0).sum())
        out, scores, sel = self._results(B, int(offs[-1]) if B > 0 else 0, total_sel, output_mode)
        t = StepTiming()
        _check(self.lib.dsd_decode_batch(self.h, B, _fp(q), _ip(offs), _ip(ids), output_mode,
                                         int(timing), _fp(out), _fp(scores), _ip(sel),
                                         ctypes.byref(t)))
        return dict(outputs=out,
                    scores=None if scores is None else scores[: int(offs[-1])],
                    selected=None if sel is None else sel[:total_sel],
                    timing={n: getattr(t, n) for n, _ in StepTiming._fields_})

    def set_request_pages(self, request_id, page_ids):
        ids = _i32(page_ids)
        _check(self.lib.dsd_request_set_pages(self.h, request_id, _ip(ids), len(ids)))

    def append_request_pages(self, request_id, page_ids):
        ids = _i32(page_ids)
        _check(self.lib.dsd_request_append_pages(self.h, request_id, _ip(ids), len(ids)))

    def append_request_pages_multi(self, request_ids, page_ids):
        """page_ids[i] joins request_ids[i]'s page table, in order, one upload."""
        reqs, ids = _i32(request_ids), _i32(page_ids)
        if len(reqs) != len(ids):
            raise InvalidArgument(int(DSD_EINVAL), "one request id per page")
        _check(self.lib.dsd_request_append_pages_multi(self.h, _ip(reqs), _ip(ids), len(ids)))

    def release_request(self, request_id, free_pages=True):
        _check(self.lib.dsd_request_release(self.h, request_id, int(free_pages)))

    def request_num_pages(self, request_id) -> int:
        return self.lib.dsd_request_num_pages(self.h, request_id)

    def decode_step(self, request_ids, queries, output_mode=OUTPUT_DEBUG, timing=False,
                    out=None):
        req = _i32(request_ids)
        q = _f32(queries)
        B = len(req)
        if output_mode == OUTPUT_DEBUG:
            n = np.array([self.request_num_pages(int(r)) for r in req])
            total_sel = int(np.minimum(n, self.cfg.top_k_pages).sum())
            out, scores, sel = self._results(B, int(n.sum()), total_sel, output_mode)
        else:
            n = np.zeros(1, np.int64)
            total_sel = 0
            scores = sel = None
            out = (np.zeros((B, self.ept), np.float32) if out is None
                   else _out_buffer(out, B, self.ept))
        t = StepTiming()
        _check(self.lib.dsd_decode_step(self.h, _ip(req), B, _fp(q), output_mode, int(timing),
                                        _fp(out), _fp(scores), _ip(sel), ctypes.byref(t)))
        return dict(outputs=out,
                    scores=None if scores is None else scores[: int(n.sum())],
                    selected=None if sel is None else sel[:total_sel],
                    timing={n_: getattr(t, n_) for n_, _ in StepTiming._fields_})

    def decode_step_begin(self, request_ids, queries, output_mode=OUTPUT_OUTPUTS):
        req, q = _i32(request_ids), _f32(queries)
        if not hasattr(self, "_pending"):
            self._pending = []
        # page counts size the debug results; other modes need none
        n = (np.array([self.request_num_pages(int(r)) for r in req])
             if output_mode == OUTPUT_DEBUG else np.zeros(1, np.int64))
        _check(self.lib.dsd_decode_step_begin(self.h, _ip(req), len(req), _fp(q), output_mode, 0))
        self._pending.append((len(req), output_mode, n))

    def decode_step_end(self, out=None):
        """Waits for the oldest pending step; `out` (float32 [B][H*D]) receives
        its outputs when given, else a new array does."""
        B, mode, n = self._pending.pop(0)
        total_sel = int(np.minimum(n, self.cfg.top_k_pages).sum())
        res_out, scores, sel = self._results(B, int(n.sum()), total_sel, mode,
                                             alloc_out=out is None)
        out = res_out if out is None else _out_buffer(out, B, self.ept)
        _check(self.lib.dsd_decode_step_end(self.h, _fp(out), _fp(scores), _ip(sel), None))
        return dict(outputs=out, scores=None if scores is None else scores[: int(n.sum())],
                    selected=None if sel is None else sel[:total_sel])

    def bind_requests(self, request_ids):
        req = _i32(request_ids)
        _check(self.lib.dsd_bind_requests(self.h, _ip(req), len(req)))

    def decode_bound(self, d_queries: int, d_outputs: int):
        _check(self.lib.dsd_decode_bound(self.h, _VP(d_queries), _VP(d_outputs)))

    def decode_bound_timed(self, d_queries: int, d_outputs: int, wait: bool = True):
        """Timed graph replay; wait=False queues it and returns None (see read_step_timing)."""
        t = StepTiming()
        _check(self.lib.dsd_decode_bound_timed(self.h, _VP(d_queries), _VP(d_outputs),
                                               ctypes.byref(t) if wait else None))
        return {n: getattr(t, n) for n, _ in StepTiming._fields_} if wait else None

    def read_step_timing(self) -> dict:
        t = StepTiming()
        _check(self.lib.dsd_read_step_timing(self.h, ctypes.byref(t)))
        return {n: getattr(t, n) for n, _ in StepTiming._fields_}
