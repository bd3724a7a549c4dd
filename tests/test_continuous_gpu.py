"""Continuous-batching step on the device vs the oracle, every step (GPU).

The serving loop of the reference (src/continuous_batching.cpp:497-696, direct
GPU upload admission) is driven through the C ABI: prompts uploaded into
LIFO-allocated pages with summaries computed on the device, one decode step
per active request over the DEVICE request page tables, the new K/V token
appended on the device (running-mean summary, a fresh page on the first
decoded token), finished requests released.  A host mirror of the pool runs
the same operations with the oracle's formulas and decodes every step with
the oracle: selected ids equal in order, scores bit for bit, outputs <= 1e-4.
Inputs come from the reference's own generators (restated in the oracle).
"""
import numpy as np
import pytest

from oracle import oracle as o

pytestmark = pytest.mark.gpu


class HostMirror:
    """PagePool + PagedKvCache bookkeeping with flat pools (oracle formulas)."""

    def __init__(self, cap, P, E, kv_format=0):
        # the rounding the context's page format applies on store
        self.rnd = o.stored_round(kv_format)
        self.free = list(range(cap))           # pops from the back: LIFO
        self.kp = np.zeros((cap, P, E), np.float32)
        self.vp = np.zeros((cap, P, E), np.float32)
        self.summ = np.zeros((cap, E), np.float32)
        self.tc = np.zeros(cap, np.int32)
        self.pages = {}
        self.P = P

    def reserve(self, rid, counts):
        ids = sorted(self.free.pop() for _ in counts)   # ReservePagesForRequest sorts ids
        self.pages.setdefault(rid, []).extend(ids)
        return ids

    def append_token(self, rid, key, value, force_new):
        pages = self.pages.setdefault(rid, [])
        if force_new or not pages or self.tc[pages[-1]] >= self.P:
            pid = self.free.pop()
            self.summ[pid] = 0
            self.tc[pid] = 0
            pages.append(pid)
            new = True
        else:
            pid = pages[-1]
            new = False
        off = int(self.tc[pid])
        key = self.rnd(key)
        self.kp[pid, off] = key
        self.vp[pid, off] = self.rnd(value)
        self.summ[pid] = self.rnd(o.running_mean_append(self.summ[pid], key, off))
        self.tc[pid] = off + 1
        return pid, off, new

    def release(self, rid):
        ids = self.pages.pop(rid, [])
        for pid in ids:
            self.summ[pid] = 0
            self.tc[pid] = 0
            self.free.append(pid)
        return ids


def run_continuous(dsd, H, D, P, K, n_req, max_active, window, pmin, pmax, dmin, dmax, seed,
                   split_step=False, depth=1, kv_format=0):
    E = H * D
    w = o.continuous_workload(H, D, n_req, window, pmin, pmax, dmin, dmax, seed)
    ids, arr, pt, ds = w["request_ids"], w["arrival_steps"], w["prompt_tokens"], w["decode_steps"]
    offs = np.concatenate([[0], np.cumsum(pt)])
    pages_for = lambda t: (t + P - 1) // P
    max_pages = int(max(pages_for(int(a)) + pages_for(int(b)) for a, b in zip(pt, ds)))
    cap = min(int(sum(pages_for(int(a)) + pages_for(int(b)) for a, b in zip(pt, ds))),
              max_active * max_pages)
    host = HostMirror(cap, P, E, kv_format)
    ctx = dsd.SparseDecodeContext(H, D, P, K, cap, max_active, max_active * max_pages,
                                  max_active * min(K, max_pages), max_requests=max_active,
                                  max_pages_per_request=max_pages, kv_format=kv_format)
    active = []            # dicts: rid, remaining, step, query
    nxt, step, checked = 0, 0, 0
    inflight = []          # oracle results of steps begun but not yet ended

    def end_oldest():
        res = ctx.decode_step_end()
        sel, out, scores, at = inflight.pop(0)
        assert np.array_equal(res["scores"].view(np.uint32), scores.view(np.uint32)), at
        assert np.array_equal(res["selected"], sel), at
        assert float(np.abs(res["outputs"] - out).max()) <= 1e-4, at
    order = list(range(n_req))
    pending = []
    while nxt < n_req or pending or active:
        if not active and not pending and nxt < n_req and step < arr[nxt]:
            step = int(arr[nxt])
        while nxt < n_req and arr[nxt] <= step:
            pending.append(order[nxt]); nxt += 1
        while len(active) < max_active and pending:
            i = pending.pop(0)
            rid, n_tok = int(ids[i]), int(pt[i])
            counts = [min(P, n_tok - t) for t in range(0, n_tok, P)]
            pids = host.reserve(rid, counts)
            keys = w["prompt_keys"][offs[i]:offs[i + 1]]
            vals = w["prompt_values"][offs[i]:offs[i + 1]]
            t0 = 0
            for pid, c in zip(pids, counts):
                host.kp[pid, :c] = host.rnd(keys[t0:t0 + c])
                host.vp[pid, :c] = host.rnd(vals[t0:t0 + c])
                host.summ[pid] = host.rnd(o.page_summary(host.kp[pid, :c]))
                host.tc[pid] = c
                t0 += c
            ctx.upload_pages(pids, counts, keys, vals)
            ctx.set_request_pages(rid, pids)
            if ds[i] > 0:
                active.append(dict(rid=rid, remaining=int(ds[i]), step=0,
                                   query=w["initial_queries"][i].copy()))
            else:
                ctx.release_request(rid, free_pages=True)
                host.release(rid)
        if not active:
            step += 1
            continue
        rids = np.array([a["rid"] for a in active], np.int32)
        q = np.stack([a["query"] for a in active])
        if split_step:
            ctx.decode_step_begin(rids, q, output_mode=dsd.OUTPUT_DEBUG)
        else:
            res = ctx.decode_step(rids, q, output_mode=dsd.OUTPUT_DEBUG)
        cand = [np.array(host.pages[a["rid"]], np.int32) for a in active]
        b = o.Batch(H, D, P, K, host.kp, host.vp, host.summ, host.tc, q,
                    np.concatenate([[0], np.cumsum([len(c) for c in cand])]).astype(np.int32),
                    np.concatenate(cand))
        sel, so, out, scores = o.sparse_decode(b)
        if split_step:
            inflight.append((sel, out, scores, step))
        else:
            assert np.array_equal(res["scores"].view(np.uint32), scores.view(np.uint32)), step
            assert np.array_equal(res["selected"], sel), step
            assert float(np.abs(res["outputs"] - out).max()) <= 1e-4, step
        checked += 1
        # append this step's token (the last step's token is never uploaded)
        up_p, up_o, up_r, up_k, up_v = [], [], [], [], []
        for a in active:
            k = o.deterministic_token_vector(E, a["rid"], a["step"], 1)
            v = o.deterministic_token_vector(E, a["rid"], a["step"], 2)
            pid, off, new = host.append_token(a["rid"], k, v, a["step"] == 0)
            if a["remaining"] > 1:
                up_p.append(pid); up_o.append(off); up_r.append(a["rid"])
                up_k.append(k); up_v.append(v)
            a["query"] = o.deterministic_token_vector(E, a["rid"], a["step"] + 1, 0)
            a["step"] += 1
            a["remaining"] -= 1
        if up_p:
            ctx.append_tokens(up_p, up_o, np.stack(up_k), np.stack(up_v), request_ids=up_r)
        if split_step and len(inflight) >= depth:
            # the appends (and, at depth 2, the next step) were queued while the
            # step was pending: it must not see them
            end_oldest()
        for a in [a for a in active if a["remaining"] == 0]:
            ctx.release_request(a["rid"], free_pages=True)
            host.release(a["rid"])
        active = [a for a in active if a["remaining"] > 0]
        step += 1
    while inflight:
        end_oldest()
    ctx.close()
    return checked


@pytest.mark.parametrize("split_step,depth", [(False, 1), (True, 1), (True, 2)],
                         ids=["sync_step", "begin_end_step", "two_steps_in_flight"])
def test_continuous_small_shapes(dsd, split_step, depth):
    assert run_continuous(dsd, 4, 16, 8, 3, 10, 4, 6, 20, 60, 3, 10, 7, split_step, depth) > 5


def test_continuous_config4_shape(dsd):
    # BASELINE config 4 shape (H32 D128 P16 k8, prompts 1024-4096) with fewer
    # requests and decode steps so the host oracle stays in seconds
    assert run_continuous(dsd, 32, 128, 16, 8, 12, 6, 8, 1024, 4096, 4, 10, 7) > 5
