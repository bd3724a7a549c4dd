"""Benchmark of the batched page-level sparse decode step (one JSON line on rank 0).

Workload (the north star's headline): 64 requests per GPU,
context ~ U{16384..32768} tokens (numpy default_rng(7)), 32 heads x 128 dims,
page_size 16, top_k_pages 64, fp32 K/V/Q ~ N(0,1) (Irwin-Hall(4) counter-based
generator, seed 7) generated on the device.  One step = one decode token for
every request: score all candidate pages, select the top 64, attend.

  value  tokens/s with queries and outputs resident in HBM (the step launched
         kernel by kernel on the context stream; CUDA events, max over ranks)
  e2e    tokens/s through the public C ABI call dsd_decode_step with host
         queries in and host outputs out, pinned host buffers (H2D + D2H inside
         the timed region)

--impl reference times the reference's own sparse_cpu code (oracle/_ref) on a
bounded sample of the same workload shape on the host cores.

Multi-GPU: torchrun, one process per GPU.  Weak scaling (default): 64*N
distinct requests, rank g owning the ids with id % N == g (64 per GPU) in its
own page pool; --strong: 64 requests in total dealt the same way.  No
collective on the data path.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, D, P, K_TOP = 32, 128, 16, 64
E = H * D
BATCH = 64
CTX_LO, CTX_HI = 16384, 32768
SEED = 7
CPU_SAMPLE_REQUESTS = 4


def workload_contexts(batch=None, seed=SEED):
    batch = BATCH if batch is None else batch
    return np.random.default_rng(seed).integers(CTX_LO, CTX_HI + 1, size=batch)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (getattr(self, "out", "") or "").splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm, mx, power = float(f[1]), float(f[2]), float(f[3])
            except ValueError:
                continue
            rows.append((sm, power))
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        loaded = [sm for sm, p in rows if p >= 300.0] or [sm for sm, _ in rows]
        return {"sm_mhz": float(np.median(loaded)) if loaded else None,
                "sm_max_mhz": mx or None, "reasons": sorted(reasons), "samples": len(rows),
                "samples_under_load": len([1 for _, p in rows if p >= 300.0])}


def profiled_traffic(kernel):
    """DRAM bytes per launch of `kernel` from the committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", f"{kernel}_kernel_config3.md")
    try:
        for line in open(path):
            if line.startswith("traffic_per_launch="):
                return int(line.split("=")[1])
    except OSError:
        pass
    return None


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ---------------------------------------------------------------- reference arm

def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_sample(steps, warmup, with_dense=True):
    """The reference's own CPU decode paths (oracle/_ref, compiled unchanged)
    on CPU_SAMPLE_REQUESTS requests of the config-3 shape built by the
    reference's BuildSyntheticBatch:
      sparse_cpu on every host thread: each step decodes one request per
                 thread (thread t takes request t mod 4 of the sample; the
                 sample is read-only and shared), `steps` steps timed;
      sparse_cpu on one thread: the 4 requests once each;
      dense_cpu on one thread: one request (every token of its context).
    Falls back to the oracle's restatement ("port") without oracle/_ref."""
    from oracle import oracle as o
    if not o.ref_available():
        o.build()
    kind = "reference" if o.ref_available() else "port"
    threads = host_threads()
    n = CPU_SAMPLE_REQUESTS
    res = {"kind": kind, "cores": threads, "host_logical_cpus": os.cpu_count(),
           "cpu_model": cpu_model()}
    if kind == "reference":
        rb = o.RefBatch(H, D, P, K_TOP, n, CTX_LO, CTX_HI, SEED)
        for _ in range(max(1, warmup)):
            rb.time_cpu(threads, threads)
        ms = sum(rb.time_cpu(threads, threads) for _ in range(steps))
        res["ms_per_step"] = ms / steps
        res["value"] = steps * threads / (ms * 1e-3)
        res["single_thread_sparse_cpu"] = n / (rb.time_cpu(n, 1) * 1e-3)
        if with_dense:
            res["single_thread_dense_cpu"] = 1 / (rb.time_cpu(1, 1, dense=True) * 1e-3)
        rb.close()
    else:
        b = o.synthetic_batch(H, D, P, K_TOP, n, CTX_LO, CTX_HI, SEED)
        t_ = min(threads, n)
        o.sparse_decode(b, n_threads=t_)
        t0 = time.perf_counter()
        for _ in range(steps):
            o.sparse_decode(b, n_threads=t_)
        ms = (time.perf_counter() - t0) * 1e3
        res.update(cores=t_, ms_per_step=ms / steps, value=steps * n / (ms * 1e-3))
        t0 = time.perf_counter()
        o.sparse_decode(b, n_threads=1)
        res["single_thread_sparse_cpu"] = n / (time.perf_counter() - t0)
    res["unit"] = "tokens/s"
    res["sample"] = (f"{n} requests of the config-3 shape (ctx U{{{CTX_LO}..{CTX_HI}}}, H{H} D{D} "
                     f"P{P} k{K_TOP}, reference BuildSyntheticBatch seed {SEED}); value: "
                     f"sparse_cpu RunNaiveSparseStep, one request per host thread per step on "
                     f"{res['cores']} threads; single_thread_*: the same requests (sparse_cpu, "
                     f"all {n}) and one request (dense_cpu RunDenseStep) on one thread")
    return res


CPU_KEYS = ("value", "unit", "cores", "kind", "sample", "host_logical_cpus", "cpu_model",
            "single_thread_sparse_cpu", "single_thread_dense_cpu")


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    cb = cpu_sample(args.steps, args.warmup, with_dense=False)
    line = {
        "impl": "reference", "metric": "sparse decode tokens/s", "value": cb["value"],
        "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": cb["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config3 sample (host)", "requests": CPU_SAMPLE_REQUESTS,
                   "context": [CTX_LO, CTX_HI], "num_heads": H, "head_dim": D, "page_size": P,
                   "top_k_pages": K_TOP},
        "cpu_baseline": {k: cb[k] for k in CPU_KEYS if k in cb},
        "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- our arm

def build_workload(dsd, ctx_lens, device, kv_format=0, global_ids=None):
    """Allocates the pool, generates K/V on device, sets the request page tables.
    Local request r holds the data of global request global_ids[r] (default r)."""
    pages_per = (ctx_lens + P - 1) // P
    cap = int(pages_per.sum())
    ctx = dsd.SparseDecodeContext(H, D, P, K_TOP, cap, BATCH, cap, BATCH * K_TOP,
                                  max_requests=BATCH, max_pages_per_request=int(pages_per.max()),
                                  device=device, kv_format=kv_format)
    page_ids, counts, reqs, first = [], [], [], []
    nxt = cap - 1
    table = []
    for r, (n_tok, n_pages) in enumerate(zip(ctx_lens, pages_per)):
        ids = np.arange(nxt, nxt - n_pages, -1, dtype=np.int32)  # LIFO PagePool order
        nxt -= n_pages
        table.append(ids)
        page_ids.append(ids)
        counts.append(np.minimum(P, n_tok - np.arange(n_pages) * P).astype(np.int32))
        reqs.append(np.full(n_pages, r if global_ids is None else int(global_ids[r]), np.int32))
        first.append((np.arange(n_pages) * P).astype(np.int32))
    ctx.generate_normal(np.concatenate(page_ids), np.concatenate(counts), np.concatenate(reqs),
                        np.concatenate(first), SEED)
    for r, ids in enumerate(table):
        ctx.set_request_pages(r, ids)
    return ctx, cap, np.concatenate(page_ids), np.concatenate(counts)


def queries_host(dsd, global_ids=None):
    q = np.empty((BATCH, E), np.float32)
    for r in range(BATCH):
        g = r if global_ids is None else int(global_ids[r])
        q[r] = dsd.generate_normal_host(SEED, 0, dsd.normal_index(g, 0, E), E)
    return q


def run_ours(args):
    import torch
    world, rank, local = dist_env()
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device(f"cuda:{local}"))
    dsd = importlib.import_module("15-618_dynamic_sparse_decode_b200")
    if not dsd.available():
        raise RuntimeError("no sm_100 GPU visible")
    torch.cuda.set_device(local)
    global BATCH
    sharding = importlib.import_module("15-618_dynamic_sparse_decode_b200.sharding")
    # Requests are dealt round-robin by global id (id % world == rank), each
    # with the context length and data of that id in one global workload.
    # strong: the --batch requests in total; weak: --batch per GPU, i.e.
    # batch * world distinct requests (at N = 1 both are requests 0..63).
    total = args.batch if args.strong else args.batch * world
    gids = sharding.shard_round_robin(np.arange(total), world, rank)
    ctx_lens = workload_contexts(total)[gids]
    BATCH = len(gids)
    fmt = {"f32": dsd.KV_F32, "bf16": dsd.KV_BF16, "fp8": dsd.KV_FP8}[args.kv]
    bf16 = fmt != dsd.KV_F32          # a narrow (opt-in) page format
    ctx, cap, all_ids, all_counts = build_workload(dsd, ctx_lens, local, fmt, gids)
    qh = queries_host(dsd, gids)
    reqs = np.arange(BATCH, dtype=np.int32)

    # algorithmic bytes of one step (exact selected token count from a debug step)
    dbg = ctx.decode_step(reqs, qh, output_mode=dsd.OUTPUT_DEBUG)
    page_tokens = np.zeros(cap, np.int64)
    page_tokens[all_ids] = all_counts
    C = cap
    S = int(dbg["selected"].size)
    T_sel = int(page_tokens[dbg["selected"]].sum())
    el = {dsd.KV_F32: 4, dsd.KV_BF16: 2, dsd.KV_FP8: 1}[fmt]    # bytes per stored element
    score_bytes = el * E * C + 4 * E * BATCH + 4 * C           # summaries + queries + ids/scores
    attn_bytes = 2 * el * E * T_sel + 4 * E * BATCH + 4 * S     # selected K/V + queries + ids
    step_bytes = (el * E * C + 2 * el * E * T_sel + 8 * E * BATCH
                  + 4 * (C + 2 * S + 3 * BATCH + 3))

    dq = torch.from_numpy(qh).cuda(local)
    do = torch.zeros_like(dq)
    torch.cuda.synchronize()
    ctx.bind_requests(reqs)
    stream = torch.cuda.ExternalStream(ctx.stream(), device=local)

    for _ in range(args.warmup):
        ctx.decode_bound(dq.data_ptr(), do.data_ptr())
        ctx.decode_bound_timed(dq.data_ptr(), do.data_ptr())
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        time.sleep(0.15)   # let nvidia-smi start sampling
        torch.cuda.synchronize()
        # timed region: K back-to-back replays of the production step graph
        start.record(stream)
        for _ in range(args.steps):
            ctx.decode_bound(dq.data_ptr(), do.data_ptr())
        stop.record(stream)
        torch.cuda.synchronize()
        # stage durations: K replays of the same step from the graph that also
        # records an event between stages (averaged over the K steps)
        per_kernel = {"score_ms": [], "topk_ms": [], "attention_ms": [], "total_ms": []}
        for _ in range(args.steps):
            t = ctx.decode_bound_timed(dq.data_ptr(), do.data_ptr())
            for k_, v in t.items():
                per_kernel[k_].append(v)
    ms_local = start.elapsed_time(stop)
    per_rank = sharding.gather_rank_stats({"ms_per_step": ms_local / args.steps},
                                          device=f"cuda:{local}")
    ms_total = sharding.max_over_ranks(ms_local, device=f"cuda:{local}")
    ms_step = ms_total / args.steps
    timed_graph_ms = float(np.mean(per_kernel["total_ms"]))

    # e2e through the public C ABI: host queries in, host outputs out, both in
    # pinned host memory (the library DMAs pinned buffers directly)
    q_pin = torch.empty((BATCH, E), dtype=torch.float32, pin_memory=True).numpy()
    q_pin[:] = qh
    host_out = torch.empty((BATCH, E), dtype=torch.float32, pin_memory=True).numpy()
    for _ in range(max(1, args.warmup)):
        ctx.decode_step(reqs, q_pin, output_mode=dsd.OUTPUT_OUTPUTS, out=host_out)
    ctx.reset_transfer_stats()
    if world > 1:
        torch.distributed.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        res = ctx.decode_step(reqs, q_pin, output_mode=dsd.OUTPUT_OUTPUTS, out=host_out)
    e2e_ms = (time.perf_counter() - t0) * 1e3 / args.steps
    st = ctx.transfer_stats()
    e2e_ms = sharding.max_over_ranks(e2e_ms, device=f"cuda:{local}")
    assert np.array_equal(res["outputs"], do.cpu().numpy()), "e2e and device-resident outputs differ"

    # the same public API with two steps in flight (decode_step_begin / _end):
    # step i+1's query upload and launch are queued before step i's outputs
    # are read back, as a serving loop over independent batches would
    ctx.decode_step_begin(reqs, q_pin)
    ctx.decode_step_end(out=host_out)
    if world > 1:
        torch.distributed.barrier()
    t0 = time.perf_counter()
    ctx.decode_step_begin(reqs, q_pin)
    for i in range(args.steps):
        if i + 1 < args.steps:
            ctx.decode_step_begin(reqs, q_pin)
        ctx.decode_step_end(out=host_out)
    e2e2_ms = sharding.max_over_ranks((time.perf_counter() - t0) * 1e3 / args.steps,
                                      device=f"cuda:{local}")
    assert np.array_equal(host_out, do.cpu().numpy()), "pipelined and device outputs differ"

    peak, peak_kind = peaks()
    score_ms = float(np.mean(per_kernel["score_ms"]))
    attn_ms = float(np.mean(per_kernel["attention_ms"]))
    dom = ("attention", attn_ms, attn_bytes) if attn_ms >= score_ms else ("score", score_ms, score_bytes)
    achieved = dom[2] / (dom[1] * 1e-3) / 1e9
    line = {
        "metric": "sparse decode tokens/s", "value": world * BATCH / (ms_step * 1e-3),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong" if args.strong else "weak", "vs_baseline": None,
        "dtype": args.kv + " pages, f32 arithmetic" if bf16 else "f32",
        "data": "synthetic (device-generated N(0,1) Irwin-Hall, seed 7)",
        "config": {"workload": ("config3: batch %d in total (strong), ctx U{16384..32768}, H32 D128 "
                                "P16 k64" % args.batch) if args.strong else
                               "config3: batch 64/GPU (global request ids rank + world*r), "
                               "ctx U{16384..32768}, H32 D128 P16 k64",
                   "kv_format": args.kv, "requests_per_gpu": BATCH, "candidate_pages_per_gpu": C,
                   "selected_pages_per_gpu": S, "selected_tokens_per_gpu": T_sel,
                   "step_bytes_per_gpu": step_bytes,
                   "step_hbm_gbps": step_bytes / (ms_step * 1e-3) / 1e9,
                   "step_roofline_frac": step_bytes / (ms_step * 1e-3) / 1e9 / peak,
                   "timed_graph_kernels_ms_per_step": timed_graph_ms,
                   "timing": "value: K back-to-back replays of the step graph (CUDA events on the "
                             "context stream, max over ranks); kernel_ms: mean over K replays of "
                             "the graph variant with event-record nodes between the stages",
                   "kernel_ms": {"score(+plan)": score_ms,
                                 "select": float(np.mean(per_kernel["topk_ms"])),
                                 "attention(+combine)": attn_ms},
                   "l2": "inputs larger than L2 (%.1f GB read per step)" % (step_bytes / 1e9),
                   "parallelism": f"request-sharded x{world}",
                   "per_rank_ms_per_step": [round(r["ms_per_step"], 4) for r in per_rank]},
        "roofline": {"bound": "hbm", "kernel": dom[0], "achieved": achieved, "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                     "algorithmic_bytes": dom[2],
                     "traffic": (profiled_traffic("attn" if dom[0] == "attention" else "score")
                                 if BATCH == 64 and not bf16 else None)},
        "e2e": {"value": world * BATCH / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": st["h2d_bytes"] / args.steps,
                "d2h_bytes_per_step": st["d2h_bytes"] / args.steps},
        "e2e_two_in_flight": {"value": world * BATCH / (e2e2_ms * 1e-3), "unit": "tokens/s",
                              "note": "decode_step_begin/_end with host buffers, two steps "
                                      "in flight; e2e is the synchronous call"},
        "gpu_launches": dsd.load_library().dsd_kernels_per_step() * args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = cpu_sample(3, 1)
        line["cpu_baseline"] = {k: cb[k] for k in CPU_KEYS if k in cb}
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        torch.distributed.destroy_process_group()


# ---------------------------------------------------------------- continuous serving

CONTINUOUS = {
    # BASELINE config 4 with the options of the reference's published run
    # (results/report_experiments/05_continuous_batching_load_sweep/...csv:25: direct GPU
    # upload, preadmit, precomputed payloads, GPU synthetic append, lazy release)
    "config4": dict(argv=[128, 32, 64, 1024, 4096, 16, 64, 7, 32, 128, 16, 8, 1, 1, 1, 1, 1, 1, 1, 0, 1, 1],
                    desc="config4: 128 req, max_active 32/GPU, arrival [0,64], prompt 1024-4096, "
                         "decode 16-64, H32 D128 P16 k8, direct GPU upload, preadmit, "
                         "precompute, GPU synthetic append, lazy release",
                    published=36236.393529, repeats=5),
    # box-scale serving, synthetic GPU prefill and append
    "config5": dict(argv=[2048, 128, 512, 8192, 32768, 64, 256, 11, 32, 128, 32, 32, 2, 0, 0, 1, 0, 1, 0, 0, 1, 1],
                    desc="config5: 2048 req, max_active 128/GPU, arrival [0,512], prompt 8192-32768, "
                         "decode 64-256, H32 D128 P32 k32, synthetic GPU prefill + append"),
}


def run_continuous(args):
    """Runs dsd_continuous_bench for this rank's shard (request_id % world == rank)."""
    world, rank, local = dist_env()
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device(f"cuda:{local}"))
        dist.barrier()
    spec = CONTINUOUS[args.workload]
    exe = os.path.join(ROOT, "15-618_dynamic_sparse_decode_b200", "bin", "dsd_continuous_bench")
    argv = [str(x) for x in spec["argv"]] + [str(world), str(rank), str(spec.get("repeats", 1)),
                                             {"f32": "0", "bf16": "1", "fp8": "2"}[args.kv]]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES=str(local))
    out = subprocess.run([exe, *argv], capture_output=True, text=True, env=env)
    if out.returncode != 0:
        raise RuntimeError(out.stderr)
    kv = dict(line.split("=", 1) for line in out.stdout.splitlines() if "=" in line)
    tokens = float(kv["total_generated_tokens"])
    ms = float(kv["continuous_sparse_total_ms"])
    steps = float(kv["continuous_sparse_run_batch_wall_ms"]) / max(1e-9, float(kv["continuous_sparse_avg_step_ms"]))
    h2d = float(kv["continuous_sparse_device_h2d_bytes"]) / max(1.0, steps)
    d2h = float(kv["continuous_sparse_device_d2h_bytes"]) / max(1.0, steps)
    local_stats = {"tokens": tokens, "ms": ms, "steps": steps, "h2d": h2d, "d2h": d2h,
                   "avg_step_ms": float(kv["continuous_sparse_avg_step_ms"]),
                   "avg_kernel_ms": float(kv["continuous_sparse_avg_kernel_ms"]),
                   "admission_ms": float(kv["continuous_sparse_runtime_admission_ms"])}
    if world > 1:
        sharding = importlib.import_module("15-618_dynamic_sparse_decode_b200.sharding")
        ranks = sharding.gather_rank_stats(local_stats, device=f"cuda:{local}")
    else:
        ranks = [local_stats]
    if rank == 0:
        tot = sum(r["tokens"] for r in ranks)
        wall = max(r["ms"] for r in ranks)
        value = tot / (wall * 1e-3)
        line = {
            "metric": "continuous sparse decode tokens/s", "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": int(max(r["steps"] for r in ranks)), "warmup": 0,
            "ms_per_step": float(np.mean([r["avg_step_ms"] for r in ranks])),
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": (value / spec["published"]
                            if spec.get("published") and world == 1 and args.kv == "f32"
                            else None),
            "dtype": args.kv + " pages, f32 arithmetic" if args.kv != "f32" else "f32",
            "data": "synthetic (reference mt19937 workload generator)",
            "config": {"workload": spec["desc"], "kv_format": args.kv, "argv": argv,
                       "per_rank": [{k: round(v, 3) for k, v in r.items()} for r in ranks],
                       "timing": "host wall time of the serving loop per rank (admission, "
                                 "steps, appends, releases); max over ranks"},
            "e2e": {"value": value, "unit": "tokens/s",
                    "h2d_bytes_per_step": float(np.mean([r["h2d"] for r in ranks])),
                    "d2h_bytes_per_step": float(np.mean([r["d2h"] for r in ranks]))},
            "gpu_launches": None,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def main():
    global BATCH
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="config3", choices=["config3", "config4", "config5"],
                    help="config3: the headline batched decode step; config4/5: continuous "
                         "serving through dsd_continuous_bench, request-sharded per GPU")
    ap.add_argument("--batch", type=int, default=BATCH,
                    help="requests per GPU (default: the config-3 batch of 64; smaller only "
                         "for profiling captures)")
    ap.add_argument("--strong", action="store_true",
                    help="config 3 strong scaling: --batch requests in total, sharded by "
                         "request id over the ranks (default: weak, --batch per GPU)")
    ap.add_argument("--kv", default="f32", choices=["f32", "bf16", "fp8"],
                    help="page format: f32 (the reference's, default) or "
                         "the opt-in bf16 / fp8 e4m3 pages (reported separately, never the headline)")
    args = ap.parse_args()
    BATCH = args.batch
    if args.impl == "reference":
        run_reference(args)
    elif args.workload != "config3":
        run_continuous(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
