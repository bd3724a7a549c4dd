// dsd_kernels.cuh -- sm_100a kernels of the batched page-level sparse decode step.
//
// One decode step (SparseCudaContext::RunBatch in the reference,
// src/cuda/sparse_batched_attention.cu:574-838) is five kernels: plan, then
// score -> select -> attention -> combine.  The production step is a CUDA
// graph that splits the requests into two ranges whose four-kernel chains
// run on two streams (fork/join inside the graph):
//
//   plan_kernel     per-request CSR offsets by a device prefix sum (replaces
//                   the host PackSparseBatchInto, :24-96)
//   score_kernel    score[c] = seqdot(q_r, summary[page_c]) * 1/sqrt(D), in the
//                   CPU's exact operation order (ScorePagesCpu,
//                   src/reference_kernels.cpp:59-80) so page selection is
//                   bit-identical to sparse_cpu; summaries stream HBM -> smem
//                   through a 3-stage ring of coalesced 16 B cp.async copies
//   select_kernel   per-request top-min(k,n) by (score desc, page id asc)
//                   (SelectTopKPagesCpu, :82-107) via a 64-bit radix select
//   attn_kernel     split-K flash decode over the selected pages, all heads
//                   of a page per CTA; K/V token rows stream HBM -> smem with
//                   cp.async.bulk (GatherPagesCpu + SparseAttentionCpu,
//                   :109-194, fused)
//   combine_kernel  log-sum-exp merge of the split-K partials
//
// Pool maintenance kernels (upload with summary, token append with running
// mean, free, synthetic generators) follow at the end.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dsdk {

// Storage element of the K/V pages and the summaries: fp32 (the parity
// path), bf16 or fp8 e4m3 (opt-in; arithmetic stays fp32, values round to nearest even
// when stored).  get/put convert one element, store4 four, round/round4
// give the value the storage will hold.
template <typename T>
struct Kv;
template <>
struct Kv<float> {
  __device__ __forceinline__ static float get(const float* p, size_t i) { return p[i]; }
  __device__ __forceinline__ static float round(float v) { return v; }
  __device__ __forceinline__ static void put(float* p, size_t i, float v) { p[i] = v; }
  __device__ __forceinline__ static void store4(float* p, float4 v) {
    *reinterpret_cast<float4*>(p) = v;
  }
  __device__ __forceinline__ static float4 round4(float4 v) { return v; }
};
template <>
struct Kv<__nv_bfloat16> {
  using T = __nv_bfloat16;
  __device__ __forceinline__ static float get(const T* p, size_t i) { return __bfloat162float(p[i]); }
  __device__ __forceinline__ static float round(float v) {
    return __bfloat162float(__float2bfloat16_rn(v));
  }
  __device__ __forceinline__ static void put(T* p, size_t i, float v) { p[i] = __float2bfloat16_rn(v); }
  __device__ __forceinline__ static void store4(T* p, float4 v) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y);
    const __nv_bfloat162 b = __floats2bfloat162_rn(v.z, v.w);
    uint2 raw;
    raw.x = *reinterpret_cast<const uint32_t*>(&a);
    raw.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = raw;
  }
  __device__ __forceinline__ static float4 round4(float4 v) {
    return make_float4(round(v.x), round(v.y), round(v.z), round(v.w));
  }
};
template <>
struct Kv<__nv_fp8_e4m3> {
  using T = __nv_fp8_e4m3;
  __device__ __forceinline__ static uint8_t enc(float v) {
    return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
  }
  __device__ __forceinline__ static float dec(uint8_t b) {
    const __half_raw hr = __nv_cvt_fp8_to_halfraw(b, __NV_E4M3);
    return __half2float(*reinterpret_cast<const __half*>(&hr));
  }
  __device__ __forceinline__ static float get(const T* p, size_t i) {
    return dec(reinterpret_cast<const uint8_t*>(p)[i]);
  }
  __device__ __forceinline__ static float round(float v) { return dec(enc(v)); }
  __device__ __forceinline__ static void put(T* p, size_t i, float v) {
    reinterpret_cast<uint8_t*>(p)[i] = enc(v);
  }
  __device__ __forceinline__ static void store4(T* p, float4 v) {
    const uint32_t w = uint32_t(enc(v.x)) | (uint32_t(enc(v.y)) << 8) |
                       (uint32_t(enc(v.z)) << 16) | (uint32_t(enc(v.w)) << 24);
    *reinterpret_cast<uint32_t*>(p) = w;
  }
  __device__ __forceinline__ static float4 round4(float4 v) {
    return make_float4(round(v.x), round(v.y), round(v.z), round(v.w));
  }
};

constexpr int kMaxBatch = 1024;
constexpr int kPlanThreads = 1024;

// score tiles: 128 candidates of one request, one per consumer thread
constexpr int kScoreTile = 128;
constexpr int kScoreChunk = 64;                     // floats of a summary row per stage
constexpr int kScoreRowStride = kScoreChunk + 4;    // +16 B: conflict-free float4 rows
constexpr int kScoreStages = 3;
constexpr int kScoreThreads = kScoreTile;
// small tiles (ts <= kScoreSmallTile candidates, small batches): the same
// ring with 33-row stages, kScoreSmallStages deep, so more chunks are in
// flight per dependent chain
constexpr int kScoreSmallTile = 32;
constexpr int kScoreSmallStages = 3;
constexpr int kScoreSmallMult = 4;     // layout chunks per stage row (256 floats)
constexpr size_t ScoreRingBytes(int tile, int stages, int mult) {
  return size_t(stages) * (tile + 1) * (kScoreChunk * mult + 4) * sizeof(float);
}
constexpr size_t kScoreSmem = ScoreRingBytes(kScoreTile, kScoreStages, 1) >
                                      ScoreRingBytes(kScoreSmallTile, kScoreSmallStages, kScoreSmallMult)
                                  ? ScoreRingBytes(kScoreTile, kScoreStages, 1)
                                  : ScoreRingBytes(kScoreSmallTile, kScoreSmallStages, kScoreSmallMult);

constexpr int kAttnThreads = 256;
constexpr int kAttnStages = 3;
constexpr int kAttnStageFloats = 16384;             // K+V floats per stage (64 KiB)
constexpr int kMaxPagesPerUnit = 16;
constexpr int kAttnMaxTokensPerStage = 8;           // logits held in registers per stage

constexpr int kSelectThreads = 512;
constexpr int kSelectMaxK = 4096;                   // selected pages per request
constexpr int kSelectSmemKeys = 8192;               // candidates staged in shared memory
constexpr size_t kSelectSmem = size_t(kSelectMaxK + kSelectSmemKeys) * 8;   // 96 KiB

// status bits written by kernels (read by the host after the step)
constexpr int kStatusTimeout = 1;
constexpr int kStatusBadInput = 2;

// A bounded wait: ~2^31 cycles (about a second at 1.9 GHz).
constexpr long long kWaitBudgetCycles = 2LL << 30;

struct StepPlan {
  // written by the host each step (one packed H2D copy)
  const int* hdr;          // [0] batch, [1] mode (0 = CSR, 1 = page tables), [2] dense
  const int* req;          // CSR: cand_offsets[B+1]; tables: slot[B]
  const int* cand_ids;     // CSR ids
  // device page tables
  const int* table;        // [max_requests][stride]
  const int* table_n;      // [max_requests]
  int table_stride;
  // computed by plan_kernel
  int* n_cand;             // [B]
  int* id_base;            // [B]  offset of request r's ids in its id array
  int* score_off;          // [B+1]
  int* sel_off;            // [B+1]
  int* tile_off;           // [B+1]
  int* unit_off;           // [B+1]
  int* misc;               // [0] pages per attention unit, [1] score tile size, [2] dense
  int* status;             // error bits
  // > 0: the CSR candidate ids are range-checked on the device against this
  // pool capacity before any page is read (callers whose ids never passed a
  // host check); 0: the host validated them
  int capacity;
};

// ------------------------------------------------------------------ PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the barrier phase with a cycle budget; on expiry sets the
// timeout bit in *status and returns false (the caller then stops issuing work).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status,
                                          long long budget = kWaitBudgetCycles) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - start > budget) {
      atomicOr(status, kStatusTimeout);
      return false;
    }
  }
  return true;
}

// Bounded wait that also gives up as soon as another warp of the CTA has
// raised *abort (a shared flag): the timeout of one waiter then ends every
// waiter's loop within one poll instead of one budget each.  On its own
// expiry it sets the timeout status bit and raises *abort.
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t* bar, uint32_t parity, int* status,
                                                   volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort) return false;
    if (clock64() - start > kWaitBudgetCycles) {
      atomicOr(status, kStatusTimeout);
      *abort = 1;
      return false;
    }
  }
  return true;
}

// After an abort: waits (bounded) for the copies of the last `nstages`
// issues of a ring to land, so that no bulk copy still writes into this
// CTA's shared memory when the CTA exits.  `issued` = stages issued so far;
// issue i went to stage i % nstages with phase parity (i / nstages) & 1, and
// only the latest issue of each stage can still be in flight.
__device__ __forceinline__ void drain_ring(uint64_t* full, uint32_t issued, int nstages,
                                           int* status) {
  const uint32_t first = issued > uint32_t(nstages) ? issued - uint32_t(nstages) : 0u;
  for (uint32_t i = first; i < issued; ++i)
    mbar_wait(&full[i % uint32_t(nstages)], (i / uint32_t(nstages)) & 1u, status);
}

// Self-test of the bounded wait: one thread waits on a barrier phase that
// nothing completes (no copy is issued, no thread arrives) with a small
// budget.  The wait gives up, sets the timeout bit and the kernel returns.
__global__ void bounded_wait_probe_kernel(int* status, long long budget) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
    mbar_wait(&bar, 0, status, budget);
  }
}

// 1-D bulk copy global -> shared (TMA), completion counted on `bar` in bytes.
// Both addresses 16 B aligned, bytes a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// index of the last segment whose start offset is <= x (offs ascending, offs[0] = 0)
__device__ __forceinline__ int upper_segment(const int* offs, int n, int x) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(offs + mid) <= x) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// ------------------------------------------------------------------ summary layout
//
// Page summaries are stored chunk-major inside groups of 128 pages:
//   element e of page p lives at ((p/128 * NC + e/CW) * 128 + p%128) * CW + e%CW
// with CW = min(64, largest power of two dividing H*D) and NC = H*D / CW.
// A score tile of consecutive page ids then reads, per stage, one contiguous
// run of 128 * CW floats instead of 128 scattered row pieces.
__host__ __device__ __forceinline__ int summary_chunk(int ept) {
  const int low = ept & -ept;
  return low < 64 ? low : 64;
}
__host__ __device__ __forceinline__ size_t summary_group_floats(int ept) {
  return size_t(128) * ept;
}
// offset of (page, chunk 0, element 0); chunk c adds c * 128 * CW
__host__ __device__ __forceinline__ size_t summary_row_base(int page, int ept) {
  return size_t(page >> 7) * summary_group_floats(ept) + size_t(page & 127) * summary_chunk(ept);
}
__host__ __device__ __forceinline__ size_t summary_off(int page, int e, int ept) {
  const int cw = summary_chunk(ept);
  return summary_row_base(page, ept) + size_t(e / cw) * 128 * cw + (e % cw);
}

// Requests [r0, r1) of part `part` of `nparts` (a step may be split into
// request ranges that run on different streams).
__device__ __forceinline__ void part_range(int B, int part, int nparts, int* r0, int* r1) {
  *r0 = static_cast<int>(static_cast<long long>(B) * part / nparts);
  *r1 = static_cast<int>(static_cast<long long>(B) * (part + 1) / nparts);
}

// ------------------------------------------------------------------ plan

// Block-wide exclusive scan of up to 4 ints per thread (one element per thread).
template <int N>
__device__ __forceinline__ void block_exclusive_scan(int (&v)[N], int (&total)[N]) {
  __shared__ int warp_sums[32][N];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl[N];
#pragma unroll
  for (int i = 0; i < N; ++i) {
    int x = v[i];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    incl[i] = x;
    if (lane == 31) warp_sums[warp][i] = x;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
#pragma unroll
    for (int i = 0; i < N; ++i) {
      int x = lane < nw ? warp_sums[lane][i] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (lane < nw) warp_sums[lane][i] = x;  // inclusive over warps
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const int before = warp > 0 ? warp_sums[warp - 1][i] : 0;
    total[i] = warp_sums[(blockDim.x >> 5) - 1][i];
    v[i] = before + incl[i] - v[i];
  }
  __syncthreads();
}

// One CTA of 1024 threads.  Computes the step's ragged layout from the
// request list: candidate counts (CSR offsets or page-table lengths),
// selected counts min(k, n), score tiles and split-K attention units.
__global__ void __launch_bounds__(kPlanThreads) plan_kernel(StepPlan plan, int top_k,
                                                            int target_units, int score_grid) {
  const int B = plan.hdr[0];
  const int mode = plan.hdr[1];
  const int dense = plan.hdr[2];   // 1: attend over every candidate (no scoring, no top-k)
  const int r = threadIdx.x;
  int n = 0, base = 0;
  if (r < B) {
    if (mode == 0) {
      base = plan.req[r];
      n = plan.req[r + 1] - base;
    } else {
      const int slot = plan.req[r];
      base = slot * plan.table_stride;
      n = plan.table_n[slot];
    }
    if (n < 0) { n = 0; atomicOr(plan.status, kStatusBadInput); }
  }
  if (plan.capacity > 0 && mode == 0) {
    // ids straight from device memory: one out-of-range id rejects the step
    // before any summary or page is loaded (every request then has no
    // candidates, so the later kernels read nothing and write zero outputs)
    const int total = B > 0 ? plan.req[B] : 0;
    bool bad = false;
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
      const int id = plan.cand_ids[i];
      bad |= id < 0 || id >= plan.capacity;
    }
    if (__syncthreads_or(bad)) {
      if (threadIdx.x == 0) atomicOr(plan.status, kStatusBadInput);
      n = 0;
    }
  }
  const int ksel = dense ? n : max(0, min(top_k, n));
  int v[2] = {n, ksel};
  int tot[2];
  block_exclusive_scan<2>(v, tot);
  // Score tile size: the smallest ts <= kScoreTile whose tile count fits a
  // whole number of waves over the score grid, so every CTA runs the same
  // number of (slightly shorter) tiles instead of a ragged last wave.
  // The 32 warps test 32 candidate sizes at a time.
  __shared__ int s_n[kMaxBatch];
  __shared__ int s_best;
  const int waves = max(1, (tot[0] + kScoreTile * score_grid - 1) / (kScoreTile * score_grid));
  const int target_tiles = waves * score_grid;
  const int ts0 = max(1, min(kScoreTile, (tot[0] + target_tiles - 1) / max(1, target_tiles)));
  if (r < kMaxBatch) s_n[r] = n;
  if (threadIdx.x == 0) s_best = kScoreTile;
  __syncthreads();
  {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int base_ts = ts0; base_ts < kScoreTile; base_ts += kPlanThreads / 32) {
      const int cand = base_ts + warp;
      if (cand < kScoreTile) {
        int c = 0;
        for (int i = lane; i < B; i += 32) c += (s_n[i] + cand - 1) / cand;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
        if (lane == 0 && c <= target_tiles) atomicMin(&s_best, cand);
      }
      __syncthreads();
      const int best = s_best;
      __syncthreads();
      if (best < kScoreTile) break;
    }
  }
  const int ts = s_best;
  int t1[1] = {dense ? 0 : (n + ts - 1) / ts};
  int ttot[1];
  block_exclusive_scan<1>(t1, ttot);
  if (r < B) {
    plan.n_cand[r] = n;
    plan.id_base[r] = base;
    plan.score_off[r] = v[0];
    plan.sel_off[r] = v[1];
    plan.tile_off[r] = t1[0];
  }
  if (r == 0) {
    plan.score_off[B] = tot[0];
    plan.sel_off[B] = tot[1];
    plan.tile_off[B] = ttot[0];
    plan.misc[1] = ts;
    plan.misc[2] = dense;
  }
  // pages per attention unit: enough units to fill the GPU, at most 16 pages
  int ppu = (tot[1] + target_units - 1) / max(1, target_units);
  ppu = max(1, min(kMaxPagesPerUnit, ppu));
  int u[1] = {(ksel + ppu - 1) / ppu};
  int utot[1];
  block_exclusive_scan<1>(u, utot);
  if (r < B) plan.unit_off[r] = u[0];
  if (r == 0) {
    plan.unit_off[B] = utot[0];
    plan.misc[0] = ppu;
  }
}

// ------------------------------------------------------------------ score

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Persistent CTAs over score tiles.  Thread t owns candidate t of the tile
// and accumulates q[i]*s[i] for i = 0..E-1 in order with round-to-nearest
// multiply and add (no FMA), exactly ScorePagesCpu's Dot.  The tile's
// summary rows stream through a STAGES-deep shared-memory ring,
// kScoreChunk floats per row per stage, filled by all threads with coalesced
// 16-byte cp.async copies (one warp moves two 256 B row chunks per
// instruction); row TILE of every stage holds the query chunk.  Tiles of up
// to 128 candidates use 3 stages of one 64-float layout chunk per row.  When
// the plan picked tiles of at most 32 candidates (small batches: a CTA runs a
// few 4096-long chains) a stage row holds M = 4 layout chunks, so the
// per-stage barrier and copy issue are paid once per 256 elements of the
// chain instead of once per 64.
// Thread t always copies rows t/kCols + kRowStep*j, column t%kCols, so it
// keeps the page offsets of the tile it is loading in registers.
template <int TILE, int STAGES, int M>
__device__ __forceinline__ void score_tiles(
    const StepPlan& plan, const float* __restrict__ queries, const float* __restrict__ summaries,
    int ept, float scale, float* __restrict__ scores, int part, int nparts,
    unsigned char* smem_raw) {
  float* stage_base = reinterpret_cast<float*>(smem_raw);
  // M layout chunks (of kScoreChunk floats, each its own 256 B run) per stage row
  constexpr int kCols = kScoreChunk * M / 4;              // float4 columns per stage row
  constexpr int kRowStep = kScoreThreads / kCols;         // rows one pass of the CTA covers
  constexpr int kRows = TILE + 1;                          // + the query chunk
  constexpr int kRowsPerThread = (kRows + kRowStep - 1) / kRowStep;
  constexpr int kStride = kScoreChunk * M + 4;             // +16 B: conflict-free float4 rows
  constexpr int kStageFloats = kRows * kStride;

  const int tid = threadIdx.x;
  const int B = plan.hdr[0];
  const int mode = plan.hdr[1];
  const int* ids_src = mode == 0 ? plan.cand_ids : plan.table;
  int r_begin, r_end;
  part_range(B, part, nparts, &r_begin, &r_end);
  const int tile_begin = plan.tile_off[r_begin];
  const int total_tiles = plan.tile_off[r_end];
  const int ts = plan.misc[1];
  const int cw = summary_chunk(ept);          // floats of a page's summary per stage
  const int nchunks = ept / (cw * M);        // M > 1 only when cw == kScoreChunk
  const size_t chunk_stride = size_t(128) * cw;
  const int col = tid % kCols;
  const int row0 = tid / kCols;

  // ---- loader state (runs STAGES-1 chunks ahead of the compute)
  int ld_tile = tile_begin + blockIdx.x, ld_ch = 0, ld_slot = 0, ld_nvalid = 0;
  const float* ld_q = queries;
  size_t ld_off[kRowsPerThread];
  auto load_tile = [&]() {
    if (ld_tile >= total_tiles) return;
    const int r = upper_segment(plan.tile_off, B, ld_tile);
    const int c0 = (ld_tile - plan.tile_off[r]) * ts;
    ld_nvalid = min(ts, plan.n_cand[r] - c0);
    ld_q = queries + size_t(r) * ept;
    const int* ids = ids_src + plan.id_base[r] + c0;
#pragma unroll
    for (int j = 0; j < kRowsPerThread; ++j) {
      const int row = row0 + kRowStep * j;
      ld_off[j] = row < ld_nvalid ? summary_row_base(__ldg(ids + row), ept) : 0;
    }
  };
  auto issue = [&]() {
    if (ld_tile < total_tiles) {
      const int len = cw;
      float* st = stage_base + size_t(ld_slot) * kStageFloats;
      if (col * 4 < len * M) {
        const size_t coff =
            size_t(ld_ch * M + col / (kScoreChunk / 4)) * chunk_stride + (col % (kScoreChunk / 4)) * 4;
        const size_t qoff = size_t(ld_ch) * cw * M + col * 4;
#pragma unroll
        for (int j = 0; j < kRowsPerThread; ++j) {
          const int row = row0 + kRowStep * j;
          if (row < ld_nvalid) {
            cp_async16(st + row * kStride + col * 4, summaries + ld_off[j] + coff);
          } else if (row == TILE) {
            cp_async16(st + row * kStride + col * 4, ld_q + qoff);
          }
        }
      }
      if (++ld_ch == nchunks) {
        ld_ch = 0;
        ld_tile += gridDim.x;
        load_tile();
      }
    }
    cp_async_commit();
    ld_slot = ld_slot + 1 == STAGES ? 0 : ld_slot + 1;
  };

  load_tile();
#pragma unroll 1
  for (int i = 0; i < STAGES - 1; ++i) issue();

  int slot = 0;
  for (int tile = tile_begin + blockIdx.x; tile < total_tiles; tile += gridDim.x) {
    const int r = upper_segment(plan.tile_off, B, tile);
    const int c0 = (tile - plan.tile_off[r]) * ts;
    const int nvalid = min(ts, plan.n_cand[r] - c0);
    float acc = 0.0f;
    for (int ch = 0; ch < nchunks; ++ch) {
      cp_async_wait<STAGES - 2>();
      __syncthreads();   // chunk `slot` landed for all threads; slot-1 is free again
      issue();
      const int len = cw;
      const float* st = stage_base + size_t(slot) * kStageFloats;
      if (tid < nvalid) {
        const float4* srow = reinterpret_cast<const float4*>(st + tid * kStride);
        const float4* qv = reinterpret_cast<const float4*>(st + TILE * kStride);
        if (len == kScoreChunk) {
#pragma unroll
          for (int i = 0; i < kScoreChunk * M / 4; ++i) {
            const float4 a = qv[i];
            const float4 b = srow[i];
            acc = __fadd_rn(acc, __fmul_rn(a.x, b.x));
            acc = __fadd_rn(acc, __fmul_rn(a.y, b.y));
            acc = __fadd_rn(acc, __fmul_rn(a.z, b.z));
            acc = __fadd_rn(acc, __fmul_rn(a.w, b.w));
          }
        } else {
          for (int i = 0; i < len / 4; ++i) {
            const float4 a = qv[i];
            const float4 b = srow[i];
            acc = __fadd_rn(acc, __fmul_rn(a.x, b.x));
            acc = __fadd_rn(acc, __fmul_rn(a.y, b.y));
            acc = __fadd_rn(acc, __fmul_rn(a.z, b.z));
            acc = __fadd_rn(acc, __fmul_rn(a.w, b.w));
          }
        }
      }
      slot = slot + 1 == STAGES ? 0 : slot + 1;
    }
    if (tid < nvalid) scores[plan.score_off[r] + c0 + tid] = __fmul_rn(acc, scale);
  }
  cp_async_wait<0>();
}

__global__ void __launch_bounds__(kScoreThreads, 2) score_kernel(
    StepPlan plan, const float* __restrict__ queries, const float* __restrict__ summaries,
    int ept, float scale, float* __restrict__ scores, int part, int nparts) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  if (plan.misc[1] > kScoreSmallTile)
    score_tiles<kScoreTile, kScoreStages, 1>(plan, queries, summaries, ept, scale, scores, part,
                                             nparts, smem_raw);
  else if (summary_chunk(ept) == kScoreChunk && (ept / kScoreChunk) % kScoreSmallMult == 0)
    score_tiles<kScoreSmallTile, kScoreSmallStages, kScoreSmallMult>(
        plan, queries, summaries, ept, scale, scores, part, nparts, smem_raw);
  else
    score_tiles<kScoreSmallTile, kScoreSmallStages, 1>(plan, queries, summaries, ept, scale,
                                                       scores, part, nparts, smem_raw);
}

// Narrow-row scoring: the score_kernel scheme with 128-byte row pieces per
// stage (32 fp32, 64 bf16 or 128 fp8 elements, 8 columns of 16 bytes), 144-byte padded
// shared-memory rows (the 8 threads of a quarter warp read 8 different 16 B
// bank groups), the fp32 query piece in its own region, and small stages so
// 4 CTAs fit on an SM: twice the warps of score_kernel to hide the
// per-thread dependent add chain.  The dot product is the same sequential
// round-to-nearest chain; bf16 and fp8 elements widen to fp32 exactly.
template <typename T>
struct ScoreRows {
  static constexpr int kEP = 16 / int(sizeof(T));          // elements per 16 B
  static constexpr int kChunk = 128 / int(sizeof(T));      // elements per row piece
  static constexpr int kStride = kChunk + kEP;             // smem row stride (elements)
  static constexpr size_t kStageBytes =
      size_t(kScoreTile) * kStride * sizeof(T) + size_t(kChunk) * 4;
};

// 16 bytes of summary -> fp32 elements
__device__ __forceinline__ void widen16(const uint4 raw, const float*, float (&f)[4]) {
  f[0] = __uint_as_float(raw.x); f[1] = __uint_as_float(raw.y);
  f[2] = __uint_as_float(raw.z); f[3] = __uint_as_float(raw.w);
}
__device__ __forceinline__ void widen16(const uint4 raw, const __nv_bfloat16*, float (&f)[8]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    f[2 * h] = __uint_as_float(w[h] << 16);              // bf16 -> fp32: exact
    f[2 * h + 1] = __uint_as_float(w[h] & 0xffff0000u);
  }
}

// two fp8 e4m3 (low byte first) -> float2, exact (through half).  The
// conversions issue on the conversion pipe, which bounds both fp8 kernels; an
// integer widening (bit moves into fp32 position plus a power-of-two rescale)
// was measured slower on every consumer split (more integer-ALU issue than
// the conversion pipe saves), so the hardware conversion stays.
__device__ __forceinline__ float2 fp8x2_to_float2(uint32_t pair) {
  const __half2_raw hr =
      __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(pair & 0xffffu), __NV_E4M3);
  return __half22float2(*reinterpret_cast<const __half2*>(&hr));
}
__device__ __forceinline__ void widen16(const uint4 raw, const __nv_fp8_e4m3*, float (&f)[16]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    const float2 lo = fp8x2_to_float2(w[h]), hi = fp8x2_to_float2(w[h] >> 16);
    f[4 * h] = lo.x; f[4 * h + 1] = lo.y; f[4 * h + 2] = hi.x; f[4 * h + 3] = hi.y;
  }
}

template <typename T, int STAGES, int MINB>
__global__ void __launch_bounds__(kScoreThreads, MINB) score_kernel_narrow(
    StepPlan plan, const float* __restrict__ queries, const T* __restrict__ summaries, int ept,
    float scale, float* __restrict__ scores, int part, int nparts) {
  using R = ScoreRows<T>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  constexpr int kCols = R::kChunk / R::kEP;               // 8 columns of 16 B
  constexpr int kRowStep = kScoreThreads / kCols;
  constexpr int kRowsPerThread = kScoreTile / kRowStep;

  const int tid = threadIdx.x;
  const int B = plan.hdr[0];
  const int mode = plan.hdr[1];
  const int* ids_src = mode == 0 ? plan.cand_ids : plan.table;
  int r_begin, r_end;
  part_range(B, part, nparts, &r_begin, &r_end);
  const int tile_begin = plan.tile_off[r_begin];
  const int total_tiles = plan.tile_off[r_end];
  const int ts = plan.misc[1];
  const int cw = summary_chunk(ept);          // layout chunk (elements)
  // elements of a row per stage (>= kEP): a full 128-byte piece when it tiles
  // the row (it may span several layout chunks, each its own run)
  const int kc = ept % R::kChunk == 0 ? R::kChunk : min(R::kChunk, cw);
  const int cw_log2 = __ffs(cw) - 1;          // cw is a power of two
  const int nchunks = ept / kc;
  const size_t chunk_stride = size_t(128) * cw;
  const int col = tid % kCols;
  const int row0 = tid / kCols;

  int ld_tile = tile_begin + blockIdx.x, ld_ch = 0, ld_slot = 0, ld_nvalid = 0;
  const float* ld_q = queries;
  size_t ld_off[kRowsPerThread];
  auto load_tile = [&]() {
    if (ld_tile >= total_tiles) return;
    const int r = upper_segment(plan.tile_off, B, ld_tile);
    const int c0 = (ld_tile - plan.tile_off[r]) * ts;
    ld_nvalid = min(ts, plan.n_cand[r] - c0);
    ld_q = queries + size_t(r) * ept;
    const int* ids = ids_src + plan.id_base[r] + c0;
#pragma unroll
    for (int j = 0; j < kRowsPerThread; ++j) {
      const int row = row0 + kRowStep * j;
      ld_off[j] = row < ld_nvalid ? summary_row_base(__ldg(ids + row), ept) : 0;
    }
  };
  auto issue = [&]() {
    if (ld_tile < total_tiles) {
      unsigned char* st = smem_raw + size_t(ld_slot) * R::kStageBytes;
      T* rows = reinterpret_cast<T*>(st);
      float* qst = reinterpret_cast<float*>(st + size_t(kScoreTile) * R::kStride * sizeof(T));
      const int e0 = ld_ch * kc;
      if (col * R::kEP < kc) {
        const int e = e0 + col * R::kEP;
        const size_t coff = size_t(e >> cw_log2) * chunk_stride + (e & (cw - 1));
#pragma unroll
        for (int j = 0; j < kRowsPerThread; ++j) {
          const int row = row0 + kRowStep * j;
          if (row < ld_nvalid)
            cp_async16(rows + row * R::kStride + col * R::kEP, summaries + ld_off[j] + coff);
        }
      }
      if (tid * 4 < kc) cp_async16(qst + tid * 4, ld_q + size_t(e0) + tid * 4);
      if (++ld_ch == nchunks) {
        ld_ch = 0;
        ld_tile += gridDim.x;
        load_tile();
      }
    }
    cp_async_commit();
    ld_slot = ld_slot + 1 == STAGES ? 0 : ld_slot + 1;
  };

  load_tile();
#pragma unroll 1
  for (int i = 0; i < STAGES - 1; ++i) issue();

  int slot = 0;
  for (int tile = tile_begin + blockIdx.x; tile < total_tiles; tile += gridDim.x) {
    const int r = upper_segment(plan.tile_off, B, tile);
    const int c0 = (tile - plan.tile_off[r]) * ts;
    const int nvalid = min(ts, plan.n_cand[r] - c0);
    float acc = 0.0f;
    for (int ch = 0; ch < nchunks; ++ch) {
      cp_async_wait<STAGES - 2>();
      __syncthreads();   // chunk `slot` landed for all threads; slot-1 is free again
      issue();
      const unsigned char* st = smem_raw + size_t(slot) * R::kStageBytes;
      if (tid < nvalid) {
        const uint4* srow =
            reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(st) + tid * R::kStride);
        const float4* qv =
            reinterpret_cast<const float4*>(st + size_t(kScoreTile) * R::kStride * sizeof(T));
        auto piece = [&](int i) {
          float f[R::kEP];
          widen16(srow[i], static_cast<const T*>(nullptr), f);
#pragma unroll
          for (int h = 0; h < R::kEP / 4; ++h) {
            const float4 a = qv[i * (R::kEP / 4) + h];
            acc = __fadd_rn(acc, __fmul_rn(a.x, f[4 * h]));
            acc = __fadd_rn(acc, __fmul_rn(a.y, f[4 * h + 1]));
            acc = __fadd_rn(acc, __fmul_rn(a.z, f[4 * h + 2]));
            acc = __fadd_rn(acc, __fmul_rn(a.w, f[4 * h + 3]));
          }
        };
        if (kc == R::kChunk) {
#pragma unroll
          for (int i = 0; i < kCols; ++i) piece(i);
        } else {
          for (int i = 0; i < kc / R::kEP; ++i) piece(i);
        }
      }
      slot = slot + 1 == STAGES ? 0 : slot + 1;
    }
    if (tid < nvalid) scores[plan.score_off[r] + c0 + tid] = __fmul_rn(acc, scale);
  }
  cp_async_wait<0>();
}

// ------------------------------------------------------------------ select

// Order-preserving 64-bit key: larger key = better page.  High word is the
// score mapped to an unsigned order (-0.0 folded onto +0.0, so they tie as
// in the CPU comparator); low word is ~page_id so lower ids win ties.
__device__ __forceinline__ unsigned long long page_key(float score, int page) {
  uint32_t b = __float_as_uint(score);
  if (b == 0x80000000u) b = 0u;
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(b) << 32) | static_cast<uint32_t>(~page);
}

// One CTA per request (grid-stride).  The request's candidate keys are
// staged in shared memory (when n <= kSelectSmemKeys; otherwise every pass
// re-reads them from global memory).  A radix select, 8 bits per pass from
// the most significant byte, narrows the prefix of the k-th largest key and
// stops as soon as every key sharing the prefix is a winner.  Keys above the
// threshold (then the ones equal to it, for duplicated ids) are gathered,
// bitonic-sorted descending and written as page ids.
__global__ void __launch_bounds__(kSelectThreads) select_kernel(StepPlan plan,
                                                                const float* __restrict__ scores,
                                                                int* __restrict__ selected,
                                                                int part, int nparts) {
  extern __shared__ __align__(16) unsigned long long sel_smem[];
  unsigned long long* keys = sel_smem;                      // winners [kSelectMaxK]
  unsigned long long* all = sel_smem + kSelectMaxK;         // candidates [kSelectSmemKeys]
  __shared__ int hist[256];
  __shared__ unsigned long long s_prefix;
  __shared__ int s_remaining;
  __shared__ int s_done;
  __shared__ int s_count_gt;
  __shared__ int s_count_eq;

  const int B = plan.hdr[0];
  const int mode = plan.hdr[1];
  const int* ids_src = mode == 0 ? plan.cand_ids : plan.table;
  const int tid = threadIdx.x;

  int r_begin, r_end;
  part_range(B, part, nparts, &r_begin, &r_end);
  for (int r = r_begin + blockIdx.x; r < r_end; r += gridDim.x) {
    const int n = plan.n_cand[r];
    const int k = plan.sel_off[r + 1] - plan.sel_off[r];
    if (k <= 0) continue;
    if (k > kSelectMaxK && !plan.misc[2]) {
      if (tid == 0) atomicOr(plan.status, kStatusBadInput);
      continue;
    }
    const int* ids = ids_src + plan.id_base[r];
    if (plan.misc[2]) {
      // dense attention: every candidate, in candidate order
      int* out = selected + plan.sel_off[r];
      for (int i = tid; i < k; i += blockDim.x) out[i] = __ldg(ids + i);
      continue;
    }
    const float* sc = scores + plan.score_off[r];
    const bool staged = n <= kSelectSmemKeys;
    if (staged) {
      for (int i = tid; i < n; i += blockDim.x) all[i] = page_key(sc[i], __ldg(ids + i));
    }
    auto key_at = [&](int i) -> unsigned long long {
      return staged ? all[i] : page_key(sc[i], __ldg(ids + i));
    };

    unsigned long long threshold = 0;  // keys >= threshold are the winners
    if (k < n) {
      if (tid == 0) { s_prefix = 0; s_remaining = k; s_done = 0; }
      unsigned long long mask = 0;
      for (int pass = 0; pass < 8; ++pass) {
        const int shift = 56 - 8 * pass;
        for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        const unsigned long long prefix = s_prefix;
        for (int i = tid; i < n; i += blockDim.x) {
          const unsigned long long key = key_at(i);
          if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 0xff], 1);
        }
        __syncthreads();
        if (tid < 32) {
          // the digit (from 255 down) where the cumulative count reaches `remaining`
          const int rem = s_remaining;
          int cnt[8];
          int local = 0;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            cnt[j] = hist[255 - (tid * 8 + j)];
            local += cnt[j];
          }
          int incl = local;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (tid >= o) incl += y;
          }
          const int excl = incl - local;
          if (excl < rem && incl >= rem) {
            int acc = excl;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              if (acc + cnt[j] >= rem) {
                const int digit = 255 - (tid * 8 + j);
                s_prefix = prefix | (static_cast<unsigned long long>(digit) << shift);
                s_remaining = rem - acc;
                // every key with this prefix is a winner: the prefix itself
                // (lower bits zero) is a valid threshold
                if (acc + cnt[j] == rem) s_done = 1;
                break;
              }
              acc += cnt[j];
            }
          }
        }
        __syncthreads();
        mask |= 0xffULL << shift;
        if (s_done) break;
      }
      threshold = s_prefix;
    }

    // ---- gather keys > threshold, then fill with keys == threshold
    if (tid == 0) { s_count_gt = 0; s_count_eq = 0; }
    __syncthreads();
    for (int i = tid; i < n; i += blockDim.x) {
      const unsigned long long key = key_at(i);
      if (key > threshold || k == n) {
        const int pos = atomicAdd(&s_count_gt, 1);
        if (pos < k) keys[pos] = key;
      }
    }
    __syncthreads();
    const int gt = min(s_count_gt, k);
    if (gt < k) {
      for (int i = tid; i < n; i += blockDim.x) {
        const unsigned long long key = key_at(i);
        if (key == threshold) {
          const int pos = gt + atomicAdd(&s_count_eq, 1);
          if (pos < k) keys[pos] = key;
        }
      }
    }
    __syncthreads();

    int* out = selected + plan.sel_off[r];
    if (k <= 64) {
      // ---- up to 64 winners: one warp sorts them in registers (bitonic,
      // descending), lane l holding elements l and l + 32, zero-padded; no
      // block barriers
      if (tid < 32) {
        unsigned long long v[2] = {tid < k ? keys[tid] : 0ULL,
                                   tid + 32 < k ? keys[tid + 32] : 0ULL};
#pragma unroll
        for (int size = 2; size <= 64; size <<= 1) {
#pragma unroll
          for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride == 32) {
              // partners are the lane's two elements; size is 64, so descending
              if (v[0] < v[1]) { const unsigned long long t = v[0]; v[0] = v[1]; v[1] = t; }
            } else {
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int e = h * 32 + tid;
                const unsigned long long pv = __shfl_xor_sync(0xffffffffu, v[h], stride);
                const bool desc = (e & size) == 0;
                const bool lower = (tid & stride) == 0;
                const bool keep_max = desc == lower;
                v[h] = keep_max ? (v[h] > pv ? v[h] : pv) : (v[h] < pv ? v[h] : pv);
              }
            }
          }
        }
        if (tid < k) out[tid] = ~static_cast<int>(v[0] & 0xffffffffULL);
        if (tid + 32 < k) out[tid + 32] = ~static_cast<int>(v[1] & 0xffffffffULL);
      }
      __syncthreads();
      continue;
    }

    // ---- bitonic sort (descending) of the k winners, padded with zero keys
    int m = 1;
    while (m < k) m <<= 1;
    for (int i = k + tid; i < m; i += blockDim.x) keys[i] = 0ULL;
    __syncthreads();
    for (int size = 2; size <= m; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int i = tid; i < m; i += blockDim.x) {
          const int j = i ^ stride;
          if (j > i) {
            const unsigned long long a = keys[i], b = keys[j];
            const bool desc = (i & size) == 0;
            if (desc ? (a < b) : (a > b)) {
              keys[i] = b;
              keys[j] = a;
            }
          }
        }
        __syncthreads();
      }
    }
    for (int i = tid; i < k; i += blockDim.x) out[i] = ~static_cast<int>(keys[i] & 0xffffffffULL);
    __syncthreads();
  }
}

// ------------------------------------------------------------------ attention

// Walks this CTA's split-K work: units u = blockIdx.x + i*gridDim.x, each a
// run of up to `ppu` selected pages of one request; every non-empty page is
// cut into stages of up to `tps` tokens.  Producer and consumers walk the
// same sequence, the producer kScoreStages ahead.
struct AttnWalk {
  int u, p, p_end, page, n, t0;
  bool has_page;
};

__device__ __forceinline__ void attn_unit_range(const StepPlan& plan, int B, int ppu, int u,
                                                int* r_out, int* p_begin, int* p_end) {
  const int r = upper_segment(plan.unit_off, B, u);
  const int lu = u - plan.unit_off[r];
  const int sb = plan.sel_off[r];
  *r_out = r;
  *p_begin = sb + lu * ppu;
  *p_end = min(*p_begin + ppu, plan.sel_off[r + 1]);
}

__device__ __forceinline__ bool attn_walk_next(AttnWalk& w, const StepPlan& plan, int B,
                                               int total_units, int ppu, int tps, int page_size,
                                               const int* __restrict__ selected,
                                               const int* __restrict__ token_counts) {
  if (w.has_page) {
    if (w.t0 + tps < w.n) { w.t0 += tps; return true; }
    ++w.p;
  }
  w.has_page = false;
  for (;;) {
    if (w.p >= w.p_end) {
      w.u += gridDim.x;
      if (w.u >= total_units) return false;
      int r;
      attn_unit_range(plan, B, ppu, w.u, &r, &w.p, &w.p_end);
      continue;
    }
    w.page = __ldg(selected + w.p);
    w.n = min(__ldg(token_counts + w.page), page_size);
    w.t0 = 0;
    if (w.n > 0) { w.has_page = true; return true; }
    ++w.p;
  }
}

// Split-K flash decode.  CTA = 256 threads.  A head's D/4 float4 columns are
// split over LP = D/(4*NV) consecutive lanes ("items"), NV float4 each at
// stride LP (so the 8 lanes of a quarter warp read 8 consecutive float4 of
// shared memory: no bank conflicts at D = 128).  Item i = t + 256*m
// (m < SLOTS) is lane i % LP of head i / LP.  q.k is reduced over the LP
// lanes with xor shuffles, so every lane of a head holds the logit.
// Stages hold `tps` K rows then `tps` V rows of one page, fetched by thread 0
// with two cp.async.bulk copies (they are contiguous in the page-major pool)
// into a kAttnStages-deep mbarrier ring.  The online softmax is blocked per
// stage: all logits of the stage first, one rescale of the accumulator, then
// the weighted V rows.  Each unit writes (m, l) per head and acc[H*D].
template <int NV, int SLOTS>
__global__ void __launch_bounds__(kAttnThreads, 1) attn_kernel(
    StepPlan plan, const float* __restrict__ queries, const float* __restrict__ key_pool,
    const float* __restrict__ value_pool, const int* __restrict__ token_counts,
    const int* __restrict__ selected, float* __restrict__ part_acc, float* __restrict__ part_ml,
    int num_heads, int head_dim, int page_size, int tps, float scale, int part, int nparts) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  constexpr int kMaxTps = kAttnMaxTokensPerStage;
  const int ept = num_heads * head_dim;
  const int vec = ept >> 2;                       // float4 per token row
  const int G = head_dim >> 2;                    // float4 per head
  const int LP = G / NV;                          // lanes per head
  const size_t stage_floats = size_t(2) * tps * ept;
  float* stages = reinterpret_cast<float*>(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + kAttnStages * stage_floats * 4);

  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int s = 0; s < kAttnStages; ++s) mbar_init(&full[s], 1);
    fence_barrier_init();
  }
  __syncthreads();

  const int B = plan.hdr[0];
  int r_begin, r_end;
  part_range(B, part, nparts, &r_begin, &r_end);
  const int unit_begin = plan.unit_off[r_begin];
  const int total_units = plan.unit_off[r_end];
  const int ppu = plan.misc[0];
  const size_t page_floats = size_t(page_size) * ept;
  int* status = plan.status;

  AttnWalk w{unit_begin + static_cast<int>(blockIdx.x) - static_cast<int>(gridDim.x), 0, 0, 0, 0,
             0, false};
  uint32_t issued = 0;                            // thread 0: stages issued
  auto issue = [&](int s) {
    ++issued;
    const int nt = min(tps, w.n - w.t0);
    const uint32_t bytes = uint32_t(nt) * uint32_t(ept) * 4u;
    float* st = stages + size_t(s) * stage_floats;
    const size_t src = size_t(w.page) * page_floats + size_t(w.t0) * ept;
    mbar_arrive_expect_tx(&full[s], 2u * bytes);
    bulk_g2s(st, key_pool + src, bytes, &full[s]);
    bulk_g2s(st + size_t(tps) * ept, value_pool + src, bytes, &full[s]);
  };
  if (tid == 0) {
    for (int s = 0; s < kAttnStages; ++s) {
      if (!attn_walk_next(w, plan, B, total_units, ppu, tps, page_size, selected, token_counts))
        break;
      issue(s);
    }
  }

  // float4 column of (slot m, vector j) and whether the item is a real head lane
  int colv[SLOTS][NV];
  bool ok[SLOTS];
#pragma unroll
  for (int m = 0; m < SLOTS; ++m) {
    const int item = tid + kAttnThreads * m;
    const int head = item / LP, li = item - (item / LP) * LP;
    ok[m] = head < num_heads;
#pragma unroll
    for (int j = 0; j < NV; ++j) colv[m][j] = ok[m] ? head * G + li + LP * j : 0;
  }

  uint32_t g = 0;
  bool alive = true;
  for (int u = unit_begin + blockIdx.x; u < total_units && alive; u += gridDim.x) {
    int r, p_begin, p_end;
    attn_unit_range(plan, B, ppu, u, &r, &p_begin, &p_end);
    float4 q[SLOTS][NV], acc[SLOTS][NV];
    float mrun[SLOTS], lrun[SLOTS];
    const float4* qrow = reinterpret_cast<const float4*>(queries + size_t(r) * ept);
#pragma unroll
    for (int m = 0; m < SLOTS; ++m) {
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        q[m][j] = ok[m] ? __ldg(qrow + colv[m][j]) : make_float4(0.f, 0.f, 0.f, 0.f);
        acc[m][j] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      mrun[m] = -INFINITY;
      lrun[m] = 0.f;
    }
    for (int p = p_begin; p < p_end && alive; ++p) {
      const int page = __ldg(selected + p);
      const int n = min(__ldg(token_counts + page), page_size);
      for (int t0 = 0; t0 < n; t0 += tps, ++g) {
        const int s = g % kAttnStages;
        // Each thread waits with its own budget; a thread that gives up still
        // runs the stage (its shuffles need every lane) and the abort is
        // decided for the whole CTA at the stage's closing barrier.
        const bool gave_up = !mbar_wait(&full[s], (g / kAttnStages) & 1, status);
        const int nt = min(tps, n - t0);
        const float4* kst = reinterpret_cast<const float4*>(stages + size_t(s) * stage_floats);
        const float4* vst = kst + size_t(tps) * vec;
#pragma unroll
        for (int m = 0; m < SLOTS; ++m) {
          float logit[kMaxTps];
          float cmax = mrun[m];
#pragma unroll
          for (int t = 0; t < kMaxTps; ++t) {
            if (t < nt) {
              float d = 0.f;
#pragma unroll
              for (int j = 0; j < NV; ++j) {
                const float4 kk = kst[size_t(t) * vec + colv[m][j]];
                d += q[m][j].x * kk.x + q[m][j].y * kk.y + q[m][j].z * kk.z + q[m][j].w * kk.w;
              }
              for (int o = LP >> 1; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
              logit[t] = d * scale;
              cmax = fmaxf(cmax, logit[t]);
            }
          }
          const float alpha = expf(mrun[m] - cmax);
          float l = lrun[m] * alpha;
#pragma unroll
          for (int j = 0; j < NV; ++j) {
            acc[m][j].x *= alpha; acc[m][j].y *= alpha; acc[m][j].z *= alpha; acc[m][j].w *= alpha;
          }
#pragma unroll
          for (int t = 0; t < kMaxTps; ++t) {
            if (t < nt) {
              const float beta = expf(logit[t] - cmax);
              l += beta;
#pragma unroll
              for (int j = 0; j < NV; ++j) {
                const float4 vv = vst[size_t(t) * vec + colv[m][j]];
                acc[m][j].x += beta * vv.x; acc[m][j].y += beta * vv.y;
                acc[m][j].z += beta * vv.z; acc[m][j].w += beta * vv.w;
              }
            }
          }
          lrun[m] = l;
          mrun[m] = cmax;
        }
        // every thread is done with stage s; a timeout anywhere stops the CTA
        if (__syncthreads_or(gave_up)) { alive = false; break; }
        if (tid == 0) {
          if (attn_walk_next(w, plan, B, total_units, ppu, tps, page_size, selected, token_counts))
            issue(s);
        }
      }
    }
    // partial of unit u
#pragma unroll
    for (int m = 0; m < SLOTS; ++m) {
      if (!ok[m]) continue;
      float4* pa = reinterpret_cast<float4*>(part_acc + size_t(u) * ept);
#pragma unroll
      for (int j = 0; j < NV; ++j) pa[colv[m][j]] = acc[m][j];
      const int item = tid + kAttnThreads * m;
      if (item % LP == 0) {
        const int head = item / LP;
        part_ml[(size_t(u) * num_heads + head) * 2 + 0] = mrun[m];
        part_ml[(size_t(u) * num_heads + head) * 2 + 1] = lrun[m];
      }
    }
  }
  if (!alive && tid == 0) drain_ring(full, issued, kAttnStages, status);
}

// bf16 / fp8 pages: split-K flash decode with 16-byte vectors of VE = 8 bf16
// or 16 fp8 elements (a head's D/VE vectors over LP = D/(VE*NV) lanes, so the
// 8 lanes of a quarter warp read 128 contiguous bytes of one row) and fp32
// queries, logits, softmax and partials.  Warp-specialised: kAttnThreads consumer threads plus one
// producer warp whose lane 0 walks the CTA's units and keeps `nstages`
// stages (tps K rows then tps V rows of one page, two cp.async.bulk copies)
// in flight.  Consumers release a stage through its `empty` mbarrier (one
// arrival per consumer warp), so refills never wait for a CTA-wide barrier
// and the producer's page-table loads stay off the consumers' path.
constexpr int kAttnBfThreads = kAttnThreads + 32;
constexpr int kAttnBfRegTokens = 4;                 // tokens per narrow stage (V held in registers)
__host__ __device__ constexpr int attn_narrow_reg_tokens(int slots) {
  return slots == 1 ? kAttnBfRegTokens : 1;
}

// 16 bytes of page elements -> float2 pairs (elements 2h, 2h+1); widening is
// exact.  bf16: a 16-bit shift / mask; fp8 e4m3: via half (exact).
__device__ __forceinline__ void unpack16(const uint4 raw, const __nv_bfloat16*, float2 (&f)[4]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int h = 0; h < 4; ++h)
    f[h] = make_float2(__uint_as_float(w[h] << 16), __uint_as_float(w[h] & 0xffff0000u));
}
__device__ __forceinline__ void unpack16(const uint4 raw, const __nv_fp8_e4m3*, float2 (&f)[8]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    f[2 * h] = fp8x2_to_float2(w[h]);
    f[2 * h + 1] = fp8x2_to_float2(w[h] >> 16);
  }
}

// The narrow-page attention keeps its softmax in base 2: logits are scaled by
// log2(e) and weights come from the hardware 2^x approximation
// (ex2.approx.ftz, relative error ~2^-22); m is stored back in natural-log
// units.  2^(x*log2 e) = e^x, so the outputs are the same softmax.
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// CTAs per SM of the narrow attention kernel: fp8 consumers are bound by
// their per-element dependent chains (conversions, FMAs, softmax), so two
// CTAs with half-size rings (18 warps per SM) beat one with a full ring
// (config 3: attention 0.189 -> 0.148 ms); bf16 keeps one CTA, whose longer
// stage hold needs the deeper ring (two CTAs measured 0.183 -> 0.219 ms).
// Threads that serve two heads (SLOTS 2) need more registers than two CTAs
// leave, so they keep one CTA per SM.
__host__ __device__ constexpr int attn_narrow_ctas(int elem_bytes, int slots) {
  return elem_bytes == 1 && slots == 1 ? 2 : 1;
}
template <typename T, int NV, int SLOTS>
__global__ void __launch_bounds__(kAttnBfThreads, attn_narrow_ctas(int(sizeof(T)), SLOTS))
    attn_kernel_narrow(
    StepPlan plan, const float* __restrict__ queries, const T* __restrict__ key_pool,
    const T* __restrict__ value_pool, const int* __restrict__ token_counts,
    const int* __restrict__ selected, float* __restrict__ part_acc, float* __restrict__ part_ml,
    int num_heads, int head_dim, int page_size, int tps, int nstages, float scale, int part,
    int nparts) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  constexpr int kConsumerWarps = kAttnThreads / 32;
  // tokens per stage held in registers: fewer when a thread serves several
  // heads, so that V, q and the accumulators of all its slots stay within the
  // 168 registers a thread of a 9-warp CTA can have (3 warps per SM sub-partition)
  constexpr int RT = attn_narrow_reg_tokens(SLOTS);
  const int ept = num_heads * head_dim;
  constexpr int VE = 16 / int(sizeof(T));         // elements per 16-byte vector
  constexpr int VP = VE / 2;                      // float2 pairs per vector
  const int vec = ept / VE;                       // 16-byte vectors per token row
  const int G = head_dim / VE;                    // vectors per head
  const int LP = G / NV;                          // lanes per head
  const size_t stage_elems = size_t(2) * tps * ept;
  T* stages = reinterpret_cast<T*>(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + nstages * stage_elems * sizeof(T));
  uint64_t* empty = full + nstages;
  __shared__ volatile int abort;                  // raised by the first waiter that gives up

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const float scale_log2 = scale * kLog2e;
  if (tid == 0) {
    for (int s = 0; s < nstages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_barrier_init();
    abort = 0;
  }
  __syncthreads();

  const int B = plan.hdr[0];
  int r_begin, r_end;
  part_range(B, part, nparts, &r_begin, &r_end);
  const int unit_begin = plan.unit_off[r_begin];
  const int total_units = plan.unit_off[r_end];
  const int ppu = plan.misc[0];
  int* status = plan.status;

  if (tid >= kAttnThreads) {
    // ---- producer warp
    if (lane == 0) {
      const size_t page_elems = size_t(page_size) * ept;
      AttnWalk w{unit_begin + static_cast<int>(blockIdx.x) - static_cast<int>(gridDim.x), 0, 0,
                 0, 0, 0, false};
      uint32_t g = 0;
      for (;; ++g) {
        if (!attn_walk_next(w, plan, B, total_units, ppu, tps, page_size, selected, token_counts))
          break;
        const int s = g % nstages;
        const uint32_t use = g / nstages;
        if (use > 0 && !mbar_wait_or_abort(&empty[s], (use - 1) & 1, status, &abort)) break;
        const int nt = min(tps, w.n - w.t0);
        const uint32_t bytes = uint32_t(nt) * uint32_t(ept) * uint32_t(sizeof(T));
        T* st = stages + size_t(s) * stage_elems;
        const size_t src = size_t(w.page) * page_elems + size_t(w.t0) * ept;
        mbar_arrive_expect_tx(&full[s], 2u * bytes);
        bulk_g2s(st, key_pool + src, bytes, &full[s]);
        bulk_g2s(st + size_t(tps) * ept, value_pool + src, bytes, &full[s]);
      }
      // Normal end: stay until the consumers have released the last stages,
      // so that an abort raised by a consumer after the last issue is seen.
      // On an abort, no copy may still be writing shared memory at exit.
      const uint32_t first = g > uint32_t(nstages) ? g - uint32_t(nstages) : 0u;
      for (uint32_t i = first; i < g && !abort; ++i)
        mbar_wait_or_abort(&empty[i % uint32_t(nstages)], (i / uint32_t(nstages)) & 1u, status,
                           &abort);
      if (abort) drain_ring(full, g, nstages, status);
    }
    return;
  }

  // ---- consumers
  int colv[SLOTS][NV];
  bool ok[SLOTS];
#pragma unroll
  for (int m = 0; m < SLOTS; ++m) {
    const int item = tid + kAttnThreads * m;
    const int head = item / LP, li = item - (item / LP) * LP;
    ok[m] = head < num_heads;
#pragma unroll
    for (int j = 0; j < NV; ++j) colv[m][j] = ok[m] ? head * G + li + LP * j : 0;
  }

  // The unit's request, page range, per-page token counts (lane j of every
  // warp holds page j's count) and this thread's query pieces are loaded one
  // unit ahead, so no global-load latency sits between two units.
  // Query element pairs (2x, 2x+1) are float2 for the packed f32x2 math.
  float2 nq[SLOTS][NV][VP];
  auto unit_info = [&](int uu, int& rr, int& pb, int& pe) {
    attn_unit_range(plan, B, ppu, uu, &rr, &pb, &pe);
    const float4* qrow = reinterpret_cast<const float4*>(queries + size_t(rr) * ept);
#pragma unroll
    for (int m = 0; m < SLOTS; ++m) {
#pragma unroll
      for (int j = 0; j < NV; ++j) {
#pragma unroll
        for (int h = 0; h < VE / 4; ++h) {
          const float4 a =
              ok[m] ? __ldg(qrow + (VE / 4) * colv[m][j] + h) : make_float4(0.f, 0.f, 0.f, 0.f);
          nq[m][j][2 * h] = make_float2(a.x, a.y);
          nq[m][j][2 * h + 1] = make_float2(a.z, a.w);
        }
      }
    }
    return pb + lane < pe ? min(__ldg(token_counts + __ldg(selected + pb + lane)), page_size) : 0;
  };
  int nx_r = 0, nx_pb = 0, nx_pe = 0, nx_cnt = 0;
  if (unit_begin + static_cast<int>(blockIdx.x) < total_units)
    nx_cnt = unit_info(unit_begin + blockIdx.x, nx_r, nx_pb, nx_pe);

  uint32_t g = 0;
  bool alive = true;
  for (int u = unit_begin + blockIdx.x; u < total_units && alive; u += gridDim.x) {
    const int p_begin = nx_pb, p_end = nx_pe, cnt = nx_cnt;
    float2 q[SLOTS][NV][VP], acc[SLOTS][NV][VP];
    float mrun[SLOTS], lrun[SLOTS];
#pragma unroll
    for (int m = 0; m < SLOTS; ++m) {
#pragma unroll
      for (int j = 0; j < NV; ++j) {
#pragma unroll
        for (int x = 0; x < VP; ++x) {
          q[m][j][x] = nq[m][j][x];
          acc[m][j][x] = make_float2(0.f, 0.f);
        }
      }
      mrun[m] = -INFINITY;
      lrun[m] = 0.f;
    }
    if (u + static_cast<int>(gridDim.x) < total_units)
      nx_cnt = unit_info(u + gridDim.x, nx_r, nx_pb, nx_pe);
    for (int p = p_begin; p < p_end && alive; ++p) {
      const int n = __shfl_sync(0xffffffffu, cnt, p - p_begin);
      for (int t0 = 0; t0 < n; t0 += tps, ++g) {
        const int s = g % nstages;
        // the warp leaves together (its shuffles need every lane), and the
        // shared flag takes the other warps and the producer with it
        const bool got = mbar_wait_or_abort(&full[s], (g / nstages) & 1, status, &abort);
        if (!__all_sync(0xffffffffu, got)) { abort = 1; alive = false; break; }
        const int nt = min(tps, n - t0);
        const uint4* kst = reinterpret_cast<const uint4*>(stages + size_t(s) * stage_elems);
        const uint4* vst = kst + size_t(tps) * vec;
        // V pieces go to registers and this lane's q.k partials are formed
        // from K in place; then the stage is released, before the cross-lane
        // reduction, the softmax and the V accumulation.  A stage is held only
        // for its shared-memory reads and the partial dot products, so more of
        // the ring stays in flight.
        uint4 vreg[SLOTS][RT][NV];
        float logit[SLOTS][RT];
#pragma unroll
        for (int m = 0; m < SLOTS; ++m) {
#pragma unroll
          for (int t = 0; t < RT; ++t) {
            if (t < nt) {
              float2 d2 = make_float2(0.f, 0.f);
#pragma unroll
              for (int j = 0; j < NV; ++j) {
                vreg[m][t][j] = vst[size_t(t) * vec + colv[m][j]];
                float2 kk[VP];
                unpack16(kst[size_t(t) * vec + colv[m][j]], static_cast<const T*>(nullptr), kk);
#pragma unroll
                for (int x = 0; x < VP; ++x) d2 = __ffma2_rn(q[m][j][x], kk[x], d2);
              }
              logit[m][t] = d2.x + d2.y;
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);   // release: this warp's reads are done
#pragma unroll
        for (int m = 0; m < SLOTS; ++m) {
#pragma unroll
          for (int t = 0; t < RT; ++t) {
            if (t < nt) {
              float d = logit[m][t];
              for (int o = LP >> 1; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
              logit[m][t] = d * scale_log2;     // base-2 logits
            }
          }
        }
#pragma unroll
        for (int m = 0; m < SLOTS; ++m) {
          float cmax = mrun[m];
#pragma unroll
          for (int t = 0; t < RT; ++t)
            if (t < nt) cmax = fmaxf(cmax, logit[m][t]);
          const float alpha = fast_exp2(mrun[m] - cmax);
          float l = lrun[m] * alpha;
          const float2 alpha2 = make_float2(alpha, alpha);
#pragma unroll
          for (int j = 0; j < NV; ++j)
#pragma unroll
            for (int x = 0; x < VP; ++x) acc[m][j][x] = __fmul2_rn(acc[m][j][x], alpha2);
#pragma unroll
          for (int t = 0; t < RT; ++t) {
            if (t < nt) {
              const float beta = fast_exp2(logit[m][t] - cmax);
              l += beta;
              const float2 beta2 = make_float2(beta, beta);
#pragma unroll
              for (int j = 0; j < NV; ++j) {
                float2 vv[VP];
                unpack16(vreg[m][t][j], static_cast<const T*>(nullptr), vv);
#pragma unroll
                for (int x = 0; x < VP; ++x) acc[m][j][x] = __ffma2_rn(beta2, vv[x], acc[m][j][x]);
              }
            }
          }
          lrun[m] = l;
          mrun[m] = cmax;
        }
      }
    }
#pragma unroll
    for (int m = 0; m < SLOTS; ++m) {
      if (!ok[m]) continue;
      float4* pa = reinterpret_cast<float4*>(part_acc + size_t(u) * ept);
#pragma unroll
      for (int j = 0; j < NV; ++j) {
#pragma unroll
        for (int h = 0; h < VE / 4; ++h)
          pa[(VE / 4) * colv[m][j] + h] = make_float4(acc[m][j][2 * h].x, acc[m][j][2 * h].y,
                                                      acc[m][j][2 * h + 1].x,
                                                      acc[m][j][2 * h + 1].y);
      }
      const int item = tid + kAttnThreads * m;
      if (item % LP == 0) {
        const int head = item / LP;
        // back to natural-log units for the combine kernel
        part_ml[(size_t(u) * num_heads + head) * 2 + 0] = mrun[m] * kLn2;
        part_ml[(size_t(u) * num_heads + head) * 2 + 1] = lrun[m];
      }
    }
  }
}

// One warp per (request, head): out = sum_u e^{m_u-M} acc_u / sum_u e^{m_u-M} l_u,
// zero when the request attended to no token (SparseAttentionCpu returns zeros).
// Units are taken 32 at a time: lane i loads unit i's (m, l) once, the warp
// reduces M and L, lane i keeps its unit's weight e^{m_i-M}, and each lane
// then sums its float4 columns over the units with the weights broadcast by
// shuffles (the partial loads of a chunk are independent, so they overlap).
__global__ void __launch_bounds__(256) combine_kernel(StepPlan plan,
                                                      const float* __restrict__ part_acc,
                                                      const float* __restrict__ part_ml,
                                                      int num_heads, int head_dim,
                                                      float* __restrict__ outputs, int part,
                                                      int nparts) {
  const int B = plan.hdr[0];
  const int lane = threadIdx.x & 31;
  const int ept = num_heads * head_dim;
  int r_begin, r_end;
  part_range(B, part, nparts, &r_begin, &r_end);
  const int pairs = r_end * num_heads;
  const int g4 = head_dim >> 2;
  for (int wg = r_begin * num_heads + ((blockIdx.x * blockDim.x + threadIdx.x) >> 5); wg < pairs;
       wg += (gridDim.x * blockDim.x) >> 5) {
    const int r = wg / num_heads, h = wg - (wg / num_heads) * num_heads;
    const int u0 = plan.unit_off[r], u1 = plan.unit_off[r + 1];
    float4* out = reinterpret_cast<float4*>(outputs + size_t(r) * ept + size_t(h) * head_dim);
    // M over all units (one pass over the (m, l) pairs; this lane's first
    // chunk stays in registers)
    float m0 = -INFINITY, l0 = 0.f;
    if (u0 + lane < u1) {
      const float2 ml =
          *reinterpret_cast<const float2*>(part_ml + (size_t(u0 + lane) * num_heads + h) * 2);
      m0 = ml.x;
      l0 = ml.y;
    }
    float M = m0;
    for (int u = u0 + 32 + lane; u < u1; u += 32)
      M = fmaxf(M, part_ml[(size_t(u) * num_heads + h) * 2]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    if (M == -INFINITY) {
      for (int d = lane; d < g4; d += 32) out[d] = make_float4(0.f, 0.f, 0.f, 0.f);
      continue;
    }
    // float4 columns lane and lane + 32 (head_dim <= 256)
    float4 acc[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
    float L = 0.f;
    const bool col[2] = {lane < g4, lane + 32 < g4};
    for (int c0 = u0; c0 < u1; c0 += 32) {
      float w = 0.f;
      if (c0 == u0) {
        w = u0 + lane < u1 ? expf(m0 - M) : 0.f;
        L += l0 * w;
      } else if (c0 + lane < u1) {
        const float2 ml =
            *reinterpret_cast<const float2*>(part_ml + (size_t(c0 + lane) * num_heads + h) * 2);
        w = expf(ml.x - M);
        L += ml.y * w;
      }
      const int nu = min(32, u1 - c0);
      const float* base = part_acc + size_t(c0) * ept + size_t(h) * head_dim + 4 * lane;
      for (int cc = 0; cc < 2; ++cc) {
        if (!__any_sync(0xffffffffu, col[cc])) break;   // the same g4 on every lane
        const float* cb = base + 128 * cc;
        int i = 0;
        for (; i + 4 <= nu; i += 4) {
          float4 a[4];
#pragma unroll
          for (int k = 0; k < 4; ++k)
            a[k] = col[cc] ? *reinterpret_cast<const float4*>(cb + size_t(i + k) * ept)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float wk = __shfl_sync(0xffffffffu, w, i + k);
            acc[cc].x += wk * a[k].x; acc[cc].y += wk * a[k].y;
            acc[cc].z += wk * a[k].z; acc[cc].w += wk * a[k].w;
          }
        }
        for (; i < nu; ++i) {
          const float4 a = col[cc] ? *reinterpret_cast<const float4*>(cb + size_t(i) * ept)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
          const float wk = __shfl_sync(0xffffffffu, w, i);
          acc[cc].x += wk * a.x; acc[cc].y += wk * a.y; acc[cc].z += wk * a.z;
          acc[cc].w += wk * a.w;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    const float inv = L > 0.f ? 1.0f / L : 0.0f;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc)
      if (col[cc])
        out[lane + 32 * cc] =
            L > 0.f ? make_float4(acc[cc].x * inv, acc[cc].y * inv, acc[cc].z * inv,
                                  acc[cc].w * inv)
                    : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// ------------------------------------------------------------------ pool maintenance

// Scatter packed pages from a staging buffer into the pool and compute the
// summary with PagedKvCache::AppendPage's formula (src/paged_kv_cache.cpp:88-99):
// token-order sum, then * (1.0f / n), both rounded to nearest, no FMA.
// grid (pages, ceil(E/4/256)); thread = one float4 column.
template <typename T>
__global__ void upload_pages_kernel(const int* __restrict__ page_ids,
                                    const int* __restrict__ counts,
                                    const long long* __restrict__ src_token_off,
                                    const float* __restrict__ staged_k,
                                    const float* __restrict__ staged_v, int ept, int page_size,
                                    int compute_summary, T* __restrict__ key_pool,
                                    T* __restrict__ value_pool, T* __restrict__ summaries,
                                    int* __restrict__ token_counts, uint8_t* __restrict__ live) {
  const int i = blockIdx.x;
  const int j = blockIdx.y * blockDim.x + threadIdx.x;
  const int vec = ept >> 2;
  const int page = page_ids[i];
  const int n = counts[i];
  if (j < vec) {
    const float4* sk = reinterpret_cast<const float4*>(staged_k + src_token_off[i] * ept);
    const float4* sv = reinterpret_cast<const float4*>(staged_v + src_token_off[i] * ept);
    T* dk = key_pool + size_t(page) * page_size * ept;
    T* dv = value_pool + size_t(page) * page_size * ept;
    float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int t = 0; t < n; ++t) {
      // the stored (rounded) key is what the summary averages
      const float4 k = Kv<T>::round4(sk[size_t(t) * vec + j]);
      Kv<T>::store4(dk + (size_t(t) * vec + j) * 4, k);
      Kv<T>::store4(dv + (size_t(t) * vec + j) * 4, sv[size_t(t) * vec + j]);
      sum.x = __fadd_rn(sum.x, k.x);
      sum.y = __fadd_rn(sum.y, k.y);
      sum.z = __fadd_rn(sum.z, k.z);
      sum.w = __fadd_rn(sum.w, k.w);
    }
    float4 out = make_float4(0.f, 0.f, 0.f, 0.f);
    if (compute_summary && n > 0) {
      const float inv = __fdiv_rn(1.0f, static_cast<float>(n));
      out = make_float4(__fmul_rn(sum.x, inv), __fmul_rn(sum.y, inv), __fmul_rn(sum.z, inv),
                        __fmul_rn(sum.w, inv));
    }
    Kv<T>::store4(summaries + summary_off(page, 4 * j, ept), out);
  }
  if (blockIdx.y == 0 && threadIdx.x == 0) {
    token_counts[page] = n;
    live[page] = 1;
  }
}

template <typename T>
__global__ void set_summaries_kernel(const int* __restrict__ page_ids,
                                     const float* __restrict__ staged, int ept,
                                     T* __restrict__ summaries) {
  const int i = blockIdx.x;
  const int page = page_ids[i];
  for (int e = threadIdx.x; e < ept; e += blockDim.x)
    Kv<T>::put(summaries, summary_off(page, e, ept), staged[size_t(i) * ept + e]);
}

// Token append.  One block per distinct page; its tokens (token_first[i] ..
// token_first[i+1]) are applied in offset order with PagedKvCache::AppendToken's
// running mean (src/paged_kv_cache.cpp:231-238): s = (s*old + k) / (old + 1).
// Optional page-table entries (slot, position, page) are written first.
template <typename T>
__global__ void append_tokens_kernel(const int* __restrict__ group_page,
                                     const int* __restrict__ token_first,
                                     const int* __restrict__ token_offset,
                                     const float* __restrict__ staged_k,
                                     const float* __restrict__ staged_v, int ept, int page_size,
                                     T* __restrict__ key_pool, T* __restrict__ value_pool,
                                     T* __restrict__ summaries, int* __restrict__ token_counts,
                                     uint8_t* __restrict__ live) {
  const int gidx = blockIdx.x;
  const int page = group_page[gidx];
  const size_t sbase = summary_row_base(page, ept);
  const int scw = summary_chunk(ept);
  int last = -1;
  for (int i = token_first[gidx]; i < token_first[gidx + 1]; ++i) {
    const int off = token_offset[i];
    const float old_c = static_cast<float>(off);
    const float new_c = __fadd_rn(old_c, 1.0f);
    T* dk = key_pool + (size_t(page) * page_size + off) * ept;
    T* dv = value_pool + (size_t(page) * page_size + off) * ept;
    for (int e = threadIdx.x; e < ept; e += blockDim.x) {
      const float k = Kv<T>::round(staged_k[size_t(i) * ept + e]);
      Kv<T>::put(dk, e, k);
      Kv<T>::put(dv, e, staged_v[size_t(i) * ept + e]);
      const size_t so = sbase + size_t(e / scw) * 128 * scw + (e % scw);
      const float s = off == 0 ? 0.0f : Kv<T>::get(summaries, so);
      Kv<T>::put(summaries, so, __fdiv_rn(__fadd_rn(__fmul_rn(s, old_c), k), new_c));
    }
    last = max(last, off);
  }
  if (threadIdx.x == 0 && last >= 0) {
    token_counts[page] = last + 1;
    live[page] = 1;
  }
}

__global__ void table_write_kernel(const int* __restrict__ entries, int n, int stride,
                                   int* __restrict__ table, int* __restrict__ table_n) {
  // entries: triples (slot, position, page)
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int slot = entries[3 * i], pos = entries[3 * i + 1], page = entries[3 * i + 2];
  table[size_t(slot) * stride + pos] = page;
  atomicMax(table_n + slot, pos + 1);
}

__global__ void table_set_count_kernel(const int* __restrict__ pairs, int n,
                                       int* __restrict__ table_n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) table_n[pairs[2 * i]] = pairs[2 * i + 1];
}

// DevicePagePool::MarkPagesFree: count 0, not live, summary zeroed.
template <typename T>
__global__ void free_pages_kernel(const int* __restrict__ page_ids, int ept,
                                  T* __restrict__ summaries, int* __restrict__ token_counts,
                                  uint8_t* __restrict__ live) {
  const int page = page_ids[blockIdx.x];
  for (int e = threadIdx.x; e < ept; e += blockDim.x)
    Kv<T>::put(summaries, summary_off(page, e, ept), 0.0f);
  if (threadIdx.x == 0) {
    token_counts[page] = 0;
    live[page] = 0;
  }
}

// The reference's synthetic prompt / decode payload hash
// (src/device_page_pool.cpp:102-138): boost-style combine of the indices,
// a 32-bit finaliser, then (x % 2001 - 1000) / 1000.
__device__ __forceinline__ uint32_t combine_hash(uint32_t x, int v, uint32_t salt) {
  return x ^ (static_cast<uint32_t>(v + static_cast<int>(salt)) + (x << 6) + (x >> 2));
}
__device__ __forceinline__ float hash_to_unit(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return static_cast<float>(static_cast<int>(x % 2001u) - 1000) / 1000.0f;
}
// (x % 2001 - 1000) / 1000 as a lookup: lut[i] holds (i - 1000) / 1000.0f,
// computed once per block with the same IEEE round-to-nearest division.
constexpr int kUnitLut = 2001;
__device__ __forceinline__ void fill_unit_lut(float* lut) {
  for (int i = threadIdx.x; i < kUnitLut; i += blockDim.x)
    lut[i] = __fdiv_rn(static_cast<float>(i - 1000), 1000.0f);
}
__device__ __forceinline__ float hash_to_unit_lut(uint32_t x, const float* lut) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return lut[x % 2001u];
}
__device__ __forceinline__ float prompt_value(int request, int page_idx, int token, int element,
                                              int stream) {
  uint32_t x = 0x9e3779b9u;
  x = combine_hash(x, request, 0x85ebca6bu);
  x = combine_hash(x, page_idx, 0xc2b2ae35u);
  x = combine_hash(x, token, 0x27d4eb2fu);
  x = combine_hash(x, element, 0x165667b1u);
  x = combine_hash(x, stream, 0xd3a2646cu);
  return hash_to_unit(x);
}
__device__ __forceinline__ float decode_value(int request, int step, int element, int stream) {
  uint32_t x = 0x9e3779b9u;
  x = combine_hash(x, request, 0x85ebca6bu);
  x = combine_hash(x, step, 0xc2b2ae35u);
  x = combine_hash(x, element, 0x165667b1u);
  x = combine_hash(x, stream, 0xd3a2646cu);
  return hash_to_unit(x);
}

// Synthetic prefill: page i is page_idx i of `request`; summary by AppendPage's formula.
// The key (stream 1) and value (stream 2) hashes share every combine step but
// the last, so the shared prefix is computed once per element and token.
// Element e of a pool row (physical head width hdp) -> its index in the
// caller's row (head width hd <= hdp), or -1 for padding columns.
__device__ __forceinline__ int logical_element(int e, int hd, int hdp) {
  const int h = e / hdp, d = e - h * hdp;
  return d < hd ? h * hd + d : -1;
}

template <typename T>
__global__ void prefill_synthetic_kernel(const int* __restrict__ page_ids,
                                         const int* __restrict__ counts, int request, int ept,
                                         int hd, int hdp, int page_size, T* __restrict__ key_pool,
                                         T* __restrict__ value_pool,
                                         T* __restrict__ summaries,
                                         int* __restrict__ token_counts,
                                         uint8_t* __restrict__ live) {
  __shared__ float lut[kUnitLut];
  fill_unit_lut(lut);
  __syncthreads();
  const int i = blockIdx.x;
  const int page = page_ids[i];
  const int n = counts[i];
  uint32_t xr = 0x9e3779b9u;
  xr = combine_hash(xr, request, 0x85ebca6bu);
  xr = combine_hash(xr, i, 0xc2b2ae35u);
  for (int e = threadIdx.x; e < ept; e += blockDim.x) {
    const int el = logical_element(e, hd, hdp);   // -1: padding
    float sum = 0.0f;
#pragma unroll 4
    for (int t = 0; t < n; ++t) {
      if (el < 0) {
        Kv<T>::put(key_pool, (size_t(page) * page_size + t) * ept + e, 0.0f);
        Kv<T>::put(value_pool, (size_t(page) * page_size + t) * ept + e, 0.0f);
        continue;
      }
      uint32_t x = combine_hash(xr, t, 0x27d4eb2fu);
      x = combine_hash(x, el, 0x165667b1u);
      const float k = Kv<T>::round(hash_to_unit_lut(combine_hash(x, 1, 0xd3a2646cu), lut));
      const float v = hash_to_unit_lut(combine_hash(x, 2, 0xd3a2646cu), lut);
      Kv<T>::put(key_pool, (size_t(page) * page_size + t) * ept + e, k);
      Kv<T>::put(value_pool, (size_t(page) * page_size + t) * ept + e, v);
      sum = __fadd_rn(sum, k);
    }
    Kv<T>::put(summaries, summary_off(page, e, ept),
               n > 0 ? __fmul_rn(sum, __fdiv_rn(1.0f, static_cast<float>(n))) : 0.0f);
  }
  if (threadIdx.x == 0) {
    token_counts[page] = n;
    live[page] = 1;
  }
}

// Synthetic append: token i = decode step steps[i] of request reqs[i].
template <typename T>
__global__ void append_synthetic_kernel(const int* __restrict__ group_page,
                                        const int* __restrict__ token_first,
                                        const int* __restrict__ token_offset,
                                        const int* __restrict__ reqs, const int* __restrict__ steps,
                                        int ept, int hd, int hdp, int page_size,
                                        T* __restrict__ key_pool,
                                        T* __restrict__ value_pool,
                                        T* __restrict__ summaries,
                                        int* __restrict__ token_counts,
                                        uint8_t* __restrict__ live) {
  const int gidx = blockIdx.x;
  const int page = group_page[gidx];
  const size_t sbase = summary_row_base(page, ept);
  const int scw = summary_chunk(ept);
  int last = -1;
  for (int i = token_first[gidx]; i < token_first[gidx + 1]; ++i) {
    const int off = token_offset[i];
    const float old_c = static_cast<float>(off);
    const float new_c = __fadd_rn(old_c, 1.0f);
    for (int e = threadIdx.x; e < ept; e += blockDim.x) {
      const int el = logical_element(e, hd, hdp);   // -1: padding (stays zero)
      const float k = el < 0 ? 0.0f : Kv<T>::round(decode_value(reqs[i], steps[i], el, 1));
      Kv<T>::put(key_pool, (size_t(page) * page_size + off) * ept + e, k);
      Kv<T>::put(value_pool, (size_t(page) * page_size + off) * ept + e,
                 el < 0 ? 0.0f : decode_value(reqs[i], steps[i], el, 2));
      const size_t so = sbase + size_t(e / scw) * 128 * scw + (e % scw);
      const float s = off == 0 ? 0.0f : Kv<T>::get(summaries, so);
      Kv<T>::put(summaries, so, __fdiv_rn(__fadd_rn(__fmul_rn(s, old_c), k), new_c));
    }
    last = max(last, off);
  }
  if (threadIdx.x == 0 && last >= 0) {
    token_counts[page] = last + 1;
    live[page] = 1;
  }
}

// Counter-based normal workload: Irwin-Hall(4) of 16-bit uniforms from a
// splitmix64-style mix of (seed, kind, index).  Integer sum, one conversion,
// one multiply: bit-identical on host and device.
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}
__host__ __device__ __forceinline__ float normal_value(uint64_t seed_mix, uint64_t index) {
  const uint64_t h = mix64(index ^ seed_mix);
  const int sum = static_cast<int>(h & 0xffff) + static_cast<int>((h >> 16) & 0xffff) +
                  static_cast<int>((h >> 32) & 0xffff) + static_cast<int>((h >> 48) & 0xffff);
#ifdef __CUDA_ARCH__
  return __fmul_rn(static_cast<float>(sum - 131070), 2.6429e-5f);
#else
  return static_cast<float>(sum - 131070) * 2.6429e-5f;
#endif
}
__host__ __device__ __forceinline__ uint64_t normal_seed_mix(uint64_t seed, int kind) {
  return mix64(seed * 0x9e3779b97f4a7c15ULL + static_cast<uint64_t>(kind));
}
__host__ __device__ __forceinline__ uint64_t normal_index(int request, long long token, int ept,
                                                          int element) {
  return (static_cast<uint64_t>(request) << 40) + static_cast<uint64_t>(token) * ept +
         static_cast<uint64_t>(element);
}

// grid (pages, ceil(E/256)); thread = one element column of one page.
template <typename T>
__global__ void generate_normal_kernel(const int* __restrict__ page_ids,
                                       const int* __restrict__ counts,
                                       const int* __restrict__ reqs,
                                       const int* __restrict__ first_token, int ept, int hd,
                                       int hdp, int page_size, uint64_t kmix, uint64_t vmix,
                                       T* __restrict__ key_pool,
                                       T* __restrict__ value_pool,
                                       T* __restrict__ summaries,
                                       int* __restrict__ token_counts,
                                       uint8_t* __restrict__ live) {
  const int i = blockIdx.x;
  const int e = blockIdx.y * blockDim.x + threadIdx.x;
  const int page = page_ids[i];
  const int n = counts[i];
  if (e < ept) {
    const int el = logical_element(e, hd, hdp);   // -1: padding
    const int lept = ept / hdp * hd;               // the caller's row length
    float sum = 0.0f;
    for (int t = 0; t < n; ++t) {
      const uint64_t idx = normal_index(reqs[i], first_token[i] + t, lept, max(el, 0));
      const float k = el < 0 ? 0.0f : Kv<T>::round(normal_value(kmix, idx));
      Kv<T>::put(key_pool, (size_t(page) * page_size + t) * ept + e, k);
      Kv<T>::put(value_pool, (size_t(page) * page_size + t) * ept + e,
                 el < 0 ? 0.0f : normal_value(vmix, idx));
      sum = __fadd_rn(sum, k);
    }
    Kv<T>::put(summaries, summary_off(page, e, ept),
               n > 0 ? __fmul_rn(sum, __fdiv_rn(1.0f, static_cast<float>(n))) : 0.0f);
  }
  if (blockIdx.y == 0 && threadIdx.x == 0) {
    token_counts[page] = n;
    live[page] = 1;
  }
}

}  // namespace dsdk
