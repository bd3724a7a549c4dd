// dsd_capi.cu -- the C ABI (include/dsd_b200.h) over the sm_100a kernels.
//
// A context is one GPU's share of the decode service: its page pool, the
// per-step scratch (sized once at creation; a step allocates nothing), one
// stream, pinned staging for the packed per-step H2D/D2H copies, the device
// request page tables and a host mirror of those tables.
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <initializer_list>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <thread>
#include <type_traits>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "dsd_b200.h"
#include "dsd_kernels.cuh"

namespace {

thread_local std::string g_last_error;

// NVTX range over a host-side phase (entry points, and each stage of the step
// while it is launched or captured), the counterpart of the reference's
// ScopedStageTimer stages in a profiler timeline.  Header-only NVTX: without
// an attached tool each push/pop is a no-op call.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

struct DsdError {
  int code;
  std::string msg;
};

[[noreturn]] void Fail(int code, const std::string& msg) { throw DsdError{code, msg}; }

void Check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    Fail(DSD_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
  }
}

template <typename F>
int Guard(F&& f) {
  try {
    f();
    return DSD_OK;
  } catch (const DsdError& e) {
    g_last_error = e.msg;
    return e.code;
  } catch (const std::bad_alloc&) {
    g_last_error = "host allocation failed";
    return DSD_ENOMEM;
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return DSD_EINVAL;
  }
}

constexpr size_t kLargeCopyBytes = size_t(1) << 20;  // DeviceTransferStats "large" threshold

template <typename T>
T* DeviceAlloc(size_t count, const char* what) {
  void* p = nullptr;
  const size_t bytes = std::max<size_t>(1, count) * sizeof(T);
  const cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    Fail(DSD_ENOMEM, std::string("cudaMalloc failed for ") + what + " (" +
                         std::to_string(bytes) + " bytes): " + cudaGetErrorString(e));
  }
  return static_cast<T*>(p);
}

template <typename T>
T* PinnedAlloc(size_t count, const char* what) {
  void* p = nullptr;
  const cudaError_t e = cudaMallocHost(&p, std::max<size_t>(1, count) * sizeof(T));
  if (e != cudaSuccess) {
    cudaGetLastError();
    Fail(DSD_ENOMEM, std::string("cudaMallocHost failed for ") + what);
  }
  return static_cast<T*>(p);
}

size_t AlignUp(size_t x, size_t a) { return (x + a - 1) / a * a; }

// fp8 e4m3 (1 sign, 4 exponent bits with bias 7, 3 mantissa bits; S.1111.111
// is NaN, no infinities) to float, exactly.
float Fp8E4m3ToFloat(unsigned char b) {
  const int sign = b >> 7, exp = (b >> 3) & 15, man = b & 7;
  float v;
  if (exp == 15 && man == 7) v = std::nanf("");
  else if (exp == 0) v = std::ldexp(static_cast<float>(man), -9);        // subnormal: m/8 * 2^-6
  else v = std::ldexp(static_cast<float>(8 + man), exp - 10);           // (1 + m/8) * 2^(e-7)
  return sign ? -v : v;
}


// Attention launch shape: NV float4 per lane, LP = D/(4*NV) lanes per head,
// SLOTS items per thread, tokens per stage and dynamic shared memory.
struct AttnShape {
  int nv = 1, slots = 1, tps = 1, nstages = 0;
  int ctas = 1;       // narrow attention CTAs per SM
  size_t smem = 0;
};

AttnShape MakeAttnShape(int num_heads, int head_dim, int page_size, int elem_bytes = 4) {
  AttnShape a;
  const int ept = num_heads * head_dim;
  if (elem_bytes < 4) {
    // 16-byte vectors of VE = 16/elem_bytes elements, at most 16 elements per
    // lane: bf16 NV = 2 (head_dim >= 16) or 1 (head_dim 8); fp8 NV = 1
    const int VE = 16 / elem_bytes;
    const int G = head_dim / VE;
    a.nv = std::max(1, std::min(G, 16 / VE));
    const int items = num_heads * (G / a.nv);
    const int slots = (items + dsdk::kAttnThreads - 1) / dsdk::kAttnThreads;
    if (slots > 4) Fail(DSD_EINVAL, "num_heads*head_dim is too large for the attention kernel");
    a.slots = slots <= 1 ? 1 : slots <= 2 ? 2 : 4;
    a.ctas = dsdk::attn_narrow_ctas(elem_bytes, a.slots);
    // 32 KiB stages, as many as fit in ~200 KiB per SM (at most 8), shared by
    // the format's CTAs per SM
    a.tps = std::max(1, std::min({page_size, 65536 / (2 * ept * elem_bytes),
                                  dsdk::attn_narrow_reg_tokens(a.slots)}));
    const size_t stage = size_t(2) * a.tps * ept * elem_bytes;
    a.nstages = int(std::max<size_t>(2, std::min<size_t>(8, (size_t(200u / a.ctas) << 10) / stage)));
    a.smem = size_t(a.nstages) * (stage + 16);
    return a;
  }
  const int G = head_dim / 4;
  a.nv = G >= 4 ? 4 : G;
  const int items = num_heads * (G / a.nv);
  const int slots = (items + dsdk::kAttnThreads - 1) / dsdk::kAttnThreads;
  if (slots > 8) Fail(DSD_EINVAL, "num_heads*head_dim is too large for the attention kernel");
  a.slots = slots <= 1 ? 1 : slots <= 2 ? 2 : slots <= 4 ? 4 : 8;
  a.tps = std::max(1, std::min({page_size, dsdk::kAttnStageFloats / (2 * ept),
                                dsdk::kAttnMaxTokensPerStage}));
  a.smem = size_t(dsdk::kAttnStages) * 2 * a.tps * ept * sizeof(float) + dsdk::kAttnStages * 8;
  return a;
}

template <int NV, int S>
void SetAttnAttr(size_t smem) {
  Check(cudaFuncSetAttribute(dsdk::attn_kernel<NV, S>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(smem)), "smem attribute");
}

// Raises the dynamic shared-memory limit of every attention instantiation.
// NV = 4 serves head_dim >= 16 (at most 512 items for H*D <= 8192), NV = 2
// head_dim 8 (<= 1024 items), NV = 1 head_dim 4 (<= 2048 items).
void SetAllAttnAttributes(size_t smem) {
  SetAttnAttr<1, 1>(smem); SetAttnAttr<1, 2>(smem); SetAttnAttr<1, 4>(smem); SetAttnAttr<1, 8>(smem);
  SetAttnAttr<2, 1>(smem); SetAttnAttr<2, 2>(smem); SetAttnAttr<2, 4>(smem);
  SetAttnAttr<4, 1>(smem); SetAttnAttr<4, 2>(smem);
}

// Narrow-row scoring (128-byte row pieces, 4 CTAs per SM, 3-stage ring each)
// serves bf16 summaries: their per-byte dependent add chain is twice fp32's
// and needs more warps in flight (config 3: 2 CTAs x 5 stages 0.178 ms,
// 3 x 3 0.149 ms, 4 x 3 0.145 ms).  For fp32 summaries score_kernel stays
// (the narrow variant measured 0.282 vs 0.279 ms).
constexpr int kScoreNarrowCtas = 4;
constexpr int kScoreNarrowStages = 3;

template <typename T>
constexpr size_t ScoreNarrowSmem() {
  return kScoreNarrowStages * dsdk::ScoreRows<T>::kStageBytes;
}

template <typename T>
void SetScoreNarrowAttributes() {
  Check(cudaFuncSetAttribute(dsdk::score_kernel_narrow<T, kScoreNarrowStages, kScoreNarrowCtas>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(ScoreNarrowSmem<T>())),
        "smem attribute");
}

template <typename T>
void LaunchScoreNarrow(int num_sms, cudaStream_t st, const dsdk::StepPlan& plan, const float* q,
                       const T* summ, int ept, float scale, float* scores, int part, int nparts) {
  dsdk::score_kernel_narrow<T, kScoreNarrowStages, kScoreNarrowCtas>
      <<<kScoreNarrowCtas * num_sms, dsdk::kScoreThreads, ScoreNarrowSmem<T>(), st>>>(
          plan, q, summ, ept, scale, scores, part, nparts);
}

template <typename T, int NV, int S>
void SetAttnAttrNarrow(size_t smem) {
  Check(cudaFuncSetAttribute(dsdk::attn_kernel_narrow<T, NV, S>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
        "smem attribute");
}

// bf16 pages: NV = 1 serves head_dim 8 (<= 1024 items), NV = 2 the rest (<= 512);
// fp8 pages: NV = 1 (head_dim 16: <= 512 items, 32..128: <= 256).
template <typename T>
void SetAllAttnAttributesNarrow(size_t smem) {
  SetAttnAttrNarrow<T, 1, 1>(smem); SetAttnAttrNarrow<T, 1, 2>(smem);
  if constexpr (sizeof(T) == 2) {
    SetAttnAttrNarrow<T, 1, 4>(smem);
    SetAttnAttrNarrow<T, 2, 1>(smem); SetAttnAttrNarrow<T, 2, 2>(smem);
  }
}

template <typename T>
void LaunchAttnNarrow(const AttnShape& a, int grid, cudaStream_t st, const dsdk::StepPlan& plan,
                      const float* q, const T* k, const T* v, const int* tc, const int* sel,
                      float* pacc, float* pml, int H, int D, int P, float scale, int part,
                      int nparts) {
#define DSD_ATTN_CASE(NV, S)                                                                  \
  if (a.nv == NV && a.slots == S) {                                                           \
    dsdk::attn_kernel_narrow<T, NV, S><<<grid, dsdk::kAttnBfThreads, a.smem, st>>>(           \
        plan, q, k, v, tc, sel, pacc, pml, H, D, P, a.tps, a.nstages, scale, part, nparts);   \
    return;                                                                                   \
  }
  DSD_ATTN_CASE(1, 1) DSD_ATTN_CASE(1, 2)
  if constexpr (sizeof(T) == 2) {
    DSD_ATTN_CASE(1, 4) DSD_ATTN_CASE(2, 1) DSD_ATTN_CASE(2, 2)
  }
#undef DSD_ATTN_CASE
  Fail(DSD_EINVAL, "unsupported attention shape");
}

template <int NV, int S>
void LaunchAttnT(const AttnShape& a, int grid, cudaStream_t st, const dsdk::StepPlan& plan,
                 const float* q, const float* k, const float* v, const int* tc, const int* sel,
                 float* pacc, float* pml, int H, int D, int P, float scale, int part, int nparts) {
  dsdk::attn_kernel<NV, S><<<grid, dsdk::kAttnThreads, a.smem, st>>>(
      plan, q, k, v, tc, sel, pacc, pml, H, D, P, a.tps, scale, part, nparts);
}

void LaunchAttn(const AttnShape& a, int grid, cudaStream_t st, const dsdk::StepPlan& plan,
                const float* q, const float* k, const float* v, const int* tc, const int* sel,
                float* pacc, float* pml, int H, int D, int P, float scale, int part = 0,
                int nparts = 1) {
#define DSD_ATTN_CASE(NV, S)                                                        \
  if (a.nv == NV && a.slots == S) {                                                 \
    LaunchAttnT<NV, S>(a, grid, st, plan, q, k, v, tc, sel, pacc, pml, H, D, P, scale, part, \
                       nparts);                                                     \
    return;                                                                         \
  }
  DSD_ATTN_CASE(1, 1) DSD_ATTN_CASE(1, 2) DSD_ATTN_CASE(1, 4) DSD_ATTN_CASE(1, 8)
  DSD_ATTN_CASE(2, 1) DSD_ATTN_CASE(2, 2) DSD_ATTN_CASE(2, 4)
  DSD_ATTN_CASE(4, 1) DSD_ATTN_CASE(4, 2)
#undef DSD_ATTN_CASE
  Fail(DSD_EINVAL, "unsupported attention shape");
}

}  // namespace

template <typename T>
struct KvTag { using type = T; };

struct dsd_ctx {
  int device = 0;
  dsd_model_config cfg{};     // cfg.head_dim is the PHYSICAL head width (see padded)
  dsd_ctx_options opt{};
  int ept = 0;                // physical elements per token row: num_heads * cfg.head_dim
  // A head_dim that is not a power of two >= 4 is stored padded to one
  // (user_head_dim 80 -> 128): every row the caller passes or receives has
  // user_ept = num_heads * user_head_dim elements and is widened / narrowed
  // at the boundary; the padding is zero, so dot products, softmax and the
  // CPU's sequential score sums are unchanged.
  int user_head_dim = 0;
  int user_ept = 0;
  bool padded = false;
  int num_sms = 0;
  AttnShape attn;     // attention launch shape
  float scale = 0.f;
  cudaStream_t stream = nullptr;
  cudaStream_t stream2 = nullptr;      // second chain of a split step
  cudaEvent_t ev[6] = {};          // [0..3] stage events (set 0), [4], [5] step-done per slot
  cudaEvent_t ev_set1[4] = {};      // stage events of the second in-flight step
  cudaEvent_t ev_inputs = nullptr;  // the step input upload has been consumed
  int ev_set = 0;                   // stage-event set the next launch records into
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  // split host I/O of a page-table step: the second request range's queries
  // go up on copy_stream while the first range computes (ev_q1, waited on
  // inside the graph), and the first range's outputs come back on
  // copy_stream while the second range computes (ev_out0, recorded inside
  // the graph)
  cudaStream_t copy_stream = nullptr;
  cudaEvent_t ev_part0_up = nullptr, ev_q1 = nullptr, ev_out0 = nullptr, ev_out0_done = nullptr;
  cudaEvent_t ev_q0 = nullptr;   // first range's queries landed (plan runs meanwhile)
  // steps queued with dsd_decode_step_begin use per-slot device input/output
  // buffers (slot 0: d_in / d_outputs / plan, slot 1: d_in1 / d_outputs1 /
  // plan1): a slot's upload and result copies run on copy_stream, so they
  // overlap the other slot's kernels on the context stream
  unsigned char* d_in1 = nullptr;
  float* d_outputs1 = nullptr;
  cudaStream_t up_stream = nullptr;   // uploads of queued steps (results use copy_stream)
  dsdk::StepPlan plan1{};
  cudaEvent_t ev_in_ready[2] = {}, ev_graph_done[2] = {}, ev_out_read[2] = {};

  // pool: fp32, bf16 or fp8 e4m3 elements (kv_format); summary_floats counts elements
  int kv_format = DSD_KV_F32;
  size_t kv_elem = 4;
  void* k_pool = nullptr;
  void* v_pool = nullptr;
  void* summaries = nullptr;      // chunk-major in 128-page groups (see summary_off)
  size_t summary_floats = 0;
  int* token_counts = nullptr;
  uint8_t* live = nullptr;
  std::vector<int> host_counts;  // mirror of token_counts for validation

  // request page tables
  int* table = nullptr;
  int* table_n = nullptr;
  std::unordered_map<int, int> slot_of;
  std::vector<int> free_slots;
  std::vector<std::vector<int>> slot_pages;

  // per-step buffers.  step_in = [hdr 4 ints][req max_batch+1 ints][pad][queries][cand ids]
  size_t in_req_off = 0, in_q_off = 0, in_ids_off = 0, in_bytes = 0;
  unsigned char* d_in = nullptr;
  unsigned char* h_in = nullptr;  // pinned
  float* d_scores = nullptr;
  int* d_selected = nullptr;
  float* d_outputs = nullptr;
  float* d_part_acc = nullptr;
  float* d_part_ml = nullptr;
  int* d_planbuf = nullptr;
  int* d_status = nullptr;
  dsdk::StepPlan plan{};
  float* h_outputs = nullptr;   // pinned D2H staging (slot 0; slot 1 below)
  float* h_outputs1 = nullptr;
  float* h_scores1 = nullptr;
  int* h_selected1 = nullptr;
  float* h_scores = nullptr;
  int* h_selected = nullptr;
  int* h_status = nullptr;

  // staging for uploads / appends (grow only, admission time)
  unsigned char* d_stage = nullptr;
  size_t d_stage_bytes = 0;

  // bulk host->device uploads: per worker two pinned chunks, a copy stream
  // and an event per chunk (created on first large pageable upload)
  struct Uploader {
    cudaStream_t stream = nullptr;
    unsigned char* pinned[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
  };
  std::vector<Uploader> uploaders;

  // bound (device-resident) steps
  int bound_batch = -1;
  // captured steps, keyed by (queries, outputs, timed); the plan inside a
  // graph reads the batch from the device header, so one graph serves every
  // batch size and composition
  struct StepGraph {
    const dsdk::StepPlan* plan;
    const float* q;
    float* out;
    bool timed;
    int ev_set;
    bool split_io;
    cudaGraph_t graph;
    cudaGraphExec_t exec;
  };
  std::vector<StepGraph> graphs;

  dsd_transfer_stats stats{};
  int dense = 0;   // attend over every candidate (dense baseline) instead of the top-k

  // steps queued by dsd_decode_step_begin and finished, oldest first, by
  // dsd_decode_step_end; up to two may be in flight (result staging slots 0/1)
  struct PendingStep {
    bool active = false;
    int batch = 0, total_cand = 0, total_sel = 0, output_mode = 0, timing = 0;
  } pend[2];
  int pend_head = 0, pend_count = 0;
};

// Calls f(KvTag<T>{}) with T the context's page element type.
template <typename F>
void WithKv(const dsd_ctx* c, F&& f) {
  if (c->kv_format == DSD_KV_BF16) f(KvTag<__nv_bfloat16>{});
  else if (c->kv_format == DSD_KV_FP8) f(KvTag<__nv_fp8_e4m3>{});
  else f(KvTag<float>{});
}

namespace {

void CountH2D(dsd_ctx* c, size_t bytes) {
  c->stats.h2d_bytes += bytes;
  c->stats.h2d_calls += 1;
  if (bytes >= kLargeCopyBytes) c->stats.h2d_large_calls += 1;
}
void CountD2H(dsd_ctx* c, size_t bytes) {
  c->stats.d2h_bytes += bytes;
  c->stats.d2h_calls += 1;
  if (bytes >= kLargeCopyBytes) c->stats.d2h_large_calls += 1;
}

void H2D(dsd_ctx* c, void* dst, const void* src, size_t bytes) {
  if (bytes == 0) return;
  Check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, c->stream), "H2D copy");
  CountH2D(c, bytes);
}
void D2H(dsd_ctx* c, void* dst, const void* src, size_t bytes) {
  if (bytes == 0) return;
  Check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, c->stream), "D2H copy");
  CountD2H(c, bytes);
}

void Sync(dsd_ctx* c) { Check(cudaStreamSynchronize(c->stream), "stream synchronize"); }

void SetDevice(dsd_ctx* c) { Check(cudaSetDevice(c->device), "cudaSetDevice"); }

void EnsureStage(dsd_ctx* c, size_t bytes) {
  if (bytes <= c->d_stage_bytes) return;
  Sync(c);
  if (c->d_stage) cudaFree(c->d_stage);
  c->d_stage = nullptr;
  c->d_stage_bytes = 0;
  c->d_stage = DeviceAlloc<unsigned char>(bytes, "staging buffer");
  c->d_stage_bytes = bytes;
}

bool IsPinnedHost(const void* p);
bool IsPinnedHostPtr(const void* p) { return IsPinnedHost(p); }

constexpr size_t kUploadChunk = size_t(4) << 20;    // bytes per pinned chunk
// host threads staging a large pageable upload (about half the cores, 2..8)
int UploadWorkers() {
  const int hw = static_cast<int>(std::thread::hardware_concurrency());
  return std::max(2, std::min(8, hw / 2));
}

// Host -> device copy of a large pageable buffer: UploadWorkers() threads each
// copy 4 MiB chunks into their two pinned buffers and DMA them on their own
// stream, so host copies and PCIe transfers overlap.  The context stream
// then waits for every worker stream.  Pinned or small sources go directly.
struct UploadSegment {
  void* dst;
  const void* src;
  size_t bytes;
};

void BulkH2D(dsd_ctx* c, const std::vector<UploadSegment>& in) {
  // small or pinned segments go directly; the rest share one worker pass
  std::vector<UploadSegment> segs;
  for (const auto& g : in) {
    if (g.bytes == 0) continue;
    if (g.bytes < 2 * kUploadChunk || IsPinnedHostPtr(g.src))
      H2D(c, g.dst, g.src, g.bytes);
    else
      segs.push_back(g);
  }
  if (segs.empty()) return;
  if (c->uploaders.empty()) {
    c->uploaders.resize(static_cast<size_t>(UploadWorkers()));
    for (auto& u : c->uploaders) {
      Check(cudaStreamCreateWithFlags(&u.stream, cudaStreamNonBlocking), "upload stream");
      for (int b = 0; b < 2; ++b) {
        u.pinned[b] = PinnedAlloc<unsigned char>(kUploadChunk, "upload staging");
        Check(cudaEventCreateWithFlags(&u.done[b], cudaEventDisableTiming), "upload event");
      }
    }
  }
  // the destination may still be read by earlier work on the context stream
  cudaEvent_t ready;
  Check(cudaEventCreateWithFlags(&ready, cudaEventDisableTiming), "event");
  Check(cudaEventRecord(ready, c->stream), "event record");
  // chunk list over all segments: (segment, offset)
  std::vector<std::pair<size_t, size_t>> chunks;
  size_t total = 0;
  for (size_t k = 0; k < segs.size(); ++k) {
    for (size_t off = 0; off < segs[k].bytes; off += kUploadChunk) chunks.emplace_back(k, off);
    total += segs[k].bytes;
  }
  const size_t nchunks = chunks.size();
  std::vector<std::string> errors(c->uploaders.size());
  std::vector<std::thread> pool;
  for (size_t w = 0; w < c->uploaders.size(); ++w) {
    pool.emplace_back([&, w]() {
      auto& u = c->uploaders[w];
      if (cudaSetDevice(c->device) != cudaSuccess ||
          cudaStreamWaitEvent(u.stream, ready, 0) != cudaSuccess) {
        errors[w] = "upload worker setup failed";
        return;
      }
      int b = 0;
      for (size_t i = w; i < nchunks; i += c->uploaders.size(), b ^= 1) {
        const UploadSegment& g = segs[chunks[i].first];
        const size_t off = chunks[i].second;
        const size_t len = std::min(kUploadChunk, g.bytes - off);
        if (cudaEventSynchronize(u.done[b]) != cudaSuccess) {
          errors[w] = "upload event wait failed";
          return;
        }
        std::memcpy(u.pinned[b], static_cast<const unsigned char*>(g.src) + off, len);
        if (cudaMemcpyAsync(static_cast<unsigned char*>(g.dst) + off, u.pinned[b], len,
                            cudaMemcpyHostToDevice, u.stream) != cudaSuccess ||
            cudaEventRecord(u.done[b], u.stream) != cudaSuccess) {
          errors[w] = "upload copy failed";
          return;
        }
      }
    });
  }
  for (auto& t : pool) t.join();
  cudaEventDestroy(ready);
  for (const auto& e : errors)
    if (!e.empty()) Fail(DSD_ECUDA, e);
  for (auto& u : c->uploaders)
    for (int b = 0; b < 2; ++b)
      Check(cudaStreamWaitEvent(c->stream, u.done[b], 0), "upload join");
  c->stats.h2d_bytes += total;
  c->stats.h2d_calls += nchunks;
  c->stats.h2d_large_calls += nchunks;
}

void ValidatePage(const dsd_ctx* c, int page) {
  if (page < 0 || page >= c->opt.capacity_pages) Fail(DSD_ERANGE, "invalid page id");
}

// Reads the kernel status word after a synchronisation and clears it.
void CheckStatus(dsd_ctx* c) {
  Check(cudaMemcpyAsync(c->h_status, c->d_status, sizeof(int), cudaMemcpyDeviceToHost, c->stream),
        "status read");
  Sync(c);
  const int s = *c->h_status;
  if (s != 0) {
    Check(cudaMemsetAsync(c->d_status, 0, sizeof(int), c->stream), "status clear");
    Sync(c);
    if (s & dsdk::kStatusTimeout) Fail(DSD_ETIMEOUT, "a device-side wait exceeded its budget");
    Fail(DSD_EINVAL, "device kernels rejected the step input (status " + std::to_string(s) + ")");
  }
}

// ------------------------------------------------------------------ row layout

// Caller rows ([rows][num_heads * user_head_dim]) into pool rows
// ([rows][num_heads * head_dim]), zero padding; a plain copy when not padded.
void PadRowsInto(const dsd_ctx* c, float* dst, const float* src, size_t rows) {
  if (!c->padded) {
    std::memcpy(dst, src, rows * size_t(c->ept) * sizeof(float));
    return;
  }
  const int H = c->cfg.num_heads, d = c->user_head_dim, dp = c->cfg.head_dim;
  for (size_t r = 0; r < rows; ++r)
    for (int h = 0; h < H; ++h) {
      float* o = dst + r * size_t(c->ept) + size_t(h) * dp;
      std::memcpy(o, src + r * size_t(c->user_ept) + size_t(h) * d, size_t(d) * sizeof(float));
      std::memset(o + d, 0, size_t(dp - d) * sizeof(float));
    }
}

std::vector<float> PadRows(const dsd_ctx* c, const float* src, size_t rows) {
  std::vector<float> out(rows * size_t(c->ept));
  PadRowsInto(c, out.data(), src, rows);
  return out;
}

// Pool rows back to caller rows (drops the padding).
void UnpadRowsInto(const dsd_ctx* c, float* dst, const float* src, size_t rows) {
  if (!c->padded) {
    std::memcpy(dst, src, rows * size_t(c->ept) * sizeof(float));
    return;
  }
  const int H = c->cfg.num_heads, d = c->user_head_dim, dp = c->cfg.head_dim;
  for (size_t r = 0; r < rows; ++r)
    for (int h = 0; h < H; ++h)
      std::memcpy(dst + r * size_t(c->user_ept) + size_t(h) * d,
                  src + r * size_t(c->ept) + size_t(h) * dp, size_t(d) * sizeof(float));
}

void RequireUnpadded(const dsd_ctx* c, const char* what) {
  if (c->padded)
    Fail(DSD_EINVAL, std::string(what) + " needs head_dim a power of two >= 4 (device rows "
                     "are used as they are)");
}

// ------------------------------------------------------------------ step

void RecordEvent(dsd_ctx* c, int i, bool capturing) {
  // inside a capture the record must become a graph node of its own
  cudaEvent_t e = c->ev_set ? c->ev_set1[i] : c->ev[i];
  Check(capturing ? cudaEventRecordWithFlags(e, c->stream, cudaEventRecordExternal)
                  : cudaEventRecord(e, c->stream), "event record");
}

// One decode step.  Untimed steps split the requests into kStepParts ranges
// whose kernel chains run on two streams (fork/join inside the captured
// graph), so one part's small kernels and kernel tails overlap the other
// part's bandwidth-bound kernels.  Timed steps run one chain with an event
// between the stages.
constexpr int kStepParts = 2;

void LaunchStep(dsd_ctx* c, const dsdk::StepPlan& plan, const float* d_q, float* d_out,
                bool timed, bool capturing = false, bool split_io = false) {
  const int target_units = 8 * c->num_sms;
  const int H = c->cfg.num_heads, D = c->cfg.head_dim, P = c->cfg.page_size;
  const int sel_grid = std::max(1, std::min(c->opt.max_batch, 2 * c->num_sms));
  const int pairs = c->opt.max_batch * H;
  const int comb_grid = std::max(1, std::min((pairs + 7) / 8, 8 * c->num_sms));
  const int nparts = timed ? 1 : kStepParts;
  if (timed) RecordEvent(c, 0, capturing);
  NvtxRange nvtx_step("dsd.step");
  const int score_ctas =
      (c->kv_format != DSD_KV_F32 ? kScoreNarrowCtas : 2) * c->num_sms;
  {
    NvtxRange r("dsd.plan");
    dsdk::plan_kernel<<<1, dsdk::kPlanThreads, 0, c->stream>>>(plan, c->cfg.top_k_pages,
                                                               target_units, score_ctas);
  }
  if (nparts > 1) {
    Check(cudaEventRecord(c->ev_fork, c->stream), "fork");
    Check(cudaStreamWaitEvent(c->stream2, c->ev_fork, 0), "fork wait");
    // the second range's queries arrive on copy_stream (recorded before launch)
    if (split_io && capturing)
      Check(cudaStreamWaitEvent(c->stream2, c->ev_q1, cudaEventWaitExternal), "query wait");
  }
  for (int part = 0; part < nparts; ++part) {
    cudaStream_t st = part == 0 ? c->stream : c->stream2;
    NvtxRange nvtx_part(part == 0 ? "dsd.step.range0" : "dsd.step.range1");
    // the first range's queries arrive on copy_stream while the plan kernel runs
    if (split_io && capturing && part == 0)
      Check(cudaStreamWaitEvent(c->stream, c->ev_q0, cudaEventWaitExternal), "query wait");
    nvtxRangePushA("dsd.score");
    if (c->kv_format == DSD_KV_F32) {
      dsdk::score_kernel<<<2 * c->num_sms, dsdk::kScoreThreads, dsdk::kScoreSmem, st>>>(
          plan, d_q, static_cast<const float*>(c->summaries), c->ept, c->scale, c->d_scores,
          part, nparts);
    } else {
      WithKv(c, [&](auto tag) {
        using T = typename decltype(tag)::type;
        if constexpr (!std::is_same<T, float>::value)
          LaunchScoreNarrow(c->num_sms, st, plan, d_q, static_cast<const T*>(c->summaries),
                            c->ept, c->scale, c->d_scores, part, nparts);
      });
    }
    nvtxRangePop();
    if (timed) RecordEvent(c, 1, capturing);
    nvtxRangePushA("dsd.select");
    dsdk::select_kernel<<<sel_grid, dsdk::kSelectThreads, dsdk::kSelectSmem, st>>>(
        plan, c->d_scores, c->d_selected, part, nparts);
    nvtxRangePop();
    if (timed) RecordEvent(c, 2, capturing);
    nvtxRangePushA("dsd.attention");
    if (c->kv_format != DSD_KV_F32)
      WithKv(c, [&](auto tag) {
        using T = typename decltype(tag)::type;
        if constexpr (!std::is_same<T, float>::value)
          LaunchAttnNarrow(c->attn, c->attn.ctas * c->num_sms, st, plan, d_q, static_cast<const T*>(c->k_pool),
                           static_cast<const T*>(c->v_pool), c->token_counts, c->d_selected,
                           c->d_part_acc, c->d_part_ml, H, D, P, c->scale, part, nparts);
      });
    else
      LaunchAttn(c->attn, c->num_sms, st, plan, d_q, static_cast<const float*>(c->k_pool),
                 static_cast<const float*>(c->v_pool), c->token_counts, c->d_selected,
                 c->d_part_acc, c->d_part_ml, H, D, P, c->scale, part, nparts);
    nvtxRangePop();
    nvtxRangePushA("dsd.combine");
    dsdk::combine_kernel<<<comb_grid, 256, 0, st>>>(plan, c->d_part_acc, c->d_part_ml, H, D,
                                                    d_out, part, nparts);
    nvtxRangePop();
    if (split_io && capturing && nparts > 1 && part == 0)
      Check(cudaEventRecordWithFlags(c->ev_out0, c->stream, cudaEventRecordExternal),
            "part output event");
  }
  if (nparts > 1) {
    Check(cudaEventRecord(c->ev_join, c->stream2), "join");
    Check(cudaStreamWaitEvent(c->stream, c->ev_join, 0), "join wait");
  }
  Check(cudaGetLastError(), "kernel launch");
  if (timed) RecordEvent(c, 3, capturing);
}

// Replays the step as a CUDA graph (captured on first use for this pointer pair).
void LaunchStepGraph(dsd_ctx* c, const float* d_q, float* d_out, bool timed,
                     bool split_io = false, const dsdk::StepPlan* plan = nullptr) {
  split_io = split_io && !timed;
  if (!plan) plan = &c->plan;
  for (auto& g : c->graphs) {
    if (g.plan == plan && g.q == d_q && g.out == d_out && g.timed == timed &&
        g.split_io == split_io && (!timed || g.ev_set == c->ev_set)) {
      Check(cudaGraphLaunch(g.exec, c->stream), "graph launch");
      return;
    }
  }
  dsd_ctx::StepGraph g{plan, d_q, d_out, timed, c->ev_set, split_io, nullptr, nullptr};
  Check(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
  try {
    LaunchStep(c, *plan, d_q, d_out, timed, true, split_io);
  } catch (...) {
    cudaGraph_t dead = nullptr;
    cudaStreamEndCapture(c->stream, &dead);
    if (dead) cudaGraphDestroy(dead);
    throw;
  }
  Check(cudaStreamEndCapture(c->stream, &g.graph), "end capture");
  Check(cudaGraphInstantiate(&g.exec, g.graph, 0), "graph instantiate");
  // one graph per (plan, query, output) pointer set; a caller cycling through
  // many result buffers keeps at most kMaxGraphs of them (oldest evicted,
  // after the stream has drained)
  constexpr size_t kMaxGraphs = 16;
  if (c->graphs.size() >= kMaxGraphs) {
    Sync(c);
    cudaGraphExecDestroy(c->graphs.front().exec);
    cudaGraphDestroy(c->graphs.front().graph);
    c->graphs.erase(c->graphs.begin());
  }
  c->graphs.push_back(g);
  Check(cudaGraphLaunch(g.exec, c->stream), "graph launch");
}

void ReadTiming(dsd_ctx* c, dsd_step_timing* t, int set = 0) {
  if (!t) return;
  const cudaEvent_t* e = set ? c->ev_set1 : c->ev;
  Check(cudaEventSynchronize(e[3]), "event sync");
  Check(cudaEventElapsedTime(&t->score_ms, e[0], e[1]), "event time");
  Check(cudaEventElapsedTime(&t->topk_ms, e[1], e[2]), "event time");
  Check(cudaEventElapsedTime(&t->attention_ms, e[2], e[3]), "event time");
  Check(cudaEventElapsedTime(&t->total_ms, e[0], e[3]), "event time");
}

// True for page-locked host memory (cudaMallocHost / cudaHostRegister):
// such buffers are DMA'd directly, without the staging copy.
bool IsPinnedHost(const void* p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

// The device-side address of page-locked, mapped host memory (kernels write
// it over PCIe), or nullptr when `p` is not such memory.
float* MappedHostOutput(float* p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return a.type == cudaMemoryTypeHost ? static_cast<float*>(a.devicePointer) : nullptr;
}

// The pinned input staging may be rewritten once the previous step's upload
// of it has completed (a second step can be queued while one is in flight).
void WaitInputStaging(dsd_ctx* c) { Check(cudaEventSynchronize(c->ev_inputs), "input staging"); }

int* HdrPtr(dsd_ctx* c) { return reinterpret_cast<int*>(c->h_in); }
int* ReqPtr(dsd_ctx* c) { return reinterpret_cast<int*>(c->h_in + c->in_req_off); }
float* QPtr(dsd_ctx* c) { return reinterpret_cast<float*>(c->h_in + c->in_q_off); }
int* IdsPtr(dsd_ctx* c) { return reinterpret_cast<int*>(c->h_in + c->in_ids_off); }

// Uploads the step header, request list and queries.  Pinned caller queries
// go straight to the device; pageable ones through the pinned staging.
void UploadQueries(dsd_ctx* c, const float* queries, int batch) {
  const size_t qbytes = size_t(batch) * c->ept * 4;
  if (!c->padded && queries != QPtr(c) && IsPinnedHost(queries)) {
    H2D(c, c->d_in, c->h_in, c->in_q_off);
    H2D(c, c->d_in + c->in_q_off, queries, qbytes);
  } else {
    if (queries != QPtr(c)) PadRowsInto(c, QPtr(c), queries, size_t(batch));
    H2D(c, c->d_in, c->h_in, c->in_q_off + qbytes);
  }
  Check(cudaEventRecord(c->ev_inputs, c->stream), "event record");
}

// Untimed page-table steps of at least two requests split their host I/O.
bool SplitIo(int batch, int timing) { return timing == 0 && batch >= kStepParts; }

// First request of the second range of a split step (part_range on the device).
int SplitRow(int batch) { return int((long long)batch * 1 / kStepParts); }

// UploadQueries for a page-table step whose host I/O is split: the header,
// request list and the first range's queries go up on the context stream,
// then (ordered after them, so they do not share the link) the second
// range's queries on copy_stream, completing ev_q1, which the step graph
// waits for before the second range's kernels.
void UploadQueriesSplit(dsd_ctx* c, const float* queries, int batch) {
  const size_t row = size_t(c->ept) * 4;
  const int h0 = SplitRow(batch);
  const bool direct = !c->padded && queries != QPtr(c) && IsPinnedHost(queries);
  if (!direct && queries != QPtr(c)) PadRowsInto(c, QPtr(c), queries, size_t(batch));
  const unsigned char* src =
      direct ? reinterpret_cast<const unsigned char*>(queries) : c->h_in + c->in_q_off;
  // header and request list on the context stream (the plan kernel needs only
  // them), then both query ranges on copy_stream, each completing the event
  // its range's chain waits for inside the step graph
  H2D(c, c->d_in, c->h_in, c->in_q_off);
  Check(cudaEventRecord(c->ev_part0_up, c->stream), "event record");
  Check(cudaStreamWaitEvent(c->copy_stream, c->ev_part0_up, 0), "copy stream wait");
  const size_t split = size_t(h0) * row, total = size_t(batch) * row;
  if (split)
    Check(cudaMemcpyAsync(c->d_in + c->in_q_off, src, split, cudaMemcpyHostToDevice,
                          c->copy_stream), "H2D copy");
  Check(cudaEventRecord(c->ev_q0, c->copy_stream), "event record");
  Check(cudaMemcpyAsync(c->d_in + c->in_q_off + split, src + split, total - split,
                        cudaMemcpyHostToDevice, c->copy_stream), "H2D copy");
  CountH2D(c, total);
  Check(cudaEventRecord(c->ev_q1, c->copy_stream), "event record");
  // the pinned staging is free again once both uploads are done
  Check(cudaEventRecord(c->ev_inputs, c->copy_stream), "event record");
}

// Output copy of a split step: the first range's rows come back on
// copy_stream as soon as the graph's first range is done (ev_out0), the
// second range's on the context stream, which then waits for the first.
void CopyOutputsSplit(dsd_ctx* c, float* h_out, int batch) {
  const size_t row = size_t(c->ept) * 4;
  const int h0 = SplitRow(batch);
  Check(cudaStreamWaitEvent(c->copy_stream, c->ev_out0, 0), "copy stream wait");
  Check(cudaMemcpyAsync(h_out, c->d_outputs, size_t(h0) * row, cudaMemcpyDeviceToHost,
                        c->copy_stream), "D2H copy");
  Check(cudaEventRecord(c->ev_out0_done, c->copy_stream), "event record");
  D2H(c, reinterpret_cast<unsigned char*>(h_out) + size_t(h0) * row,
      reinterpret_cast<const unsigned char*>(c->d_outputs) + size_t(h0) * row,
      size_t(batch - h0) * row);
  CountD2H(c, size_t(h0) * row);
  Check(cudaStreamWaitEvent(c->stream, c->ev_out0_done, 0), "output join");
}

// Common tail of a host-facing step: launch, copy results back, unpack.
void RunHostStep(dsd_ctx* c, int batch, int total_cand, int total_sel, int output_mode,
                 int timing, float* outputs, float* scores, int32_t* selected,
                 dsd_step_timing* out_timing, bool split_io = false) {
  // queued (begin/end) steps may still be copying results out of d_outputs
  for (cudaEvent_t e : c->ev_out_read) Check(cudaStreamWaitEvent(c->stream, e, 0), "wait");
  const size_t out_bytes = size_t(batch) * c->ept * sizeof(float);
  const bool want_out = output_mode != DSD_OUTPUT_NONE && outputs;
  const bool direct_out =
      !c->padded && want_out && outputs != c->h_outputs && IsPinnedHost(outputs);
  // A split-I/O step with a mapped, page-locked result buffer has its combine
  // kernels write the outputs straight into it over PCIe: no output copy,
  // each range's rows leave as they are computed.
  float* zero_copy = split_io && direct_out ? MappedHostOutput(outputs) : nullptr;
  LaunchStepGraph(c, reinterpret_cast<const float*>(c->d_in + c->in_q_off),
                  zero_copy ? zero_copy : c->d_outputs, timing != 0, split_io);
  if (zero_copy) CountD2H(c, out_bytes);   // written over PCIe by the kernels themselves
  if (want_out && !zero_copy) {
    if (split_io)
      CopyOutputsSplit(c, direct_out ? outputs : c->h_outputs, batch);
    else
      D2H(c, direct_out ? outputs : c->h_outputs, c->d_outputs, out_bytes);
  }
  if (output_mode == DSD_OUTPUT_DEBUG) {
    if (scores && total_cand > 0)
      D2H(c, c->h_scores, c->d_scores, size_t(total_cand) * sizeof(float));
    if (selected && total_sel > 0)
      D2H(c, c->h_selected, c->d_selected, size_t(total_sel) * sizeof(int));
  }
  CheckStatus(c);  // synchronises the stream
  if (timing) ReadTiming(c, out_timing);
  if (output_mode != DSD_OUTPUT_NONE && outputs && outputs != c->h_outputs && !direct_out)
    UnpadRowsInto(c, outputs, c->h_outputs, size_t(batch));
  if (output_mode == DSD_OUTPUT_DEBUG) {
    if (scores && total_cand > 0)
      std::memcpy(scores, c->h_scores, size_t(total_cand) * sizeof(float));
    if (selected && total_sel > 0)
      std::memcpy(selected, c->h_selected, size_t(total_sel) * sizeof(int));
  }
}

// Queues a step in a free slot: the step input goes up on up_stream into the
// slot's device buffer (after the slot's previous step has consumed it), the
// context stream runs the step graph once its input has landed and the
// slot's previous outputs have been read, and the results (status word
// included) come back on copy_stream into the slot's pinned staging; the
// slot's done event marks the end.  Uploads and downloads use separate
// streams, so the next step's upload does not queue behind this step's
// download: one slot's copies overlap the other slot's kernels.
void EnqueueStep(dsd_ctx* c, const float* queries, int batch, int total_cand, int total_sel,
                 int output_mode, int timing) {
  if (c->pend_count >= 2) Fail(DSD_EINVAL, "two decode steps are already pending");
  const int slot = (c->pend_head + c->pend_count) & 1;
  unsigned char* din = slot ? c->d_in1 : c->d_in;
  float* dout = slot ? c->d_outputs1 : c->d_outputs;
  const dsdk::StepPlan* plan = slot ? &c->plan1 : &c->plan;
  cudaStream_t cs = c->copy_stream, us = c->up_stream;
  const size_t qbytes = size_t(batch) * c->ept * 4;
  // input
  Check(cudaStreamWaitEvent(us, c->ev_graph_done[slot], 0), "slot wait");
  const bool direct = !c->padded && queries != QPtr(c) && IsPinnedHost(queries);
  if (!direct && queries != QPtr(c)) PadRowsInto(c, QPtr(c), queries, size_t(batch));
  Check(cudaMemcpyAsync(din, c->h_in, direct ? c->in_q_off : c->in_q_off + qbytes,
                        cudaMemcpyHostToDevice, us), "H2D copy");
  if (direct)
    Check(cudaMemcpyAsync(din + c->in_q_off, queries, qbytes, cudaMemcpyHostToDevice, us),
          "H2D copy");
  CountH2D(c, c->in_q_off + qbytes);
  Check(cudaEventRecord(c->ev_inputs, us), "event record");
  Check(cudaEventRecord(c->ev_in_ready[slot], us), "event record");
  // the step
  Check(cudaStreamWaitEvent(c->stream, c->ev_in_ready[slot], 0), "input wait");
  Check(cudaStreamWaitEvent(c->stream, c->ev_out_read[slot], 0), "output wait");
  const int other = slot ^ 1;
  if (c->pend_count > 0 && c->pend[other].output_mode == DSD_OUTPUT_DEBUG)
    // scores and selected ids live in one device buffer: the other slot's copy first
    Check(cudaStreamWaitEvent(c->stream, c->ev_out_read[other], 0), "output wait");
  c->ev_set = slot;
  LaunchStepGraph(c, reinterpret_cast<const float*>(din + c->in_q_off), dout, timing != 0,
                  false, plan);
  c->ev_set = 0;
  Check(cudaEventRecord(c->ev_graph_done[slot], c->stream), "event record");
  // results
  Check(cudaStreamWaitEvent(cs, c->ev_graph_done[slot], 0), "result wait");
  float* h_out = slot ? c->h_outputs1 : c->h_outputs;
  auto d2h = [&](void* dst, const void* src, size_t bytes) {
    if (bytes == 0) return;
    Check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, cs), "D2H copy");
    CountD2H(c, bytes);
  };
  if (output_mode != DSD_OUTPUT_NONE) d2h(h_out, dout, qbytes);
  if (output_mode == DSD_OUTPUT_DEBUG) {
    d2h(slot ? c->h_scores1 : c->h_scores, c->d_scores, size_t(total_cand) * sizeof(float));
    d2h(slot ? c->h_selected1 : c->h_selected, c->d_selected, size_t(total_sel) * sizeof(int));
  }
  Check(cudaMemcpyAsync(c->h_status, c->d_status, sizeof(int), cudaMemcpyDeviceToHost, cs),
        "status read");
  Check(cudaEventRecord(c->ev_out_read[slot], cs), "event record");
  Check(cudaEventRecord(c->ev[4 + slot], cs), "event record");
  c->pend[slot] = dsd_ctx::PendingStep{true, batch, total_cand, total_sel, output_mode, timing};
  ++c->pend_count;
}

void FinishStep(dsd_ctx* c, float* outputs, float* scores, int32_t* selected,
                dsd_step_timing* out_timing) {
  if (c->pend_count == 0) Fail(DSD_EINVAL, "no decode step is pending");
  const int slot = c->pend_head;
  const auto p = c->pend[slot];
  c->pend[slot].active = false;
  c->pend_head ^= 1;
  --c->pend_count;
  Check(cudaEventSynchronize(c->ev[4 + slot]), "step wait");
  const int st = *c->h_status;
  if (st != 0) {
    Check(cudaMemsetAsync(c->d_status, 0, sizeof(int), c->stream), "status clear");
    Sync(c);
    if (st & dsdk::kStatusTimeout) Fail(DSD_ETIMEOUT, "a device-side wait exceeded its budget");
    Fail(DSD_EINVAL, "device kernels rejected the step input (status " + std::to_string(st) + ")");
  }
  if (p.timing) ReadTiming(c, out_timing, slot);
  const float* h_out = slot ? c->h_outputs1 : c->h_outputs;
  if (p.output_mode != DSD_OUTPUT_NONE && outputs && outputs != h_out)
    UnpadRowsInto(c, outputs, h_out, size_t(p.batch));
  if (p.output_mode == DSD_OUTPUT_DEBUG) {
    if (scores && p.total_cand > 0)
      std::memcpy(scores, slot ? c->h_scores1 : c->h_scores, size_t(p.total_cand) * sizeof(float));
    if (selected && p.total_sel > 0)
      std::memcpy(selected, slot ? c->h_selected1 : c->h_selected,
                  size_t(p.total_sel) * sizeof(int));
  }
}

int SlotOf(dsd_ctx* c, int request_id, bool create) {
  auto it = c->slot_of.find(request_id);
  if (it != c->slot_of.end()) return it->second;
  if (!create) Fail(DSD_EINVAL, "unknown request id " + std::to_string(request_id));
  if (c->free_slots.empty()) Fail(DSD_ENOMEM, "no free request page-table slot");
  const int slot = c->free_slots.back();
  c->free_slots.pop_back();
  c->slot_of[request_id] = slot;
  c->slot_pages[slot].clear();
  return slot;
}

void RequireTables(dsd_ctx* c) {
  if (c->opt.max_requests <= 0 || c->table == nullptr)
    Fail(DSD_EINVAL, "context was created without request page tables");
}

// Writes (slot, position, page) triples plus explicit counts to the device tables.
void UploadTableEntries(dsd_ctx* c, const std::vector<int>& triples,
                        const std::vector<int>& count_pairs) {
  const size_t nt = triples.size() / 3, nc = count_pairs.size() / 2;
  const size_t bytes = (triples.size() + count_pairs.size()) * sizeof(int);
  if (bytes == 0) return;
  EnsureStage(c, bytes);
  std::vector<int> packed(triples);
  packed.insert(packed.end(), count_pairs.begin(), count_pairs.end());
  Check(cudaMemcpyAsync(c->d_stage, packed.data(), bytes, cudaMemcpyHostToDevice, c->stream),
        "table upload");
  CountH2D(c, bytes);
  int* d = reinterpret_cast<int*>(c->d_stage);
  if (nc) dsdk::table_set_count_kernel<<<(unsigned)((nc + 255) / 256), 256, 0, c->stream>>>(
      d + triples.size(), (int)nc, c->table_n);
  if (nt) dsdk::table_write_kernel<<<(unsigned)((nt + 255) / 256), 256, 0, c->stream>>>(
      d, (int)nt, c->opt.max_pages_per_request, c->table, c->table_n);
  Check(cudaGetLastError(), "table kernels");
  // no wait: later users of the staging buffer are ordered on the same stream
}

// Groups tokens by page: indices sorted by (page, offset); one group per page.
void GroupTokens(const int32_t* page_ids, const int32_t* offs, int n, std::vector<int>* order,
                 std::vector<int>* group_page, std::vector<int>* group_first) {
  order->resize(static_cast<size_t>(n));
  for (int i = 0; i < n; ++i) (*order)[static_cast<size_t>(i)] = i;
  std::sort(order->begin(), order->end(), [&](int a, int b) {
    return page_ids[a] != page_ids[b] ? page_ids[a] < page_ids[b] : offs[a] < offs[b];
  });
  group_page->clear();
  group_first->clear();
  for (int j = 0; j < n; ++j) {
    const int i = (*order)[static_cast<size_t>(j)];
    if (j == 0 || page_ids[i] != page_ids[(*order)[static_cast<size_t>(j - 1)]]) {
      group_page->push_back(page_ids[i]);
      group_first->push_back(j);
    }
  }
  group_first->push_back(n);
}

}  // namespace

extern "C" {

const char* dsd_last_error(void) { return g_last_error.c_str(); }

int dsd_available(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    return 0;
  }
  int dev = 0;
  cudaDeviceProp prop{};
  if (cudaGetDevice(&dev) != cudaSuccess || cudaGetDeviceProperties(&prop, dev) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return prop.major >= 10 ? 1 : 0;
}

int dsd_kernels_per_step(void) { return 5; }

int dsd_set_attention_mode(dsd_ctx* c, int dense) {
  return Guard([&]() {
    if (!c) Fail(DSD_EINVAL, "null context");
    if (c->pend_count) Fail(DSD_EINVAL, "a decode step is pending");
    c->dense = dense ? 1 : 0;
  });
}

int dsd_selftest_bounded_wait(dsd_ctx* c, int64_t budget_cycles) {
  return Guard([&]() {
    if (!c) Fail(DSD_EINVAL, "null context");
    if (budget_cycles <= 0 || budget_cycles > (int64_t(1) << 32))
      Fail(DSD_EINVAL, "budget must be in (0, 2^32] cycles");
    SetDevice(c);
    dsdk::bounded_wait_probe_kernel<<<1, 32, 0, c->stream>>>(c->d_status, budget_cycles);
    Check(cudaGetLastError(), "probe launch");
    CheckStatus(c);  // DSD_ETIMEOUT when the wait gave up, as it must
  });
}

int dsd_ctx_create(int device, const dsd_model_config* config, const dsd_ctx_options* options,
                   dsd_ctx** out) {
  return dsd_ctx_create_ex(device, config, options, DSD_KV_F32, out);
}

int dsd_ctx_kv_format(dsd_ctx* c) { return c ? c->kv_format : -1; }

int dsd_ctx_create_ex(int device, const dsd_model_config* config, const dsd_ctx_options* options,
                      int kv_format, dsd_ctx** out) {
  return Guard([&]() {
    if (!config || !options || !out) Fail(DSD_EINVAL, "null argument");
    if (kv_format != DSD_KV_F32 && kv_format != DSD_KV_BF16 && kv_format != DSD_KV_FP8)
      Fail(DSD_EINVAL, "unknown kv_format");
    *out = nullptr;
    dsd_model_config cfg = *config;
    const dsd_ctx_options opt = *options;
    const int user_d = cfg.head_dim;
    // the reference accepts head_dim in (0, 128] for the sparse path and
    // (0, 256] for its dense baseline (src/cuda/kernels.cu:42-43); both use
    // this context
    if (cfg.num_heads <= 0 || user_d < 1 || user_d > 256)
      Fail(DSD_EINVAL, "head_dim must be in [1, 256] and num_heads positive");
    // physical head width: the next power of two, at least 4
    int D = 4;
    while (D < user_d) D *= 2;
    cfg.head_dim = D;
    if (kv_format == DSD_KV_BF16 && D < 8)
      Fail(DSD_EINVAL, "bf16 pages need head_dim > 4");
    if (kv_format == DSD_KV_FP8 && D < 16)
      Fail(DSD_EINVAL, "fp8 pages need head_dim > 8");
    if (cfg.page_size <= 0) Fail(DSD_EINVAL, "page_size must be positive");
    if (cfg.top_k_pages < 0) Fail(DSD_EINVAL, "top_k_pages must be non-negative");
    if (cfg.top_k_pages > dsdk::kSelectMaxK)
      Fail(DSD_EINVAL, "top_k_pages exceeds " + std::to_string(dsdk::kSelectMaxK));
    if (opt.capacity_pages < 0 || opt.max_batch < 0 || opt.max_candidates < 0 ||
        opt.max_selected < 0 || opt.max_requests < 0 || opt.max_pages_per_request < 0)
      Fail(DSD_EINVAL, "sparse CUDA context capacities must be non-negative");
    if (opt.max_batch > dsdk::kMaxBatch) Fail(DSD_EINVAL, "max_batch exceeds 1024");
    const int ept = cfg.num_heads * D;
    if (ept > 8192) Fail(DSD_EINVAL, "num_heads*head_dim exceeds 8192");

    Check(cudaSetDevice(device), "cudaSetDevice");
    cudaDeviceProp prop{};
    Check(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    if (prop.major < 10) Fail(DSD_EUNAVAILABLE, "an sm_100 (B200) GPU is required");

    auto* c = new dsd_ctx();
    try {
      c->device = device;
      c->cfg = cfg;
      c->opt = opt;
      c->ept = ept;
      c->user_head_dim = user_d;
      c->user_ept = cfg.num_heads * user_d;
      c->padded = user_d != D;
      c->num_sms = prop.multiProcessorCount;
      c->kv_format = kv_format;
      c->kv_elem = kv_format == DSD_KV_BF16 ? 2 : kv_format == DSD_KV_FP8 ? 1 : 4;
      c->attn = MakeAttnShape(cfg.num_heads, D, cfg.page_size, int(c->kv_elem));
      c->scale = 1.0f / std::sqrt(static_cast<float>(user_d));   // the caller's head_dim
      Check(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "stream");
      for (auto& e : c->ev) Check(cudaEventCreate(&e), "event");
      for (auto& e : c->ev_set1) Check(cudaEventCreate(&e), "event");
      Check(cudaEventCreateWithFlags(&c->ev_inputs, cudaEventDisableTiming), "event");
      Check(cudaStreamCreateWithFlags(&c->stream2, cudaStreamNonBlocking), "stream");
      Check(cudaEventCreateWithFlags(&c->ev_fork, cudaEventDisableTiming), "event");
      Check(cudaEventCreateWithFlags(&c->ev_join, cudaEventDisableTiming), "event");
      Check(cudaStreamCreateWithFlags(&c->copy_stream, cudaStreamNonBlocking), "stream");
      Check(cudaStreamCreateWithFlags(&c->up_stream, cudaStreamNonBlocking), "stream");
      for (cudaEvent_t* e : {&c->ev_part0_up, &c->ev_q1, &c->ev_out0, &c->ev_out0_done, &c->ev_q0,
                             &c->ev_in_ready[0], &c->ev_in_ready[1], &c->ev_graph_done[0],
                             &c->ev_graph_done[1], &c->ev_out_read[0], &c->ev_out_read[1]})
        Check(cudaEventCreateWithFlags(e, cudaEventDisableTiming), "event");

      const size_t cap = size_t(opt.capacity_pages);
      const size_t el = c->kv_elem;
      c->k_pool = DeviceAlloc<unsigned char>(cap * cfg.page_size * ept * el, "key pool");
      c->v_pool = DeviceAlloc<unsigned char>(cap * cfg.page_size * ept * el, "value pool");
      c->summary_floats = (cap + 127) / 128 * dsdk::summary_group_floats(ept);
      c->summaries = DeviceAlloc<unsigned char>(c->summary_floats * el, "page summaries");
      c->token_counts = DeviceAlloc<int>(cap, "token counts");
      c->live = DeviceAlloc<uint8_t>(cap, "live mask");
      Check(cudaMemsetAsync(c->summaries, 0, std::max<size_t>(1, c->summary_floats) * el,
                            c->stream), "memset");
      Check(cudaMemsetAsync(c->token_counts, 0, std::max<size_t>(1, cap) * 4, c->stream), "memset");
      Check(cudaMemsetAsync(c->live, 0, std::max<size_t>(1, cap), c->stream), "memset");
      c->host_counts.assign(cap, 0);

      if (opt.max_requests > 0) {
        c->table = DeviceAlloc<int>(size_t(opt.max_requests) * std::max(1, opt.max_pages_per_request),
                                    "request page tables");
        c->table_n = DeviceAlloc<int>(size_t(opt.max_requests), "request page counts");
        Check(cudaMemsetAsync(c->table_n, 0, size_t(opt.max_requests) * 4, c->stream), "memset");
        c->slot_pages.resize(size_t(opt.max_requests));
        for (int s = opt.max_requests - 1; s >= 0; --s) c->free_slots.push_back(s);
      }

      const int mb = std::max(1, opt.max_batch);
      const int mc = std::max(1, opt.max_candidates);
      const int ms = std::max(1, opt.max_selected);
      c->in_req_off = 16;
      c->in_q_off = AlignUp(c->in_req_off + size_t(mb + 1) * 4, 128);
      c->in_ids_off = AlignUp(c->in_q_off + size_t(mb) * ept * 4, 128);
      c->in_bytes = c->in_ids_off + size_t(mc) * 4;
      c->d_in = DeviceAlloc<unsigned char>(c->in_bytes, "step input");
      c->h_in = PinnedAlloc<unsigned char>(c->in_bytes, "step input staging");
      c->d_scores = DeviceAlloc<float>(mc, "scores");
      c->d_selected = DeviceAlloc<int>(ms, "selected ids");
      c->d_outputs = DeviceAlloc<float>(size_t(mb) * ept, "outputs");
      // one split-K unit holds at least one selected page
      c->d_part_acc = DeviceAlloc<float>(size_t(ms) * ept, "attention partials");
      c->d_part_ml = DeviceAlloc<float>(size_t(ms) * cfg.num_heads * 2, "attention partial stats");
      const size_t plan_ints = size_t(mb) * 2 + size_t(mb + 1) * 4 + 4;
      c->d_planbuf = DeviceAlloc<int>(plan_ints, "step plan");
      c->d_status = DeviceAlloc<int>(1, "status word");
      Check(cudaMemsetAsync(c->d_status, 0, 4, c->stream), "memset");
      c->h_outputs = PinnedAlloc<float>(size_t(mb) * ept, "output staging");
      c->h_outputs1 = PinnedAlloc<float>(size_t(mb) * ept, "output staging");
      c->h_scores1 = PinnedAlloc<float>(mc, "score staging");
      c->h_selected1 = PinnedAlloc<int>(ms, "selected staging");
      c->h_scores = PinnedAlloc<float>(mc, "score staging");
      c->h_selected = PinnedAlloc<int>(ms, "selected staging");
      c->h_status = PinnedAlloc<int>(1, "status staging");

      dsdk::StepPlan& p = c->plan;
      p.hdr = reinterpret_cast<const int*>(c->d_in);
      p.req = reinterpret_cast<const int*>(c->d_in + c->in_req_off);
      p.cand_ids = reinterpret_cast<const int*>(c->d_in + c->in_ids_off);
      p.table = c->table;
      p.table_n = c->table_n;
      p.table_stride = std::max(1, opt.max_pages_per_request);
      int* q = c->d_planbuf;
      p.n_cand = q; q += mb;
      p.id_base = q; q += mb;
      p.score_off = q; q += mb + 1;
      p.sel_off = q; q += mb + 1;
      p.tile_off = q; q += mb + 1;
      p.unit_off = q; q += mb + 1;
      p.misc = q;
      p.status = c->d_status;
      if (opt.max_requests > 0) {
        // second slot of queued steps: own input / output buffers, shared plan arrays
        c->d_in1 = DeviceAlloc<unsigned char>(c->in_bytes, "step input (slot 1)");
        c->d_outputs1 = DeviceAlloc<float>(size_t(mb) * ept, "outputs (slot 1)");
        c->plan1 = p;
        c->plan1.hdr = reinterpret_cast<const int*>(c->d_in1);
        c->plan1.req = reinterpret_cast<const int*>(c->d_in1 + c->in_req_off);
        c->plan1.cand_ids = reinterpret_cast<const int*>(c->d_in1 + c->in_ids_off);
      }

      Check(cudaFuncSetAttribute(dsdk::score_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)dsdk::kScoreSmem), "smem attribute");
      if (kv_format == DSD_KV_BF16) {
        SetScoreNarrowAttributes<__nv_bfloat16>();
        SetAllAttnAttributesNarrow<__nv_bfloat16>(c->attn.smem);
      } else if (kv_format == DSD_KV_FP8) {
        SetScoreNarrowAttributes<__nv_fp8_e4m3>();
        SetAllAttnAttributesNarrow<__nv_fp8_e4m3>(c->attn.smem);
      } else {
        SetAllAttnAttributes(c->attn.smem);
      }
      Check(cudaFuncSetAttribute(dsdk::select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 int(dsdk::kSelectSmem)), "smem attribute");
      Sync(c);
    } catch (...) {
      dsd_ctx_destroy(c);
      throw;
    }
    *out = c;
  });
}

int dsd_ctx_destroy(dsd_ctx* c) {
  if (!c) return DSD_OK;
  cudaSetDevice(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  if (c->copy_stream) cudaStreamSynchronize(c->copy_stream);
  if (c->up_stream) cudaStreamSynchronize(c->up_stream);
  for (auto& g : c->graphs) {
    if (g.exec) cudaGraphExecDestroy(g.exec);
    if (g.graph) cudaGraphDestroy(g.graph);
  }
  for (auto& u : c->uploaders) {
    if (u.stream) cudaStreamSynchronize(u.stream);
    for (int b = 0; b < 2; ++b) {
      if (u.pinned[b]) cudaFreeHost(u.pinned[b]);
      if (u.done[b]) cudaEventDestroy(u.done[b]);
    }
    if (u.stream) cudaStreamDestroy(u.stream);
  }
  void* dev[] = {c->k_pool, c->v_pool, c->summaries, c->token_counts, c->live, c->table,
                 c->table_n, c->d_in, c->d_in1, c->d_outputs1, c->d_scores, c->d_selected,
                 c->d_outputs, c->d_part_acc,
                 c->d_part_ml, c->d_planbuf, c->d_status, c->d_stage};
  for (void* p : dev)
    if (p) cudaFree(p);
  void* host[] = {c->h_in, c->h_outputs, c->h_scores, c->h_selected, c->h_status,
                  c->h_outputs1, c->h_scores1, c->h_selected1};
  for (void* p : host)
    if (p) cudaFreeHost(p);
  for (auto& e : c->ev)
    if (e) cudaEventDestroy(e);
  for (auto& e : c->ev_set1)
    if (e) cudaEventDestroy(e);
  if (c->ev_inputs) cudaEventDestroy(c->ev_inputs);
  if (c->ev_fork) cudaEventDestroy(c->ev_fork);
  if (c->ev_join) cudaEventDestroy(c->ev_join);
  for (cudaEvent_t e : {c->ev_part0_up, c->ev_q1, c->ev_out0, c->ev_out0_done, c->ev_q0,
                        c->ev_in_ready[0],
                        c->ev_in_ready[1], c->ev_graph_done[0], c->ev_graph_done[1],
                        c->ev_out_read[0], c->ev_out_read[1]})
    if (e) cudaEventDestroy(e);
  if (c->copy_stream) cudaStreamDestroy(c->copy_stream);
  if (c->up_stream) cudaStreamDestroy(c->up_stream);
  if (c->stream2) cudaStreamDestroy(c->stream2);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
  return DSD_OK;
}

int dsd_ctx_device_pointers(dsd_ctx* c, float** keys, float** values, float** summaries,
                            int32_t** token_counts) {
  return Guard([&]() {
    if (!c) Fail(DSD_EINVAL, "null context");
    if (keys) *keys = static_cast<float*>(c->k_pool);
    if (values) *values = static_cast<float*>(c->v_pool);
    if (summaries) *summaries = static_cast<float*>(c->summaries);
    if (token_counts) *token_counts = c->token_counts;
  });
}

void* dsd_ctx_stream(dsd_ctx* c) { return c ? static_cast<void*>(c->stream) : nullptr; }

int dsd_step_staging_wait(dsd_ctx* c) {
  return Guard([&]() {
    if (!c) Fail(DSD_EINVAL, "null context");
    SetDevice(c);
    WaitInputStaging(c);
  });
}

int dsd_step_host_buffers(dsd_ctx* c, float** queries, float** outputs) {
  return Guard([&]() {
    if (!c) Fail(DSD_EINVAL, "null context");
    RequireUnpadded(c, "dsd_step_host_buffers");
    if (queries) *queries = QPtr(c);
    if (outputs) *outputs = c->h_outputs;
  });
}

int dsd_pool_reset(dsd_ctx* c) {
  return Guard([&]() {
    if (!c) Fail(DSD_EINVAL, "null context");
    SetDevice(c);
    const size_t cap = size_t(c->opt.capacity_pages);
    Check(cudaMemsetAsync(c->summaries, 0, std::max<size_t>(1, c->summary_floats) * c->kv_elem,
                          c->stream), "memset");
    Check(cudaMemsetAsync(c->token_counts, 0, std::max<size_t>(1, cap) * 4, c->stream), "memset");
    Check(cudaMemsetAsync(c->live, 0, std::max<size_t>(1, cap), c->stream), "memset");
    std::fill(c->host_counts.begin(), c->host_counts.end(), 0);
    if (c->table_n) {
      Check(cudaMemsetAsync(c->table_n, 0, size_t(c->opt.max_requests) * 4, c->stream), "memset");
      c->slot_of.clear();
      c->free_slots.clear();
      for (int s = c->opt.max_requests - 1; s >= 0; --s) c->free_slots.push_back(s);
      for (auto& v : c->slot_pages) v.clear();
    }
    Sync(c);
  });
}

int dsd_pool_upload_pages(dsd_ctx* c, const int32_t* page_ids, const int32_t* token_counts, int n,
                          const float* keys, const float* values, int compute_summary) {
  return Guard([&]() {
    NvtxRange nvtx("dsd_pool_upload_pages");
    if (!c) Fail(DSD_EINVAL, "null context");
    if (n < 0) Fail(DSD_EINVAL, "negative page count");
    if (n == 0) return;
    if (!page_ids || !token_counts) Fail(DSD_EINVAL, "null page metadata");
    SetDevice(c);
    long long total_tokens = 0;
    for (int i = 0; i < n; ++i) {
      ValidatePage(c, page_ids[i]);
      if (token_counts[i] <= 0 || token_counts[i] > c->cfg.page_size)
        Fail(DSD_EINVAL, "token_count must be in (0, page_size]");
      total_tokens += token_counts[i];
    }
    if (!keys || !values) Fail(DSD_EINVAL, "host page payload pointers must be non-null");
    std::vector<float> pad_k, pad_v;
    if (c->padded) {
      pad_k = PadRows(c, keys, size_t(total_tokens));
      pad_v = PadRows(c, values, size_t(total_tokens));
      keys = pad_k.data();
      values = pad_v.data();
    }
    const size_t row = size_t(c->ept) * sizeof(float);
    // process in groups whose payload fits a bounded staging buffer
    const size_t max_stage = size_t(256) << 20;
    int i0 = 0;
    long long tok0 = 0;
    while (i0 < n) {
      int i1 = i0;
      long long toks = 0;
      while (i1 < n && (i1 == i0 || size_t(toks + token_counts[i1]) * row * 2 <= max_stage)) {
        toks += token_counts[i1];
        ++i1;
      }
      const int np = i1 - i0;
      const size_t payload = size_t(toks) * row;
      const size_t meta_off = AlignUp(2 * payload, 256);
      // meta = [long long src_token_off[np]][int page_ids[np]][int counts[np]]
      std::vector<long long> meta(size_t(np) + size_t(np + 1) / 2 * 2, 0);
      long long* m_off = meta.data();
      int* m_ids = reinterpret_cast<int*>(meta.data() + np);
      int* m_cnt = m_ids + np;
      long long acc = 0;
      for (int i = 0; i < np; ++i) {
        m_off[i] = acc;
        m_ids[i] = page_ids[i0 + i];
        m_cnt[i] = token_counts[i0 + i];
        acc += token_counts[i0 + i];
      }
      const size_t meta_bytes = meta.size() * sizeof(long long);
      EnsureStage(c, meta_off + meta_bytes);
      BulkH2D(c, {{c->d_stage, keys + tok0 * c->ept, payload},
                  {c->d_stage + payload, values + tok0 * c->ept, payload}});
      H2D(c, c->d_stage + meta_off, meta.data(), meta_bytes);
      const long long* d_off = reinterpret_cast<const long long*>(c->d_stage + meta_off);
      const int* d_ids = reinterpret_cast<const int*>(d_off + np);
      const int vec = c->ept / 4;
      dim3 grid(np, (vec + 255) / 256);
      WithKv(c, [&](auto tag) {
        using T = typename decltype(tag)::type;
        dsdk::upload_pages_kernel<T><<<grid, 256, 0, c->stream>>>(
            d_ids, d_ids + np, d_off, reinterpret_cast<const float*>(c->d_stage),
            reinterpret_cast<const float*>(c->d_stage + payload), c->ept, c->cfg.page_size,
            compute_summary, static_cast<T*>(c->k_pool), static_cast<T*>(c->v_pool),
            static_cast<T*>(c->summaries), c->token_counts, c->live);
      });
      Check(cudaGetLastError(), "upload kernel");
      Sync(c);  // the staging buffer is reused by the next group
      for (int i = i0; i < i1; ++i) c->host_counts[page_ids[i]] = token_counts[i];
      tok0 += toks;
      i0 = i1;
    }
  });
}

int dsd_pool_upload_summaries(dsd_ctx* c, const int32_t* page_ids, int n, const float* summaries) {
  return Guard([&]() {
    NvtxRange nvtx("dsd_pool_upload_summaries");
    if (!c) Fail(DSD_EINVAL, "null context");
    if (n <= 0) return;
    SetDevice(c);
    for (int i = 0; i < n; ++i) ValidatePage(c, page_ids[i]);
    std::vector<float> pad_s;
    if (c->padded) {
      pad_s = PadRows(c, summaries, size_t(n));
      summaries = pad_s.data();
    }
    const size_t sb = size_t(n) * c->ept * sizeof(float);
    const size_t ids_off = AlignUp(sb, 256);
    EnsureStage(c, ids_off + size_t(n) * 4);
    H2D(c, c->d_stage, summaries, sb);
    H2D(c, c->d_stage + ids_off, page_ids, size_t(n) * 4);
    WithKv(c, [&](auto tag) {
      using T = typename decltype(tag)::type;
      dsdk::set_summaries_kernel<T><<<n, 256, 0, c->stream>>>(
          reinterpret_cast<const int*>(c->d_stage + ids_off),
          reinterpret_cast<const float*>(c->d_stage), c->ept, static_cast<T*>(c->summaries));
    });
    Check(cudaGetLastError(), "summary kernel");
    Sync(c);
  });
}

int dsd_pool_prefill_synthetic(dsd_ctx* c, const int32_t* page_ids, const int32_t* token_counts,
                               int n, int request_id) {
  return Guard([&]() {
    NvtxRange nvtx("dsd_pool_prefill_synthetic");
    if (!c) Fail(DSD_EINVAL, "null context");
    if (n <= 0) return;
    SetDevice(c);
    for (int i = 0; i < n; ++i) {
      ValidatePage(c, page_ids[i]);
      if (token_counts[i] <= 0 || token_counts[i] > c->cfg.page_size)
        Fail(DSD_EINVAL, "token_count must be in (0, page_size]");
    }
    EnsureStage(c, size_t(n) * 8);
    H2D(c, c->d_stage, page_ids, size_t(n) * 4);
    H2D(c, c->d_stage + size_t(n) * 4, token_counts, size_t(n) * 4);
    const int* d = reinterpret_cast<const int*>(c->d_stage);
    WithKv(c, [&](auto tag) {
      using T = typename decltype(tag)::type;
      dsdk::prefill_synthetic_kernel<T><<<n, 256, 0, c->stream>>>(
          d, d + n, request_id, c->ept, c->user_head_dim, c->cfg.head_dim, c->cfg.page_size,
          static_cast<T*>(c->k_pool),
          static_cast<T*>(c->v_pool), static_cast<T*>(c->summaries), c->token_counts, c->live);
    });
    Check(cudaGetLastError(), "prefill kernel");
    // no wait: later users of the staging buffer are ordered on the same stream
    for (int i = 0; i < n; ++i) c->host_counts[page_ids[i]] = token_counts[i];
  });
}

int dsd_pool_generate_normal(dsd_ctx* c, const int32_t* page_ids, const int32_t* token_counts,
                             const int32_t* request_ids, const int32_t* first_token, int n,
                             uint64_t seed) {
  return Guard([&]() {
    NvtxRange nvtx("dsd_pool_generate_normal");
    if (!c) Fail(DSD_EINVAL, "null context");
    if (n <= 0) return;
    SetDevice(c);
    for (int i = 0; i < n; ++i) {
      ValidatePage(c, page_ids[i]);
      if (token_counts[i] <= 0 || token_counts[i] > c->cfg.page_size)
        Fail(DSD_EINVAL, "token_count must be in (0, page_size]");
    }
    const int chunk = 1 << 16;
    for (int i0 = 0; i0 < n; i0 += chunk) {
      const int m = std::min(chunk, n - i0);
      EnsureStage(c, size_t(chunk) * 16);
      int* d = reinterpret_cast<int*>(c->d_stage);
      H2D(c, d, page_ids + i0, size_t(m) * 4);
      H2D(c, d + m, token_counts + i0, size_t(m) * 4);
      H2D(c, d + 2 * m, request_ids + i0, size_t(m) * 4);
      H2D(c, d + 3 * m, first_token + i0, size_t(m) * 4);
      dim3 grid(m, (c->ept + 255) / 256);
      WithKv(c, [&](auto tag) {
        using T = typename decltype(tag)::type;
        dsdk::generate_normal_kernel<T><<<grid, 256, 0, c->stream>>>(
            d, d + m, d + 2 * m, d + 3 * m, c->ept, c->user_head_dim, c->cfg.head_dim,
            c->cfg.page_size, dsdk::normal_seed_mix(seed, 1), dsdk::normal_seed_mix(seed, 2),
            static_cast<T*>(c->k_pool), static_cast<T*>(c->v_pool),
            static_cast<T*>(c->summaries), c->token_counts, c->live);
      });
      Check(cudaGetLastError(), "generate kernel");
      Sync(c);
    }
    for (int i = 0; i < n; ++i) c->host_counts[page_ids[i]] = token_counts[i];
  });
}

void dsd_generate_normal_host(uint64_t seed, int kind, uint64_t first_index, int64_t count,
                              float* out) {
  const uint64_t mix = dsdk::normal_seed_mix(seed, kind);
  for (int64_t i = 0; i < count; ++i) out[i] = dsdk::normal_value(mix, first_index + uint64_t(i));
}

int dsd_append_tokens(dsd_ctx* c, const int32_t* page_ids, const int32_t* token_offsets,
                      const int32_t* request_ids, int n, const float* keys, const float* values) {
  return Guard([&]() {
    NvtxRange nvtx("dsd_append_tokens");
    if (!c) Fail(DSD_EINVAL, "null context");
    if (n <= 0) return;
    if (!keys || !values) Fail(DSD_EINVAL, "token payload pointers must be non-null");
    SetDevice(c);
    for (int i = 0; i < n; ++i) {
      ValidatePage(c, page_ids[i]);
      if (token_offsets[i] < 0 || token_offsets[i] >= c->cfg.page_size)
        Fail(DSD_ERANGE, "token_offset is outside the page");
    }
    std::vector<int> triples, counts;
    if (request_ids) {
      RequireTables(c);
      for (int i = 0; i < n; ++i) {
        if (token_offsets[i] != 0) continue;
        const int slot = SlotOf(c, request_ids[i], true);
        auto& pages = c->slot_pages[slot];
        if (int(pages.size()) >= c->opt.max_pages_per_request)
          Fail(DSD_EINVAL, "request page table is full");
        triples.insert(triples.end(), {slot, int(pages.size()), page_ids[i]});
        pages.push_back(page_ids[i]);
      }
    }
    std::vector<int> order, gpage, gfirst;
    GroupTokens(page_ids, token_offsets, n, &order, &gpage, &gfirst);
    const size_t row = size_t(c->ept) * 4;
    const size_t payload = size_t(n) * row;
    const size_t meta_off = AlignUp(2 * payload, 256);
    std::vector<int> meta;
    meta.insert(meta.end(), gpage.begin(), gpage.end());
    meta.insert(meta.end(), gfirst.begin(), gfirst.end());
    for (int i : order) meta.push_back(token_offsets[i]);
    EnsureStage(c, meta_off + meta.size() * 4);
    // payload in grouped order
    std::vector<float> sk(size_t(n) * c->ept), sv(size_t(n) * c->ept);
    for (int j = 0; j < n; ++j) {
      PadRowsInto(c, sk.data() + size_t(j) * c->ept, keys + size_t(order[j]) * c->user_ept, 1);
      PadRowsInto(c, sv.data() + size_t(j) * c->ept, values + size_t(order[j]) * c->user_ept, 1);
    }
    H2D(c, c->d_stage, sk.data(), payload);
    H2D(c, c->d_stage + payload, sv.data(), payload);
    H2D(c, c->d_stage + meta_off, meta.data(), meta.size() * 4);
    const int ng = int(gpage.size());
    const int* d = reinterpret_cast<const int*>(c->d_stage + meta_off);
    WithKv(c, [&](auto tag) {
      using T = typename decltype(tag)::type;
      dsdk::append_tokens_kernel<T><<<ng, 256, 0, c->stream>>>(
          d, d + ng, d + 2 * ng + 1, reinterpret_cast<const float*>(c->d_stage),
          reinterpret_cast<const float*>(c->d_stage + payload), c->ept, c->cfg.page_size,
          static_cast<T*>(c->k_pool), static_cast<T*>(c->v_pool), static_cast<T*>(c->summaries),
          c->token_counts, c->live);
    });
    Check(cudaGetLastError(), "append kernel");
    // no wait: later users of the staging buffer are ordered on the same stream
    for (int i = 0; i < n; ++i)
      c->host_counts[page_ids[i]] = std::max(c->host_counts[page_ids[i]], token_offsets[i] + 1);
    UploadTableEntries(c, triples, counts);
  });
}

int dsd_append_tokens_synthetic(dsd_ctx* c, const int32_t* page_ids, const int32_t* token_offsets,
                                const int32_t* request_ids, const int32_t* decode_steps, int n) {
  return Guard([&]() {
    NvtxRange nvtx("dsd_append_tokens_synthetic");
    if (!c) Fail(DSD_EINVAL, "null context");
    if (n <= 0) return;
    SetDevice(c);
    for (int i = 0; i < n; ++i) {
      ValidatePage(c, page_ids[i]);
      if (token_offsets[i] < 0 || token_offsets[i] >= c->cfg.page_size)
        Fail(DSD_ERANGE, "token_offset is outside the page");
    }
    std::vector<int> order, gpage, gfirst;
    GroupTokens(page_ids, token_offsets, n, &order, &gpage, &gfirst);
    std::vector<int> meta;
    meta.insert(meta.end(), gpage.begin(), gpage.end());
    meta.insert(meta.end(), gfirst.begin(), gfirst.end());
    for (int i : order) meta.push_back(token_offsets[i]);
    for (int i : order) meta.push_back(request_ids[i]);
    for (int i : order) meta.push_back(decode_steps[i]);
    EnsureStage(c, meta.size() * 4);
    H2D(c, c->d_stage, meta.data(), meta.size() * 4);
    const int ng = int(gpage.size());
    const int* d = reinterpret_cast<const int*>(c->d_stage);
    const int* toff = d + 2 * ng + 1;
    WithKv(c, [&](auto tag) {
      using T = typename decltype(tag)::type;
      dsdk::append_synthetic_kernel<T><<<ng, 256, 0, c->stream>>>(
          d, d + ng, toff, toff + n, toff + 2 * n, c->ept, c->user_head_dim, c->cfg.head_dim,
          c->cfg.page_size, static_cast<T*>(c->k_pool), static_cast<T*>(c->v_pool),
          static_cast<T*>(c->summaries), c->token_counts, c->live);
    });
    Check(cudaGetLastError(), "synthetic append kernel");
    // no wait: later users of the staging buffer are ordered on the same stream
    for (int i = 0; i < n; ++i)
      c->host_counts[page_ids[i]] = std::max(c->host_counts[page_ids[i]], token_offsets[i] + 1);
  });
}

int dsd_pool_free_pages(dsd_ctx* c, const int32_t* page_ids, int n) {
  return Guard([&]() {
    NvtxRange nvtx("dsd_pool_free_pages");
    if (!c) Fail(DSD_EINVAL, "null context");
    if (n <= 0) return;
    SetDevice(c);
    for (int i = 0; i < n; ++i) ValidatePage(c, page_ids[i]);
    EnsureStage(c, size_t(n) * 4);
    H2D(c, c->d_stage, page_ids, size_t(n) * 4);
    WithKv(c, [&](auto tag) {
      using T = typename decltype(tag)::type;
      dsdk::free_pages_kernel<T><<<n, 256, 0, c->stream>>>(
          reinterpret_cast<const int*>(c->d_stage), c->ept, static_cast<T*>(c->summaries),
          c->token_counts, c->live);
    });
    Check(cudaGetLastError(), "free kernel");
    // no wait: later users of the staging buffer are ordered on the same stream
    for (int i = 0; i < n; ++i) c->host_counts[page_ids[i]] = 0;
  });
}

int dsd_download_page(dsd_ctx* c, int page_id, float* keys, float* values, float* summary,
                      int32_t* token_count) {
  return Guard([&]() {
    if (!c) Fail(DSD_EINVAL, "null context");
    ValidatePage(c, page_id);
    SetDevice(c);
    const size_t pf = size_t(c->cfg.page_size) * c->ept;
    // padded head_dim: download pool rows, then drop the padding
    float* const user_keys = keys;
    float* const user_values = values;
    float* const user_summary = summary;
    std::vector<float> tk, tv, ts;
    if (c->padded) {
      if (keys) { tk.resize(pf); keys = tk.data(); }
      if (values) { tv.resize(pf); values = tv.data(); }
      if (summary) { ts.resize(size_t(c->ept)); summary = ts.data(); }
    }
    const size_t el = c->kv_elem;
    const bool narrow = c->kv_format != DSD_KV_F32;
    // bf16 / fp8 pools land in host bytes and widen to fp32 after the sync
    std::vector<unsigned char> hk(narrow && keys ? pf * el : 0), hv(narrow && values ? pf * el : 0),
        hs(narrow && summary ? size_t(c->ept) * el : 0);
    const auto* kp = static_cast<const unsigned char*>(c->k_pool);
    const auto* vp = static_cast<const unsigned char*>(c->v_pool);
    if (keys) D2H(c, narrow ? static_cast<void*>(hk.data()) : keys,
                  kp + size_t(page_id) * pf * el, pf * el);
    if (values) D2H(c, narrow ? static_cast<void*>(hv.data()) : values,
                    vp + size_t(page_id) * pf * el, pf * el);
    if (summary) {
      // gather the page's NC chunks of CW elements (stride 128*CW) into one row
      const int cw = dsdk::summary_chunk(c->ept);
      Check(cudaMemcpy2DAsync(narrow ? static_cast<void*>(hs.data()) : summary, size_t(cw) * el,
                              static_cast<const unsigned char*>(c->summaries) +
                                  dsdk::summary_row_base(page_id, c->ept) * el,
                              size_t(128) * cw * el, size_t(cw) * el, size_t(c->ept / cw),
                              cudaMemcpyDeviceToHost, c->stream), "summary download");
      CountD2H(c, size_t(c->ept) * el);
    }
    if (token_count) D2H(c, token_count, c->token_counts + page_id, 4);
    Sync(c);
    const bool fp8 = c->kv_format == DSD_KV_FP8;
    auto widen = [&](const std::vector<unsigned char>& src, float* dst) {
      const size_t n = src.size() / el;
      for (size_t i = 0; i < n; ++i) {
        if (fp8) {
          dst[i] = Fp8E4m3ToFloat(src[i]);
        } else {
          uint16_t h;
          std::memcpy(&h, src.data() + 2 * i, 2);
          const uint32_t b = uint32_t(h) << 16;
          std::memcpy(dst + i, &b, 4);
        }
      }
    };
    if (narrow) {
      if (keys) widen(hk, keys);
      if (values) widen(hv, values);
      if (summary) widen(hs, summary);
    }
    if (c->padded) {
      const size_t P = size_t(c->cfg.page_size);
      if (user_keys) UnpadRowsInto(c, user_keys, tk.data(), P);
      if (user_values) UnpadRowsInto(c, user_values, tv.data(), P);
      if (user_summary) UnpadRowsInto(c, user_summary, ts.data(), 1);
    }
  });
}

int dsd_download_metadata(dsd_ctx* c, int32_t* token_counts, uint8_t* live_mask) {
  return Guard([&]() {
    if (!c) Fail(DSD_EINVAL, "null context");
    SetDevice(c);
    const size_t cap = size_t(c->opt.capacity_pages);
    if (token_counts) D2H(c, token_counts, c->token_counts, cap * 4);
    if (live_mask) D2H(c, live_mask, c->live, cap);
    Sync(c);
  });
}

int dsd_get_transfer_stats(dsd_ctx* c, dsd_transfer_stats* out) {
  return Guard([&]() {
    if (!c || !out) Fail(DSD_EINVAL, "null argument");
    *out = c->stats;
  });
}

int dsd_reset_transfer_stats(dsd_ctx* c) {
  return Guard([&]() {
    if (!c) Fail(DSD_EINVAL, "null context");
    c->stats = dsd_transfer_stats{};
  });
}

int dsd_decode_batch(dsd_ctx* c, int batch, const float* queries, const int32_t* cand_offsets,
                     const int32_t* cand_ids, int output_mode, int timing, float* outputs,
                     float* scores, int32_t* selected, dsd_step_timing* out_timing) {
  return Guard([&]() {
    NvtxRange nvtx("dsd_decode_batch");
    if (!c) Fail(DSD_EINVAL, "null context");
    if (batch < 0) Fail(DSD_EINVAL, "negative batch");
    if (out_timing) *out_timing = dsd_step_timing{};
    if (batch == 0) return;
    if (!queries || !cand_offsets) Fail(DSD_EINVAL, "null step input");
    if (batch > c->opt.max_batch)
      Fail(DSD_EINVAL, "request batch exceeds sparse CUDA context capacity");
    if (cand_offsets[0] != 0) Fail(DSD_EINVAL, "cand_offsets[0] must be 0");
    int total_sel = 0;
    for (int r = 0; r < batch; ++r) {
      const int n = cand_offsets[r + 1] - cand_offsets[r];
      if (n < 0) Fail(DSD_EINVAL, "cand_offsets must be non-decreasing");
      total_sel += c->dense ? n : std::min(c->cfg.top_k_pages, n);
    }
    const int total_cand = cand_offsets[batch];
    if (total_cand > c->opt.max_candidates)
      Fail(DSD_EINVAL, "candidate page count exceeds sparse CUDA context capacity");
    if (total_sel > c->opt.max_selected)
      Fail(DSD_EINVAL, "selected page count exceeds sparse CUDA context capacity");
    for (int i = 0; i < total_cand; ++i) ValidatePage(c, cand_ids[i]);
    SetDevice(c);
    WaitInputStaging(c);
    int* hdr = HdrPtr(c);
    hdr[0] = batch;
    hdr[1] = 0;
    hdr[2] = c->dense;
    std::memcpy(ReqPtr(c), cand_offsets, size_t(batch + 1) * 4);
    std::memcpy(IdsPtr(c), cand_ids, size_t(total_cand) * 4);
    UploadQueries(c, queries, batch);
    if (total_cand > 0) H2D(c, c->d_in + c->in_ids_off, IdsPtr(c), size_t(total_cand) * 4);
    RunHostStep(c, batch, total_cand, total_sel, output_mode, timing, outputs, scores, selected,
                out_timing);
  });
}

int dsd_request_set_pages(dsd_ctx* c, int request_id, const int32_t* page_ids, int n) {
  return Guard([&]() {
    NvtxRange nvtx("dsd_request_set_pages");
    if (!c) Fail(DSD_EINVAL, "null context");
    RequireTables(c);
    if (n < 0 || n > c->opt.max_pages_per_request)
      Fail(DSD_EINVAL, "page count exceeds the request page table");
    for (int i = 0; i < n; ++i) ValidatePage(c, page_ids[i]);
    SetDevice(c);
    const int slot = SlotOf(c, request_id, true);
    std::vector<int> triples;
    c->slot_pages[slot].assign(page_ids, page_ids + n);
    for (int i = 0; i < n; ++i) triples.insert(triples.end(), {slot, i, page_ids[i]});
    UploadTableEntries(c, triples, std::vector<int>{slot, 0});
  });
}

int dsd_request_append_pages_multi(dsd_ctx* c, const int32_t* request_ids,
                                   const int32_t* page_ids, int n) {
  return Guard([&]() {
    NvtxRange nvtx("dsd_request_append_pages_multi");
    if (!c) Fail(DSD_EINVAL, "null context");
    RequireTables(c);
    if (n <= 0) return;
    if (!request_ids || !page_ids) Fail(DSD_EINVAL, "null argument");
    for (int i = 0; i < n; ++i) ValidatePage(c, page_ids[i]);
    SetDevice(c);
    // check every request's room (and free slots for new requests) first, so a
    // refused call changes nothing
    std::unordered_map<int, int> added;
    int new_requests = 0;
    for (int i = 0; i < n; ++i) {
      const auto it = c->slot_of.find(request_ids[i]);
      const int have = it == c->slot_of.end() ? 0 : int(c->slot_pages[it->second].size());
      int& a = added[request_ids[i]];
      if (it == c->slot_of.end() && a == 0) ++new_requests;
      if (have + ++a > c->opt.max_pages_per_request)
        Fail(DSD_EINVAL, "page count exceeds the request page table");
    }
    if (new_requests > int(c->free_slots.size()))
      Fail(DSD_ENOMEM, "no free request page-table slot");
    std::vector<int> triples;
    for (int i = 0; i < n; ++i) {
      const int slot = SlotOf(c, request_ids[i], true);
      auto& pages = c->slot_pages[slot];
      triples.insert(triples.end(), {slot, int(pages.size()), page_ids[i]});
      pages.push_back(page_ids[i]);
    }
    UploadTableEntries(c, triples, {});
  });
}

int dsd_request_append_pages(dsd_ctx* c, int request_id, const int32_t* page_ids, int n) {
  return Guard([&]() {
    NvtxRange nvtx("dsd_request_append_pages");
    if (!c) Fail(DSD_EINVAL, "null context");
    RequireTables(c);
    for (int i = 0; i < n; ++i) ValidatePage(c, page_ids[i]);
    SetDevice(c);
    const int slot = SlotOf(c, request_id, true);
    auto& pages = c->slot_pages[slot];
    if (int(pages.size()) + n > c->opt.max_pages_per_request)
      Fail(DSD_EINVAL, "page count exceeds the request page table");
    std::vector<int> triples;
    for (int i = 0; i < n; ++i) {
      triples.insert(triples.end(), {slot, int(pages.size()), page_ids[i]});
      pages.push_back(page_ids[i]);
    }
    UploadTableEntries(c, triples, {});
  });
}

int dsd_request_release(dsd_ctx* c, int request_id, int free_pages) {
  return Guard([&]() {
    NvtxRange nvtx("dsd_request_release");
    if (!c) Fail(DSD_EINVAL, "null context");
    RequireTables(c);
    auto it = c->slot_of.find(request_id);
    if (it == c->slot_of.end()) return;
    const int slot = it->second;
    std::vector<int> pages = c->slot_pages[slot];
    c->slot_pages[slot].clear();
    c->slot_of.erase(it);
    c->free_slots.push_back(slot);
    UploadTableEntries(c, {}, std::vector<int>{slot, 0});
    if (free_pages && !pages.empty()) {
      const int rc = dsd_pool_free_pages(c, pages.data(), int(pages.size()));
      if (rc != DSD_OK) Fail(rc, g_last_error);
    }
  });
}

int dsd_request_num_pages(dsd_ctx* c, int request_id) {
  if (!c) return -1;
  auto it = c->slot_of.find(request_id);
  if (it == c->slot_of.end()) return 0;
  return int(c->slot_pages[it->second].size());
}

namespace {
void PackSlots(dsd_ctx* c, const int32_t* request_ids, int batch, int* total_cand,
               int* total_sel) {
  if (batch > c->opt.max_batch) Fail(DSD_EINVAL, "request batch exceeds sparse CUDA context capacity");
  WaitInputStaging(c);
  int* req = ReqPtr(c);
  int tc = 0, ts = 0;
  for (int r = 0; r < batch; ++r) {
    const int slot = SlotOf(c, request_ids[r], false);
    req[r] = slot;
    const int n = int(c->slot_pages[slot].size());
    tc += n;
    ts += c->dense ? n : std::min(c->cfg.top_k_pages, n);
  }
  req[batch] = 0;
  if (tc > c->opt.max_candidates)
    Fail(DSD_EINVAL, "candidate page count exceeds sparse CUDA context capacity");
  if (ts > c->opt.max_selected)
    Fail(DSD_EINVAL, "selected page count exceeds sparse CUDA context capacity");
  int* hdr = HdrPtr(c);
  hdr[0] = batch;
  hdr[1] = 1;
  hdr[2] = c->dense;
  *total_cand = tc;
  *total_sel = ts;
}
}  // namespace

int dsd_decode_step(dsd_ctx* c, const int32_t* request_ids, int batch, const float* queries,
                    int output_mode, int timing, float* outputs, float* scores,
                    int32_t* selected, dsd_step_timing* out_timing) {
  return Guard([&]() {
    NvtxRange nvtx("dsd_decode_step");
    if (!c) Fail(DSD_EINVAL, "null context");
    RequireTables(c);
    if (out_timing) *out_timing = dsd_step_timing{};
    if (batch <= 0) return;
    if (!queries || !request_ids) Fail(DSD_EINVAL, "null step input");
    SetDevice(c);
    int tc = 0, ts = 0;
    PackSlots(c, request_ids, batch, &tc, &ts);
    const bool split = SplitIo(batch, timing);
    if (split) UploadQueriesSplit(c, queries, batch); else UploadQueries(c, queries, batch);
    RunHostStep(c, batch, tc, ts, output_mode, timing, outputs, scores, selected, out_timing,
                split);
  });
}

int dsd_decode_step_begin(dsd_ctx* c, const int32_t* request_ids, int batch,
                          const float* queries, int output_mode, int timing) {
  return Guard([&]() {
    NvtxRange nvtx("dsd_decode_step_begin");
    if (!c) Fail(DSD_EINVAL, "null context");
    RequireTables(c);
    if (c->pend_count >= 2) Fail(DSD_EINVAL, "two decode steps are already pending");
    if (batch <= 0) Fail(DSD_EINVAL, "empty batch");
    if (!queries || !request_ids) Fail(DSD_EINVAL, "null step input");
    SetDevice(c);
    int tc = 0, ts = 0;
    PackSlots(c, request_ids, batch, &tc, &ts);
    EnqueueStep(c, queries, batch, tc, ts, output_mode, timing);
  });
}

int dsd_decode_step_end(dsd_ctx* c, float* outputs, float* scores, int32_t* selected,
                        dsd_step_timing* out_timing) {
  return Guard([&]() {
    NvtxRange nvtx("dsd_decode_step_end");
    if (!c) Fail(DSD_EINVAL, "null context");
    if (out_timing) *out_timing = dsd_step_timing{};
    SetDevice(c);
    FinishStep(c, outputs, scores, selected, out_timing);
  });
}

int dsd_bind_requests(dsd_ctx* c, const int32_t* request_ids, int batch) {
  return Guard([&]() {
    if (!c) Fail(DSD_EINVAL, "null context");
    RequireTables(c);
    if (batch <= 0) Fail(DSD_EINVAL, "empty request set");
    SetDevice(c);
    int tc = 0, ts = 0;
    PackSlots(c, request_ids, batch, &tc, &ts);
    H2D(c, c->d_in, c->h_in, c->in_q_off);
    Sync(c);
    c->bound_batch = batch;
  });
}

int dsd_decode_bound(dsd_ctx* c, const float* d_queries, float* d_outputs) {
  return Guard([&]() {
    NvtxRange nvtx("dsd_decode_bound");
    if (!c) Fail(DSD_EINVAL, "null context");
    RequireUnpadded(c, "dsd_decode_bound");
    if (c->bound_batch <= 0) Fail(DSD_EINVAL, "no request set bound");
    SetDevice(c);
    LaunchStepGraph(c, d_queries, d_outputs, false);
  });
}

int dsd_decode_bound_timed(dsd_ctx* c, const float* d_queries, float* d_outputs,
                           dsd_step_timing* out_timing) {
  return Guard([&]() {
    NvtxRange nvtx("dsd_decode_bound_timed");
    if (!c) Fail(DSD_EINVAL, "null context");
    RequireUnpadded(c, "dsd_decode_bound_timed");
    if (c->bound_batch <= 0) Fail(DSD_EINVAL, "no request set bound");
    SetDevice(c);
    LaunchStepGraph(c, d_queries, d_outputs, true);
    if (out_timing) {
      CheckStatus(c);
      ReadTiming(c, out_timing);
    }
  });
}

int dsd_read_step_timing(dsd_ctx* c, dsd_step_timing* out_timing) {
  return Guard([&]() {
    if (!c || !out_timing) Fail(DSD_EINVAL, "null argument");
    SetDevice(c);
    CheckStatus(c);
    ReadTiming(c, out_timing);
  });
}

}  // extern "C"

// ------------------------------------------------------------------ allocation-free step
//
// For callers that may not allocate device memory (see dsd_decode_batch_noalloc
// in include/dsd_b200.h).  The step's working memory is one file-scope device
// array; its host-side name is only a stand-in, so host code passes the
// address that cudaGetSymbolAddress returns for the current device.
namespace {

constexpr int kNaMaxBatch = 256;
constexpr int kNaMaxCandidates = 131072;
constexpr int kNaMaxSelected = 8192;
constexpr int kNaMaxEpt = 4096;
constexpr int kNaMaxUnitsTarget = 512;   // split-K units requested from the plan
// units <= max(target, selected / kMaxPagesPerUnit) + batch
constexpr int kNaMaxUnits =
    (kNaMaxUnitsTarget > kNaMaxSelected / dsdk::kMaxPagesPerUnit
         ? kNaMaxUnitsTarget : kNaMaxSelected / dsdk::kMaxPagesPerUnit) + kNaMaxBatch;

// layout of the array, in 4-byte words (each region 64-word aligned)
constexpr size_t NaAlign(size_t w) { return (w + 63) / 64 * 64; }
constexpr size_t kNaHdr = 0;                                            // hdr[4] + status
constexpr size_t kNaReq = 64;                                           // cand offsets [B+1]
constexpr size_t kNaPlan = kNaReq + NaAlign(kNaMaxBatch + 1);           // 2B + 4(B+1) + 4
constexpr size_t kNaScores = kNaPlan + NaAlign(6 * (kNaMaxBatch + 1) + 4);
constexpr size_t kNaSelected = kNaScores + NaAlign(kNaMaxCandidates);
constexpr size_t kNaPartAcc = kNaSelected + NaAlign(kNaMaxSelected);
constexpr size_t kNaPartMl = kNaPartAcc + NaAlign(size_t(kNaMaxUnits) * kNaMaxEpt);
constexpr size_t kNaWords = kNaPartMl + NaAlign(size_t(kNaMaxUnits) * (kNaMaxEpt / 4) * 2);

static __device__ __align__(256) int g_noalloc_scratch[kNaWords];

struct NaDevice {
  bool ready = false;
  int* scratch = nullptr;   // device address of g_noalloc_scratch on this device
  int num_sms = 0;
};
std::mutex g_na_mutex;
NaDevice g_na[64];

__global__ void noalloc_init_kernel(int* hdr, int batch) {
  hdr[0] = batch;
  hdr[1] = 0;   // CSR mode
  hdr[4] = 0;   // status word: the previous call's bits must not leak
}

NaDevice& NaSetup(int device) {
  if (device < 0 || device >= 64) Fail(DSD_EINVAL, "device index out of range");
  std::lock_guard<std::mutex> lock(g_na_mutex);
  NaDevice& d = g_na[device];
  if (d.ready) return d;
  void* p = nullptr;
  Check(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(scratch)");
  Check(cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, device), "SM count");
  Check(cudaFuncSetAttribute(dsdk::score_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(dsdk::kScoreSmem)), "smem attribute");
  // largest attention stage for any shape within the limits
  const size_t max_attn = size_t(dsdk::kAttnStages) * dsdk::kAttnStageFloats * 4 +
                          dsdk::kAttnStages * 8;
  SetAllAttnAttributes(max_attn);
  Check(cudaFuncSetAttribute(dsdk::select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(dsdk::kSelectSmem)), "smem attribute");
  d.scratch = static_cast<int*>(p);
  d.ready = true;
  return d;
}

// Makes `device` current for the call and restores the caller's device on
// every exit path (including a failure thrown by Fail/Check).
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int device) {
    Check(cudaGetDevice(&prev), "cudaGetDevice");
    if (prev != device) Check(cudaSetDevice(device), "cudaSetDevice");
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace

extern "C" int dsd_decode_batch_noalloc(int device, const dsd_model_config* config,
                                        int capacity_pages, int batch,
                                        const int32_t* cand_offsets, const int32_t* d_cand_ids,
                                        const float* d_queries, const float* d_summaries,
                                        const float* d_keys, const float* d_values,
                                        const int32_t* d_token_counts, float* d_outputs,
                                        void* stream) {
  return Guard([&]() {
    NvtxRange nvtx("dsd_decode_batch_noalloc");
    if (!config || !cand_offsets) Fail(DSD_EINVAL, "null argument");
    const dsd_model_config cfg = *config;
    const int D = cfg.head_dim;
    if (cfg.num_heads <= 0 || D < 4 || D > 128 || (D & (D - 1)) != 0 || cfg.page_size <= 0 ||
        cfg.top_k_pages < 0 || cfg.top_k_pages > dsdk::kSelectMaxK)
      Fail(DSD_EINVAL, "unsupported model config");
    const int ept = cfg.num_heads * D;
    if (ept > kNaMaxEpt) Fail(DSD_EINVAL, "num_heads*head_dim exceeds the no-alloc limit 4096");
    if (capacity_pages <= 0) Fail(DSD_EINVAL, "capacity_pages must be positive");
    if (batch < 0 || batch > kNaMaxBatch)
      Fail(DSD_EINVAL, "batch exceeds the no-alloc limit of 256 requests");
    if (batch == 0) return;
    if (cand_offsets[0] != 0) Fail(DSD_EINVAL, "cand_offsets[0] must be 0");
    long long total_sel = 0;
    for (int r = 0; r < batch; ++r) {
      const int n = cand_offsets[r + 1] - cand_offsets[r];
      if (n < 0) Fail(DSD_EINVAL, "cand_offsets must be non-decreasing");
      total_sel += std::min(cfg.top_k_pages, n);
    }
    if (cand_offsets[batch] > kNaMaxCandidates)
      Fail(DSD_EINVAL, "total candidates exceed the no-alloc limit of 131072");
    if (total_sel > kNaMaxSelected)
      Fail(DSD_EINVAL, "total selected pages exceed the no-alloc limit of 8192");
    const void* ptrs[] = {d_queries, d_summaries, d_keys, d_values, d_outputs};
    for (const void* p : ptrs)
      if (!p || (reinterpret_cast<uintptr_t>(p) & 15u) != 0)
        Fail(DSD_EINVAL, "device float arrays must be non-null and 16-byte aligned");
    if (!d_token_counts || (cand_offsets[batch] > 0 && !d_cand_ids))
      Fail(DSD_EINVAL, "null device array");

    DeviceGuard device_guard(device);
    NaDevice& nd = NaSetup(device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int* base = nd.scratch;

    dsdk::StepPlan plan{};
    plan.hdr = base + kNaHdr;
    plan.req = base + kNaReq;
    plan.cand_ids = d_cand_ids;
    plan.table = nullptr;
    plan.table_n = nullptr;
    plan.table_stride = 1;
    int* q = base + kNaPlan;
    plan.n_cand = q; q += kNaMaxBatch;
    plan.id_base = q; q += kNaMaxBatch;
    plan.score_off = q; q += kNaMaxBatch + 1;
    plan.sel_off = q; q += kNaMaxBatch + 1;
    plan.tile_off = q; q += kNaMaxBatch + 1;
    plan.unit_off = q; q += kNaMaxBatch + 1;
    plan.misc = q;
    plan.status = base + kNaHdr + 4;
    plan.capacity = capacity_pages;   // the ids are checked on the device before use
    float* scores = reinterpret_cast<float*>(base + kNaScores);
    int* selected = base + kNaSelected;
    float* part_acc = reinterpret_cast<float*>(base + kNaPartAcc);
    float* part_ml = reinterpret_cast<float*>(base + kNaPartMl);

    noalloc_init_kernel<<<1, 1, 0, s>>>(base + kNaHdr, batch);
    Check(cudaMemcpyAsync(base + kNaReq, cand_offsets, size_t(batch + 1) * sizeof(int),
                          cudaMemcpyHostToDevice, s), "offsets copy");
    const int target = std::min(kNaMaxUnitsTarget, 2 * nd.num_sms);
    const float scale = 1.0f / std::sqrt(static_cast<float>(D));
    dsdk::plan_kernel<<<1, dsdk::kPlanThreads, 0, s>>>(plan, cfg.top_k_pages, target, 2 * nd.num_sms);
    dsdk::score_kernel<<<2 * nd.num_sms, dsdk::kScoreThreads, dsdk::kScoreSmem, s>>>(
        plan, d_queries, d_summaries, ept, scale, scores, 0, 1);
    dsdk::select_kernel<<<std::min(batch, 2 * nd.num_sms), dsdk::kSelectThreads,
                          dsdk::kSelectSmem, s>>>(plan, scores, selected, 0, 1);
    const AttnShape ash = MakeAttnShape(cfg.num_heads, D, cfg.page_size);
    LaunchAttn(ash, nd.num_sms, s, plan, d_queries, d_keys, d_values, d_token_counts, selected,
               part_acc, part_ml, cfg.num_heads, D, cfg.page_size, scale);
    const int pairs = batch * cfg.num_heads;
    dsdk::combine_kernel<<<std::max(1, std::min((pairs + 7) / 8, 8 * nd.num_sms)), 256, 0, s>>>(
        plan, part_acc, part_ml, cfg.num_heads, D, d_outputs, 0, 1);
    Check(cudaGetLastError(), "kernel launch");
    int status = 0;
    Check(cudaMemcpyAsync(&status, plan.status, sizeof(int), cudaMemcpyDeviceToHost, s),
          "status read");
    Check(cudaStreamSynchronize(s), "stream synchronize");
    if (status & dsdk::kStatusTimeout) Fail(DSD_ETIMEOUT, "a device-side wait exceeded its budget");
    if (status) Fail(DSD_EINVAL, "a candidate page id is outside [0, capacity_pages)");
  });
}
