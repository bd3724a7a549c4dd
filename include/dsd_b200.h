/*
 * dsd_b200.h -- C ABI of the B200 batched page-level dynamic sparse decode path.
 *
 * Plain C: pointers, sizes and status codes only.  Every function returns
 * DSD_OK (0) or a negative-free error code below and leaves a message for
 * dsd_last_error() (thread local).  Host pointers are borrowed for the call.
 *
 * The entry points replace the device side of the reference's
 * SparseCudaContext / DevicePagePool (JudySun233/15-618_Dynamic_Sparse_Decode):
 *   include/dsd/cuda_sparse_attention.h:50-104  (SparseCudaContext)
 *   include/dsd/device_page_pool.h:17-100       (DevicePagePool)
 * The C++ drop-in classes in the package (csrc/host) are thin wrappers over
 * this ABI; a C, cgo, JNI or ctypes caller binds it directly.
 *
 * Data layout in HBM (one context = one GPU).  D below is the stored head
 * width: the caller's head_dim when it is a power of two >= 4, otherwise the
 * next power of two (at least 4), the extra columns zero.  Every host row an
 * entry point takes or returns (queries, outputs, keys, values, summaries)
 * has the caller's num_heads*head_dim elements; the widening is internal.
 *   keys, values  float [capacity_pages][page_size][H*D]   page-major, 16 B aligned rows
 *   summaries     mean key of each page, chunk-major in groups of 128 pages:
 *                 element e of page p at ((p/128*NC + e/CW)*128 + p%128)*CW + e%CW,
 *                 CW = min(64, largest power of two dividing H*D), NC = H*D/CW
 *   token_counts  int32 [capacity_pages]; live  uint8 [capacity_pages]
 *   request page tables int32 [max_requests][max_pages_per_request] (+ counts)
 */
#ifndef DSD_B200_H_
#define DSD_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  The C++ wrapper maps them to the reference's exception
 * types: EINVAL -> std::invalid_argument, ERANGE -> std::out_of_range,
 * everything else -> std::runtime_error (include/dsd/cuda_utils.h:43-53). */
enum {
  DSD_OK = 0,
  DSD_EINVAL = 1,       /* bad argument / size / capacity overflow            */
  DSD_ERANGE = 2,       /* page id or token offset out of range               */
  DSD_ENOMEM = 3,       /* device allocation failed / page pool exhausted     */
  DSD_ECUDA = 4,        /* CUDA runtime error                                 */
  DSD_ETIMEOUT = 5,     /* a bounded device-side wait gave up                 */
  DSD_EUNAVAILABLE = 6  /* no sm_100 GPU visible                              */
};

/* SparseBatchOutputMode (include/dsd/cuda_sparse_attention.h:19-23). */
enum { DSD_OUTPUT_NONE = 0, DSD_OUTPUT_OUTPUTS = 1, DSD_OUTPUT_DEBUG = 2 };

/* ModelConfig (include/dsd/config.h:5-10). */
typedef struct dsd_model_config {
  int32_t num_heads;
  int32_t head_dim;     /* 1..256 (the reference: sparse 1..128, dense 1..256); stored
                           padded to a power of two */
  int32_t page_size;
  int32_t top_k_pages;
} dsd_model_config;

/* Capacities fixed at creation (SparseCudaContext ctor arguments,
 * include/dsd/cuda_sparse_attention.h:52-57, plus the device page tables). */
typedef struct dsd_ctx_options {
  int32_t capacity_pages;
  int32_t max_batch;              /* <= 1024 */
  int32_t max_candidates;         /* total candidate pages per step */
  int32_t max_selected;           /* total selected pages per step */
  int32_t max_requests;           /* device page-table slots (0 = none) */
  int32_t max_pages_per_request;  /* page-table row length */
} dsd_ctx_options;

/* StageTimings of one step (include/dsd/types.h:69-75); CUDA-event ms. */
typedef struct dsd_step_timing {
  float score_ms;
  float topk_ms;
  float attention_ms;   /* attention + log-sum-exp combine */
  float total_ms;       /* first to last kernel of the step */
} dsd_step_timing;

/* DeviceTransferStats (include/dsd/types.h:50-57). */
typedef struct dsd_transfer_stats {
  uint64_t h2d_bytes, d2h_bytes, h2d_calls, d2h_calls, h2d_large_calls, d2h_large_calls;
} dsd_transfer_stats;

typedef struct dsd_ctx dsd_ctx;

const char* dsd_last_error(void);

/* SparseAttentionCudaAvailable (include/dsd/cuda_sparse_attention.h:17):
 * 1 when an sm_100 device is visible, else 0. */
int dsd_available(void);

/* SparseCudaContext ctor / dtor (src/cuda/sparse_batched_attention.cu:444-549);
 * allocates the page pool (DevicePagePool ctor, src/device_page_pool.cpp:241-284)
 * and all per-step scratch once.  No allocation happens per step. */
int dsd_ctx_create(int device, const dsd_model_config* config, const dsd_ctx_options* options,
                   dsd_ctx** out);
int dsd_ctx_destroy(dsd_ctx* ctx);

/* Page element formats.  DSD_KV_F32 is the reference's format (fp32 pages and
 * summaries, the parity path).  DSD_KV_BF16 stores K, V and summaries as bf16
 * (round to nearest even on every store) while queries, dot products, the
 * softmax and outputs stay fp32; it halves the bytes a step reads.  A key is
 * rounded before it enters a summary, a summary is computed in fp32 and
 * rounded once, and a running-mean update reads the stored bf16 mean.  No
 * reference counterpart: the reference pool is fp32 only
 * (src/device_page_pool.cpp:241-284); the host API (float payloads in, float
 * downloads out) is the same for every format.  DSD_KV_FP8 follows the same
 * rules with fp8 e4m3 storage (a quarter of the fp32 bytes). */
#define DSD_KV_F32 0
#define DSD_KV_BF16 1
#define DSD_KV_FP8 2   /* fp8 e4m3 (saturating, round to nearest even); head_dim >= 16 */
/* dsd_ctx_create with an explicit page format (bf16 needs head_dim > 4,
 * fp8 head_dim > 8).
 * dsd_ctx_device_pointers then returns the pools as raw storage of that
 * format (cast the float pointers to __nv_bfloat16* for DSD_KV_BF16). */
int dsd_ctx_create_ex(int device, const dsd_model_config* config, const dsd_ctx_options* options,
                      int kv_format, dsd_ctx** out);
/* The context's DSD_KV_* format, -1 for a null context. */
int dsd_ctx_kv_format(dsd_ctx* ctx);

/* Device pointers for callers that keep their own data in HBM (bench, tests).
 * The arrays are in the stored layout above (padded head width D). */
int dsd_ctx_device_pointers(dsd_ctx* ctx, float** keys, float** values, float** summaries,
                            int32_t** token_counts);
/* The CUDA stream every call of this context is ordered on (cudaStream_t). */
void* dsd_ctx_stream(dsd_ctx* ctx);
/* The context's pinned per-step staging: queries [max_batch][H*D] and outputs
 * [max_batch][H*D].  Passing these pointers as `queries` / `outputs` to
 * dsd_decode_batch / dsd_decode_step skips one host copy each way.  Valid
 * until the context is destroyed; the next step overwrites them.  Rows are in
 * the stored layout, so a context whose head_dim is padded returns DSD_EINVAL
 * (pass ordinary host rows instead). */
int dsd_step_host_buffers(dsd_ctx* ctx, float** queries, float** outputs);
/* Waits until the previous step's upload of the pinned query staging has
 * completed; call before writing the staging while a step is in flight. */
int dsd_step_staging_wait(dsd_ctx* ctx);

/* DevicePagePool::Reset (src/device_page_pool.cpp:286-302): zero counts, live
 * flags and summaries; drop every request page table. */
int dsd_pool_reset(dsd_ctx* ctx);

/* DevicePagePool::UploadPage / UploadPagesFromCache / UploadPromptDirect
 * (src/device_page_pool.cpp:304-624).  keys/values hold the pages' tokens
 * back to back ([sum token_counts][H*D]).  compute_summary = 1 computes the
 * summary on the device with PagedKvCache::AppendPage's formula
 * (src/paged_kv_cache.cpp:88-99: token-order sum, then * (1/n)); 0 leaves it
 * zero (AppendPage with compute_summary = false). */
int dsd_pool_upload_pages(dsd_ctx* ctx, const int32_t* page_ids, const int32_t* token_counts,
                          int n, const float* keys, const float* values, int compute_summary);

/* Overwrite page summaries with host values ([n][H*D]), e.g. a host cache
 * whose summaries were built by running-mean appends. */
int dsd_pool_upload_summaries(dsd_ctx* ctx, const int32_t* page_ids, int n,
                              const float* summaries);

/* DevicePagePool::PrefillPromptSynthetic (src/device_page_pool.cpp:626-679):
 * K/V from the reference's integer hash; summary by AppendPage's formula. */
int dsd_pool_prefill_synthetic(dsd_ctx* ctx, const int32_t* page_ids,
                               const int32_t* token_counts, int n, int request_id);

/* Long-context workload generator (no reference counterpart: the reference
 * draws everything on the host).  Page i holds tokens
 * [first_token[i], first_token[i] + token_counts[i]) of request
 * request_ids[i]; values are Irwin-Hall(4) normals of (seed, kind, index),
 * summaries by AppendPage's formula. */
int dsd_pool_generate_normal(dsd_ctx* ctx, const int32_t* page_ids, const int32_t* token_counts,
                             const int32_t* request_ids, const int32_t* first_token, int n,
                             uint64_t seed);
/* Host copy of the same generator (queries, checks). kind 0=query 1=key 2=value. */
void dsd_generate_normal_host(uint64_t seed, int kind, uint64_t first_index, int64_t count,
                              float* out);

/* DevicePagePool::UploadTokensDirect / UploadTokensFromCache + K7
 * (src/device_page_pool.cpp:700-902), with the summary updated ON DEVICE by
 * PagedKvCache::AppendToken's running mean (src/paged_kv_cache.cpp:231-238).
 * Token i goes to (page_ids[i], token_offsets[i]); the page's count becomes
 * token_offsets[i] + 1.  Tokens of one page must come in offset order.
 * request_ids may be NULL; otherwise a token whose offset is 0 also appends
 * its page to that request's device page table. */
int dsd_append_tokens(dsd_ctx* ctx, const int32_t* page_ids, const int32_t* token_offsets,
                      const int32_t* request_ids, int n, const float* keys, const float* values);

/* DevicePagePool::AppendTokensSynthetic + K9 (src/device_page_pool.cpp:904-983). */
int dsd_append_tokens_synthetic(dsd_ctx* ctx, const int32_t* page_ids,
                                const int32_t* token_offsets, const int32_t* request_ids,
                                const int32_t* decode_steps, int n);

/* DevicePagePool::MarkPagesFree (src/device_page_pool.cpp:989-1043). */
int dsd_pool_free_pages(dsd_ctx* ctx, const int32_t* page_ids, int n);

/* DevicePagePool::DownloadPage / DownloadMetadata (src/device_page_pool.cpp:1045-1091).
 * keys/values receive page_size*H*D floats, summary H*D (each nullable). */
int dsd_download_page(dsd_ctx* ctx, int page_id, float* keys, float* values, float* summary,
                      int32_t* token_count);
int dsd_download_metadata(dsd_ctx* ctx, int32_t* token_counts, uint8_t* live_mask);

int dsd_get_transfer_stats(dsd_ctx* ctx, dsd_transfer_stats* out);
int dsd_reset_transfer_stats(dsd_ctx* ctx);

/* SparseCudaContext::RunBatch (src/cuda/sparse_batched_attention.cu:574-838)
 * with the caller's candidate lists in CSR: request r scores candidates
 * cand_ids[cand_offsets[r] .. cand_offsets[r+1]) against summaries with the
 * query queries[r*H*D ..], selects min(k, n_r) pages (score desc, page id
 * asc) and attends over their tokens.  Outputs [batch][H*D]; in
 * DSD_OUTPUT_DEBUG mode scores [C] (candidate order) and selected ids packed
 * by min(k, n_r) per request.  timing != 0 fills *timing with CUDA events. */
int dsd_decode_batch(dsd_ctx* ctx, int batch, const float* queries, const int32_t* cand_offsets,
                     const int32_t* cand_ids, int output_mode, int timing, float* outputs,
                     float* scores, int32_t* selected, dsd_step_timing* out_timing);

/* Device request page tables (north-star item 5: no host CSR packing).
 * set replaces the request's page list, append extends it, release drops it
 * (and frees its pages on the device when free_pages != 0). */
int dsd_request_set_pages(dsd_ctx* ctx, int request_id, const int32_t* page_ids, int n);
int dsd_request_append_pages(dsd_ctx* ctx, int request_id, const int32_t* page_ids, int n);
/* Appends page_ids[i] to the page table of request_ids[i], i = 0..n-1 in
 * order, with one upload for all of them (the continuous step's new pages of
 * many requests; per-request equivalent: dsd_request_append_pages). */
int dsd_request_append_pages_multi(dsd_ctx* ctx, const int32_t* request_ids,
                                   const int32_t* page_ids, int n);
int dsd_request_release(dsd_ctx* ctx, int request_id, int free_pages);
int dsd_request_num_pages(dsd_ctx* ctx, int request_id);

/* One decode step over requests whose candidates are their device page
 * tables (the continuous-batching step).  The CSR offsets are a device prefix
 * sum; only the queries cross H2D and the outputs D2H.  With at least two
 * requests, a page-locked `outputs` buffer (cudaHostAlloc / pinned memory) is
 * written by the kernels directly over PCIe; any other buffer is filled from
 * the context's staging.  Either way the call returns with the outputs in
 * place.  A context keeps a step graph per such buffer (at most 16). */
int dsd_decode_step(dsd_ctx* ctx, const int32_t* request_ids, int batch, const float* queries,
                    int output_mode, int timing, float* outputs, float* scores,
                    int32_t* selected, dsd_step_timing* out_timing);

/* The same step split in two, so the caller's host work overlaps the GPU:
 * begin uploads the queries and queues the step and its result copies;
 * end waits for the OLDEST pending step and returns its results (copied out
 * of the context's pinned staging).  Work the caller queues on this context
 * in between (token appends, frees, the next begin) runs after the step on
 * the GPU.  Up to two steps may be pending; they alternate between two device
 * input/output slots whose uploads and result copies run on their own
 * streams, so one step's copies overlap the other's kernels.  Pinned caller
 * queries passed to begin must stay unchanged until the step ends. */
int dsd_decode_step_begin(dsd_ctx* ctx, const int32_t* request_ids, int batch,
                          const float* queries, int output_mode, int timing);
int dsd_decode_step_end(dsd_ctx* ctx, float* outputs, float* scores, int32_t* selected,
                        dsd_step_timing* out_timing);

/* Device-resident variant: bind a request set once, then run steps whose
 * queries and outputs already live in HBM ([batch][H*D] each).  The step is
 * replayed from a CUDA graph; nothing crosses PCIe.  Device rows are used as
 * they are, so these two need head_dim a power of two >= 4 (DSD_EINVAL
 * otherwise). */
int dsd_bind_requests(dsd_ctx* ctx, const int32_t* request_ids, int batch);
int dsd_decode_bound(dsd_ctx* ctx, const float* d_queries, float* d_outputs);
/* Same step from a second graph that also records a CUDA event between the
 * stages.  out_timing != NULL waits for the step and fills it; NULL returns
 * at once (steps stay back to back) and dsd_read_step_timing later reads the
 * stage times of the most recent timed step. */
int dsd_decode_bound_timed(dsd_ctx* ctx, const float* d_queries, float* d_outputs,
                           dsd_step_timing* out_timing);
int dsd_read_step_timing(dsd_ctx* ctx, dsd_step_timing* out_timing);

/* Dense baseline (DenseCudaContext, src/cuda/kernels.cu:76-330 in the
 * reference): with dense != 0 every later step of this context attends over
 * ALL candidate pages in candidate order (no scoring, no top-k); selected
 * counts then equal candidate counts, so max_selected must cover them. */
int dsd_set_attention_mode(dsd_ctx* ctx, int dense);

/* Number of kernels one decode step launches (for launch accounting). */
int dsd_kernels_per_step(void);

/* Failure-detection self-test: launches a kernel whose single wait (on a
 * shared-memory barrier that nothing completes) uses the same bounded-wait
 * routine as the decode kernels, with `budget_cycles` instead of ~2^31.
 * Returns DSD_ETIMEOUT after the wait gives up; the context stays usable. */
int dsd_selftest_bounded_wait(dsd_ctx* ctx, int64_t budget_cycles);

/* Allocation-free decode step.  No counterpart in the reference: it exists
 * for callers that must not allocate device memory at all -- code running
 * under a host framework that owns every allocation (a custom caching
 * allocator or a fixed memory budget), or code that runs where cudaMalloc is
 * not allowed.  It needs no context: the caller passes every input and the
 * output as device pointers, and the step's working memory (plan, scores,
 * selected ids, split-K partials) lives in one static device array of about
 * 20 MiB that every GPU which loads this library keeps until the process
 * exits.  Limits: batch <= 256, total candidates <= 131072, total selected
 * pages (sum of min(k, n_r)) <= 8192, num_heads*head_dim <= 4096, head_dim a
 * power of two in [4, 128] (device rows are used as they are), top_k <= 4096;
 * larger sizes are rejected with DSD_EINVAL.
 *   capacity_pages  pages in the pool the device arrays below describe
 *   cand_offsets  HOST array [batch+1] (validated here, copied to the device)
 *   d_cand_ids, d_queries [batch][H*D], d_summaries (pool summary layout),
 *   d_keys/d_values [cap][page_size][H*D], d_token_counts [cap], d_outputs
 *   [batch][H*D]: device pointers, float arrays 16-byte aligned; d_summaries in the
 *   pool's summary layout above (e.g. the pointer dsd_ctx_device_pointers returns).
 * The page ids live on the device, so the first kernel checks every one
 * against capacity_pages before any summary or page is read; an id outside
 * [0, capacity_pages) makes the call return DSD_EINVAL with nothing loaded
 * (d_outputs is then zero-filled).  Work is queued on `stream` (a
 * cudaStream_t, NULL = default stream) and the call waits for it.  The call
 * makes `device` current while it runs and restores the caller's current
 * device before it returns.
 * The first call on a device looks up the array's device address and sets
 * kernel attributes; make that first call before any stream capture.  All
 * calls share the one array: calls that overlap on the GPU (other threads,
 * other streams) race and must be serialised by the caller. */
int dsd_decode_batch_noalloc(int device, const dsd_model_config* config, int capacity_pages,
                             int batch,
                             const int32_t* cand_offsets, const int32_t* d_cand_ids,
                             const float* d_queries, const float* d_summaries,
                             const float* d_keys, const float* d_values,
                             const int32_t* d_token_counts, float* d_outputs, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DSD_B200_H_ */
