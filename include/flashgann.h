/*
 * flashgann.h -- C ABI of the B200 FlashGANN search engine (libflashgann.so).
 *
 * Drop-in boundary for the reference's search path (SophiaSun18/FlashGANN):
 * plain pointers and sizes, no C++ or torch types, every failure returned as
 * a status code instead of the reference's exit()/throw.  Each entry point
 * names the reference interface it replaces (file:line in that project).
 *
 * Threading: an fg_index may be used by one host thread at a time.
 * Devices: every call runs on the device the index was created on and
 * restores the caller's current device before returning.
 */
#ifndef FLASHGANN_H
#define FLASHGANN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (the reference exits or throws instead) ---- */
#define FG_OK 0
#define FG_ERR_IO 1          /* file cannot be opened or is short      (qg.hpp:22-23 throws) */
#define FG_ERR_FORMAT 2      /* codebook/vecs content inconsistent     (data_io.hpp:41 asserts) */
#define FG_ERR_ARG 3         /* invalid argument                       */
#define FG_ERR_CUDA 4        /* CUDA runtime error                     (utils.cuh:42-50 exits) */
#define FG_ERR_OOM 5         /* not enough device memory               (gpu_search_adaptive.cu:61-63 throws) */
#define FG_ERR_UNSUPPORTED 6 /* outside this build's supported envelope */
#define FG_ERR_NO_DEVICE 7   /* no CUDA device / product kernels not loadable */

/* ---- metric (include/metric.hpp:9) ---- */
#define FG_METRIC_L2 0
#define FG_METRIC_IP 1

/* ---- device argument of fg_index_load / fg_index_create: the calling
 * thread's current CUDA device, which is where the reference's search runs
 * (gpu_search_adaptive.cu:30-34) ---- */
#define FG_DEVICE_CURRENT (-1)

typedef struct fg_index fg_index;

/* Codebook layout in float words, as QuantizationGraph's getters report it
 * (include/qg.hpp:49-60,66-73). */
typedef struct fg_layout {
    uint64_t num_nodes;
    uint64_t dim;
    uint64_t padded_dim;
    uint64_t code_offset;
    uint64_t factor_offset;
    uint64_t neighbor_offset;
    uint64_t row_offset;
    int32_t degree;
    uint32_t entry_point; /* resolved: the centroid fallback already applied */
    int32_t metric;
    int32_t device;
} fg_layout;

/* Per-query counters written by fg_search_device_ex (all optional). */
typedef struct fg_query_stats {
    uint32_t iterations;  /* loop iterations that merged candidates into the beam */
    uint32_t expansions;  /* parents expanded (neighbour lists read) */
    uint32_t evaluations; /* exact distances computed, entry point included */
    uint32_t estimates;   /* RaBitQ estimates computed */
} fg_query_stats;

const char* fg_status_string(int status);
/* Message of the last failure on the calling thread ("" if none). */
const char* fg_last_error(void);

/* Replaces QuantizationGraph::QuantizationGraph(n, dim, degree, path)
 * (include/qg.hpp:17-42) together with the index upload of
 * QuantizationGraph::gpu_search_adaptive (gpu_search_adaptive.cu:46-77):
 * reads the qg_codebook file, resolves entry point UINT32_MAX to the node
 * nearest the centroid (include/common.hpp:26-47), checks free memory and
 * keeps the codebook resident on `device` (FG_DEVICE_CURRENT: the current
 * device) until fg_index_free. */
int fg_index_load(const char* path, uint64_t num_nodes, uint64_t dim, int32_t degree, int32_t metric,
                  int32_t device, fg_index** out);

/* Same, from a codebook already in host memory: rows[num_nodes*row_offset]
 * and signs[padded_dim] in the qg_codebook layout. */
int fg_index_create(const float* rows, const float* signs, uint32_t entry_point, uint64_t num_nodes,
                    uint64_t dim, int32_t degree, int32_t metric, int32_t device, fg_index** out);

/* Same, from a codebook already in device memory on `device` (d_rows,
 * d_signs: device pointers, copied device to device; the caller keeps or
 * frees its buffers) -- for indexes built on the GPU, such as the shards of
 * a base too large for one host.  entry_point must be a node id (the
 * UINT32_MAX centroid fallback needs the rows on the host). */
int fg_index_create_device(const float* d_rows, const float* d_signs, uint32_t entry_point, uint64_t num_nodes,
                           uint64_t dim, int32_t degree, int32_t metric, int32_t device, fg_index** out);

/* Replaces ~QuantizationGraph (include/qg.hpp:44-47). NULL is accepted. */
int fg_index_free(fg_index* index);

/* Replaces the layout getters (include/qg.hpp:49-60). */
int fg_index_layout(const fg_index* index, fg_layout* out);

/* Replaces QuantizationGraph::set_metric (include/qg.hpp:54). */
int fg_index_set_metric(fg_index* index, int32_t metric);

/* What the kernel planner aims for (fg_index_set_plan_goal). */
#define FG_GOAL_LATENCY 0
#define FG_GOAL_THROUGHPUT 1

/* Sets what the planner optimises an index's searches for; no counterpart in
 * the reference (one kernel shape for every batch).  Every kernel returns the
 * same results, only their speed differs.
 * FG_GOAL_LATENCY (the default): the shortest time for one batch on an
 * otherwise idle GPU -- the CTA kernel for batches of up to 4 queries per SM,
 * the warp kernel's pair mode while the whole batch is resident at once, one
 * warp per query above.
 * FG_GOAL_THROUGHPUT: the most queries per second when the caller keeps
 * batches in flight on two or more streams (fg_search_async, or
 * fg_search_device on several streams), so that each batch shares the GPU
 * with the next: the pair mode while two batches of this size are resident at
 * once, one warp per query above.  FG_KERNEL=cta|pair|warp|staged in the
 * environment overrides either goal. */
int fg_index_set_plan_goal(fg_index* index, int32_t goal);

/* Kernel codes of fg_search_plan. */
#define FG_PLAN_CTA 0    /* one CTA per query */
#define FG_PLAN_WARP 1   /* one warp per query */
#define FG_PLAN_STAGED 2 /* one warp per query, parent blocks staged in shared memory */
#define FG_PLAN_PAIR 3   /* two warps per query */

/* The kernel the planner picks for a batch of nq queries at (K, beam) under
 * the index's goal, and how many queries it holds resident on the device at
 * once (kernel and resident_queries may be NULL).  No counterpart in the
 * reference; launches nothing. */
int fg_search_plan(fg_index* index, int32_t nq, int32_t K, int32_t beam, int32_t* kernel, int32_t* resident_queries);

/* Replaces QuantizationGraph::gpu_search_adaptive(nq, queries, K, result_idx,
 * beam_sz, elapsed) (gpu_search_adaptive.cu:12-114): host buffers in and out,
 * synchronous.  queries[nq*dim] row-major fp32, result_idx[nq*K].
 * elapsed_s (optional) = wall time of the search launch and its
 * synchronisation, excluding the copies, as the reference measures it
 * (gpu_search_adaptive.cu:98-107).  Supported: 1 <= K, 1 <= beam <= 1024,
 * degree <= 32, dim <= 4096. */
int fg_search(fg_index* index, int32_t nq, const float* queries, int32_t K, uint32_t* result_idx, int32_t beam,
              double* elapsed_s);

/* Replicated index on several devices from one host thread: `indexes` holds
 * `count` handles of the same codebook, each loaded on its own device
 * (fg_index_load with device = 0, 1, ...).  The batch is split into
 * contiguous, balanced slices in handle order; every device's copies and
 * launch are issued before any is awaited, so the devices search concurrently;
 * result_idx[nq*K] (and result_dist[nq*K], optional) are gathered in query
 * order.  elapsed_s (optional) = wall time from the first launch to the last
 * device's completion, excluding the copies.  Same arguments and errors as
 * fg_search otherwise; no counterpart in the reference (its search uses the
 * current device only, gpu_search_adaptive.cu:30-34). */
int fg_search_multi(fg_index* const* indexes, int32_t count, int32_t nq, const float* queries, int32_t K,
                    uint32_t* result_idx, float* result_dist, int32_t beam, double* elapsed_s);

/* Number of buffer slots of fg_search_async per index. */
#define FG_ASYNC_SLOTS 4

/* Streamed variant of fg_search for pipelines of query batches (the
 * reference re-uploads its index and synchronises on every call,
 * gpu_search_adaptive.cu:65-113): enqueues on `stream` the upload of
 * queries[nq*dim], the search and the download of the ids into
 * result_idx[nq*K], and returns without waiting.  `slot` (0 ..
 * FG_ASYNC_SLOTS-1) names the index's device buffers the batch uses, so
 * batches in different slots may be in flight at once -- one slot per stream
 * lets batch i+1's upload overlap batch i's search.  Host buffers should be
 * pinned (cudaHostAlloc) for the copies to run asynchronously.  The caller
 * synchronises the stream before reading result_idx and before reusing the
 * slot or the host buffers.  The first use of a slot, or a larger batch than
 * it has held, allocates its buffers. */
int fg_search_async(fg_index* index, int32_t slot, int32_t nq, const float* queries, int32_t K, uint32_t* result_idx,
                    int32_t beam, void* stream);

/* Size of the fixed device scratch used by fg_search_noalloc (8 MiB). */
#define FG_NOALLOC_SCRATCH_BYTES 8388608

/* fg_search without any device allocation; it has no counterpart in the
 * reference.  Same arguments, results and errors as fg_search, but the
 * queries, the result ids and the kernel's work counter are staged in a fixed
 * FG_NOALLOC_SCRATCH_BYTES array of device memory that is part of the
 * library, where fg_search grows buffers with cudaMalloc on demand (and the
 * reference allocates and frees them on every call).  It is for callers that
 * must not allocate during a search: a serving loop that must not stall its
 * other streams on the device-wide synchronisation cudaFree implies, or a
 * process whose device memory is entirely owned by another allocator.
 * Limit: 256 + round_up(nq*dim*4, 256) + nq*K*4 <= FG_NOALLOC_SCRATCH_BYTES
 * (e.g. 14,000 queries of dim 128 with K = 10); a larger batch returns
 * FG_ERR_ARG with a message -- split it or call fg_search.
 * Like fg_search the call is synchronous: it waits for the query upload, the
 * search and the download of the ids before it returns.
 * The first call on each device looks up the scratch's address on that
 * device; make that first call before any stream capture.  All calls on a
 * device share the one scratch array: calls that overlap in time (from
 * several threads, or on several indexes of one device) race on it and must
 * be serialised by the caller. */
int fg_search_noalloc(fg_index* index, int32_t nq, const float* queries, int32_t K, uint32_t* result_idx,
                      int32_t beam, double* elapsed_s);

/* Device-resident variant: d_queries / d_result_idx / d_result_dist (optional)
 * are device pointers on the index's device; the call is asynchronous on
 * `stream` (a cudaStream_t, NULL = default stream).  Searches on different
 * streams may run at the same time (each stream gets its own work counter,
 * allocated on its first search; at most 64 streams per index). */
int fg_search_device(fg_index* index, int32_t nq, const float* d_queries, int32_t K, uint32_t* d_result_idx,
                     float* d_result_dist, int32_t beam, void* stream);

/* Extended device variant: optional per-query counters d_stats[nq] and an
 * optional traversal trace d_trace[nq*trace_cap*8] (expander node ids per
 * iteration, 0xFFFFFFFF when unused) with d_trace_count[nq*trace_cap]. */
int fg_search_device_ex(fg_index* index, int32_t nq, const float* d_queries, int32_t K, uint32_t* d_result_idx,
                        float* d_result_dist, int32_t beam, void* stream, fg_query_stats* d_stats,
                        uint32_t* d_trace, int32_t* d_trace_count, int32_t trace_cap);

/* Query-side rotation and quantisation (include/utils.cuh:790-939) as a
 * standalone kernel: per query the rotated vector d_rotated[nq*D], the 6-bit
 * codes d_quant[nq*D], the 16-entry nibble LUT d_lut[nq*4*D] and
 * d_factors[nq*3] = (low, high, width), d_sum_q[nq].  Any output may be NULL
 * except d_factors. */
int fg_query_prepare_device(const float* d_queries, int32_t nq, int32_t dim, const float* d_signs,
                            float* d_rotated, uint8_t* d_quant, uint8_t* d_lut, float* d_factors,
                            int32_t* d_sum_q, void* stream);

/* Beam merge primitive on device, for verification (include/utils.cuh:1369-1399):
 * ncase independent cases, each [itopk beam entries | cbs candidates] in
 * d_idx/d_dist, merged in place with the reference's tie order. */
int fg_beam_merge_device(uint32_t* d_idx, float* d_dist, int32_t ncase, int32_t itopk, int32_t cbs, int32_t first,
                         void* stream);

/* Global top-K of a sharded index (the base split into
 * `shards` parts, each with its own graph): d_ids / d_dists hold, shard-major,
 * every shard's ascending top-k of the same nq queries ([shards][nq][k],
 * local ids as fg_search_device returns them, e.g. after an all-gather);
 * shard_offsets (host, `shards` entries, NULL = all 0) is the global id of
 * each shard's node 0.  Writes d_out_ids[nq*K] (global ids) and optionally
 * d_out_dists[nq*K]: the lists' stable merge by (distance, shard, position).
 * Asynchronous on `stream`.  Needs shards*k >= K and shards <= 64.  No
 * counterpart in the reference, whose index is one graph on one device
 * (gpu_search_adaptive.cu:65-72). */
int fg_shard_merge_device(const uint32_t* d_ids, const float* d_dists, const uint32_t* shard_offsets, int32_t shards,
                          int32_t nq, int32_t k, int32_t K, uint32_t* d_out_ids, float* d_out_dists, void* stream);

/* ---- host helpers of the reference CLI ---- */

/* include/utils.cuh:119-127 */
uint32_t fg_effective_sort_beam_size(uint32_t beam);

/* include/common.hpp:26-47: the entry point a codebook gets when its header
 * holds UINT32_MAX -- the node whose raw vector (the first dim floats of each
 * row of row_floats floats) is nearest the centroid of all raw vectors (largest
 * inner product for FG_METRIC_IP), the first such node on ties.  fg_index_load
 * and fg_index_create apply it.  Returns UINT32_MAX for invalid arguments
 * (NULL rows, num_nodes or dim 0, row_floats < dim). */
uint32_t fg_entry_point_centroid(const float* rows, uint64_t num_nodes, uint64_t dim, uint64_t row_floats,
                                 int32_t metric);

/* include/common.hpp:49-66: recall of predicted[nq*topk] against
 * groundtruth[nq*gt_k]; duplicates in a prediction row are all counted. */
float fg_compute_recall(const uint32_t* predicted, const int32_t* groundtruth, uint64_t nq, int32_t topk,
                        int32_t gt_k);

/* include/common.hpp:68-94: append TopK,Beam_size,Runtime,Latency,Throughput,Recall. */
int fg_append_run_stats_csv(const char* path, int32_t k, int32_t beam, double runtime, double latency,
                            double throughput, double recall);

/* include/metric.hpp:13-28: FG_METRIC_IP iff the path contains "text2image1m". */
int32_t fg_infer_metric_from_path(const char* path);

/* include/data_io.hpp:18-77: count and dim of an fvecs/ivecs file
 * (count = file_size / (4 + 4*dim)), then read it into dst[count*dim]. */
int fg_vecs_info(const char* path, uint64_t* count, int32_t* dim);
int fg_vecs_read(const char* path, void* dst, uint64_t count, int32_t dim);

#ifdef __cplusplus
}
#endif
#endif
