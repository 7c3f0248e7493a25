/*
 * fg_oracle.h -- CPU restatement of FlashGANN's adaptive quantised beam search.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA search
 * path in flashgann_b200/csrc and the CPU baseline timed by bench.py.  Only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs
 * may load it.  The product never links or calls it.
 *
 * Every function restates one piece of the reference search
 * (SophiaSun18/FlashGANN); the file:line it follows is cited beside it in
 * fg_oracle.c.  Parity pins: tests/golden/ holds vectors produced by the
 * reference's own sm_100a build (oracle/ref_harness.cu, run on a B200) and
 * tests/test_oracle_golden.py checks this restatement against them.
 */
#ifndef FG_ORACLE_H
#define FG_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Compile-time knobs of the reference (src/adaptive_search_config.cuh:3-73,
 * include/utils.cuh:21-34,683), carried at run time so tests can vary them.
 * og_default_knobs() returns the reference defaults. */
typedef struct og_knobs {
    int block_size;        /* BLOCK_SIZE = 256: merge-path segment cap, WARPS_PER_BLOCK = block_size/32 */
    int search_width;      /* SEARCH_WIDTH = WARPS_PER_BLOCK */
    int theta_min;         /* THETA_MIN = 1 */
    int theta_max;         /* THETA_MAX = WARPS_PER_BLOCK */
    float rho_min;         /* RHO_MIN = 0 */
    float rho_max;         /* RHO_MAX = 0.99 */
    int min_phase2_keep;   /* MIN_PHASE2_KEEP = 4 */
    int check_interval;    /* CHECK_INTERVAL = 1 */
    int buffer_bound;      /* BUFFER_BOUND = 32 */
    int phase1_theta;      /* PHASE1_THETA = THETA_MIN */
    float phase1_rho;      /* PHASE1_RHO = 0.25 */
    int phase2_theta;      /* PHASE2_THETA = THETA_MAX */
    int stall_iters;       /* TOP1_WARMUP_STALL_ITERS = 4 */
    int max_iterations;    /* MAX_ITERATIONS = 1024 */
    int reset_interval;    /* SMALL_HASH_RESET_INTERVAL = 16 */
    int hash_base_bitlen;  /* GPU_HASH_BASE_BITLEN = 11 */
} og_knobs;

void og_default_knobs(og_knobs* k);

/* Codebook layout in float words (include/qg.hpp:66-73). */
typedef struct og_layout {
    uint64_t dim, padded_dim, code_off, factor_off, nbr_off, row;
    int degree;
} og_layout;

void og_compute_layout(uint64_t dim, int degree, og_layout* out);

/* A resident codebook (host memory, caller-owned). */
typedef struct og_index {
    og_layout L;
    uint64_t n;
    const float* data;     /* n * L.row floats */
    const float* signs;    /* L.padded_dim floats */
    uint32_t entry_point;  /* already resolved (not UINT32_MAX) */
    int use_ip;
} og_index;

/* Query factors (include/utils.cuh:57-65, 840-939). */
typedef struct og_qfactors {
    float low, high, width;
    int32_t sum_q;
} og_qfactors;

/* rotated[D], quant[D] (uint8 codes) and lut[4D] are caller-allocated. */
void og_query_prepare(const float* query, const float* signs, int dim, int padded_dim,
                      float* rotated, uint8_t* quant, uint8_t* lut, og_qfactors* qf);

/* Per-query counters (device-side equivalents are produced by the CUDA path). */
typedef struct og_stats {
    uint64_t iterations;    /* loop iterations that reached the merge */
    uint64_t expansions;    /* parents expanded */
    uint64_t evaluations;   /* exact distances computed (entry point included) */
    uint64_t estimates;     /* RaBitQ estimates computed */
    uint64_t phase2_iter;   /* iteration at which phase 2 began (0 = never) */
} og_stats;

/* Optional traversal trace: for each iteration t < trace_cap the expander
 * node ids (up to search_width) are written at trace[t*search_width + j] and
 * their count at trace_count[t].  Unused entries are 0xFFFFFFFF. */
typedef struct og_trace {
    uint32_t* trace;
    int32_t* trace_count;
    int trace_cap;
    int n_iters;            /* out: iterations recorded */
} og_trace;

/* Status codes shared with the product's C ABI. */
#define OG_OK 0
#define OG_ERR_ARG 3

/* Search one query.  out_ids[K], out_dists_opt[K] (may be NULL). */
int og_search_one(const og_index* idx, const og_knobs* kn, const float* query, int K, int beam,
                  uint32_t* out_ids, float* out_dists_opt, og_stats* stats, og_trace* trace);

/* Search nq queries with `threads` OpenMP threads (<=0: all).  out_ids[nq*K]. */
int og_search_batch(const og_index* idx, const og_knobs* kn, int nq, const float* queries,
                    int K, int beam, uint32_t* out_ids, int threads, og_stats* total_stats);

/* ---- primitives exposed for unit tests against golden vectors ---- */

/* include/utils.cuh:683-750: reference hash (same function, linear probe). */
uint32_t og_hash_bitlen(uint32_t padded_beam, uint32_t cand_buf, uint32_t reset_interval,
                        uint32_t base_bitlen);

/* Beam merge: idx/dist hold [itopk beam | cbs candidates]; merged in place. */
int og_beam_merge(uint32_t* idx, float* dist, uint32_t cbs, uint32_t itopk, int first,
                  int block_size);

/* 32-entry candidate bitonic sort (include/utils.cuh:417-457, N_1 = 1). */
void og_candidate_sort(uint32_t* idx, float* dist, uint32_t cbs);

/* RaBitQ estimate of one neighbour (include/utils.cuh:941-1027).
 * zero_on_invalid selects the theta=1 variant that returns 0.0 when
 * triple_x == FLT_MAX (the speculative variant returns FLT_MAX). */
float og_estimate(const uint8_t* lut, const og_qfactors* qf, const uint8_t* codes, int neighbor,
                  int padded_dim, float triple_x, float f_dq, float f_vq, float parent_dist,
                  int zero_on_invalid);

/* Warp-order exact distance (include/utils.cuh:270-305). */
float og_warp_distance(int dim, const float* a, const float* b, int use_ip);

/* One adaptive rho update (phase 1) and the keep count that follows
 * (src/adaptive_search_utils.cuh:121-135,177-205). */
void og_rho_update(float rho_prev, int policy_iters, float rate, float phase2_rho, uint32_t active, int cut_valid,
                   uint32_t near, const og_knobs* kn, float* rho_out, int* keep_out);

/* Sizes (include/utils.cuh:119-127, src/adaptive_search_utils.cuh:231-236). */
uint32_t og_effective_sort_beam(uint32_t beam);
uint32_t og_candidate_buffer_size(int degree, const og_knobs* kn);

/* Host helpers restating include/common.hpp:26-66. */
uint32_t og_entry_point_centroid(const float* data, uint64_t n, uint64_t dim, uint64_t row, int use_ip);
float og_compute_recall(const uint32_t* predicted, const int32_t* gt, uint64_t nq, int topk,
                        int gt_k);

#ifdef __cplusplus
}
#endif
#endif
