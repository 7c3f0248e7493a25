// fg_internal.h -- launch interface between the C ABI (fg_api.cu) and the
// kernels (fg_search.cu, fg_search_warp.cu).  Not installed; the public surface is
// include/flashgann.h.
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

#include "../../include/flashgann.h"

namespace fg {

// Everything a search launch needs; sizes in float words like the codebook.
struct SearchArgs {
    const float* rows = nullptr;      // device, n * row floats
    const float* signs = nullptr;     // device, padded_dim floats
    const float* queries = nullptr;   // device, nq * dim
    uint32_t* out_ids = nullptr;      // device, nq * K
    float* out_dists = nullptr;       // device, nq * K (optional)
    fg_query_stats* stats = nullptr;  // device, nq (optional)
    uint32_t* trace = nullptr;        // device, nq * trace_cap * SEARCH_WIDTH (optional)
    int32_t* trace_count = nullptr;   // device, nq * trace_cap (optional)
    int trace_cap = 0;
    uint32_t* work_counter = nullptr; // device scratch, one uint32 (zeroed by the launcher)
    uint64_t n = 0, row = 0, code_off = 0, factor_off = 0, nbr_off = 0;
    int dim = 0, padded_dim = 0, degree = 0;
    uint32_t entry = 0;
    int use_ip = 0;
    int nq = 0, K = 0, beam = 0;
    int goal = 0;  // FG_GOAL_LATENCY or FG_GOAL_THROUGHPUT: what plan_search optimises for
};

// Derived per-launch constants, computed on the host (plan_search).
struct SearchPlan {
    uint32_t padded = 0;       // effective sort beam (include/utils.cuh:119-127)
    uint32_t cbs = 0;          // candidate buffer size (adaptive_search_utils.cuh:231-236)
    uint32_t collect_cap = 0;  // min(BUFFER_BOUND, cbs)
    int hbits = 0;             // visited table bits
    float phase2_rho = 0.0f;   // adaptive_search_utils.cuh:20-23
    int max_iter = 0;          // gpu_search_adaptive.cu:96
    int merge_n2 = 0;          // 1/2/4: register bitonic merge, 0: merge path
    int mp_active = 0;         // merge-path output segments
    int vec_codes = 0;         // codes 16-byte aligned: 128-bit code loads
    int variant = 0;           // CTA kernel variant (warps per query, register budget)
    int kernel = 0;            // 0: one CTA per query (fg_search.cu), 1: one warp per query (fg_search_warp.cu)
    uint32_t slots = 0;        // warp kernel: visited-set slots
    size_t slice_bytes = 0;    // warp kernel: shared memory per query
    int min_ctas = 0;          // warp kernel: CTAs per SM its register budget is compiled for
    uint32_t blk = 0;          // warp kernel, staged variant: bytes of one parent block (0: not staged)
    int warp_mode = 0;         // warp kernel: 0 one warp per query, 1 staged, 2 a pair of warps per query
    int resident_queries = 0;  // warp kernel: queries resident at once on the device
    size_t smem_bytes = 0;
    int grid = 0;
    int threads = 0;
    int blocks_per_sm = 0;
};

int plan_search(const SearchArgs& a, SearchPlan* plan, int device, char* err, size_t errlen);
cudaError_t launch_search(const SearchArgs& a, const SearchPlan& plan, cudaStream_t stream);

// The warp-per-query kernel (fg_search_warp.cu): padded dimensions 32..256.
bool warp_kernel_supports(int padded_dim);
// mode: 0 one warp per query, 1 its staged variant, 2 a pair of warps per query
int plan_search_warp(const SearchArgs& a, SearchPlan* plan, int device, char* err, size_t errlen, int mode);
cudaError_t launch_search_warp(const SearchArgs& a, const SearchPlan& plan, cudaStream_t stream);

cudaError_t launch_query_prepare(const float* queries, int nq, int dim, const float* signs, float* rotated,
                                 uint8_t* quant, uint8_t* lut, float* factors, int32_t* sum_q,
                                 cudaStream_t stream);

cudaError_t launch_beam_merge(uint32_t* idx, float* dist, int ncase, int itopk, int cbs, int first,
                              cudaStream_t stream);

// Per-query merge of a sharded index's top-k lists (fg_shard_merge.cu).
int shard_merge_max_shards();
cudaError_t launch_shard_merge(const uint32_t* ids, const float* dists, const uint32_t* offsets, int shards, int nq,
                               int k, int K, uint32_t* out_ids, float* out_dists, cudaStream_t stream);

// Host restatements shared with the CLI and the API.
uint32_t effective_sort_beam(uint32_t beam);
uint32_t candidate_buffer_size(int degree);
int hash_bits(uint32_t padded, uint32_t cbs);

}  // namespace fg
