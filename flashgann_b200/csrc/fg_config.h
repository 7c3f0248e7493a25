// fg_config.h -- build knobs of the search, with the reference's names and
// defaults (src/adaptive_search_config.cuh:3-73, include/utils.cuh:21-34,683).
//
// The knobs that define WHAT the search computes keep the reference's meaning:
// BLOCK_SIZE is the reference's CTA width and only fixes its derived semantic
// values (THETA_MAX, SEARCH_WIDTH and the merge-path segment count); the
// threads this build launches per query are the planner's choice (one warp
// per query, or a CTA of warps per query for small batches and dims > 256).
// INTERNAL_TOPK is accepted and reported; as in the reference it does not
// change results (the beam buffer is sized from the beam argument).
#pragma once

#ifndef INTERNAL_TOPK
#define INTERNAL_TOPK 128
#endif

#ifndef BLOCK_SIZE
#define BLOCK_SIZE 256
#endif
#define FG_REF_WARPS_PER_BLOCK (BLOCK_SIZE / 32)

#ifndef SEARCH_WIDTH
#define SEARCH_WIDTH (FG_REF_WARPS_PER_BLOCK)
#endif
#ifndef MAX_ITERATIONS
#define MAX_ITERATIONS (1 << 10)
#endif
#ifndef THETA_MIN
#define THETA_MIN 1
#endif
#ifndef THETA_MAX
#define THETA_MAX FG_REF_WARPS_PER_BLOCK
#endif
#ifndef RHO_MIN
#define RHO_MIN 0.0f
#endif
#ifndef RHO_MAX
#define RHO_MAX 0.99f
#endif
#ifndef MIN_PHASE2_KEEP
#define MIN_PHASE2_KEEP 4
#endif
#ifndef CHECK_INTERVAL
#define CHECK_INTERVAL 1
#endif
#ifndef BUFFER_BOUND
#define BUFFER_BOUND 32
#endif
#ifndef PHASE1_THETA
#define PHASE1_THETA THETA_MIN
#endif
#ifndef PHASE1_RHO
#define PHASE1_RHO 0.25f
#endif
#ifndef PHASE2_THETA
#define PHASE2_THETA THETA_MAX
#endif
#ifndef TOP1_WARMUP_STALL_ITERS
#define TOP1_WARMUP_STALL_ITERS 4
#endif
#ifndef SMALL_HASH_RESET_INTERVAL
#define SMALL_HASH_RESET_INTERVAL 16
#endif
// The reference's visited table has at least 2^11 slots; any exact set gives
// the same search, so this build sizes its table by the same load rule from
// a smaller floor.
#ifndef FG_HASH_BASE_BITLEN
#define FG_HASH_BASE_BITLEN 10
#endif

#define FG_QG_BQUERY 6           // include/common.hpp:17
#define FG_MAX_BEAM 1024
#define FG_MAX_DEGREE 32
#define FG_MAX_DIM 4096

static_assert(SEARCH_WIDTH >= 1 && SEARCH_WIDTH <= 32, "SEARCH_WIDTH must be in [1, 32]");
static_assert(THETA_MIN >= 1, "THETA_MIN must be >= 1");
static_assert(BUFFER_BOUND > 0 && BUFFER_BOUND <= 32, "BUFFER_BOUND must be in [1, 32]");
static_assert(THETA_MAX >= THETA_MIN, "THETA_MAX must be >= THETA_MIN");
static_assert(THETA_MAX <= SEARCH_WIDTH, "THETA_MAX must not exceed SEARCH_WIDTH");
static_assert(CHECK_INTERVAL >= 1, "CHECK_INTERVAL must be >= 1");
static_assert(RHO_MIN >= 0.0f && RHO_MIN < 1.0f, "RHO_MIN must be in [0, 1)");
static_assert(RHO_MAX >= RHO_MIN && RHO_MAX < 1.0f, "RHO_MAX must be in [RHO_MIN, 1)");
static_assert(TOP1_WARMUP_STALL_ITERS >= 1, "TOP1_WARMUP_STALL_ITERS must be >= 1");
static_assert(PHASE1_THETA >= THETA_MIN && PHASE1_THETA <= THETA_MAX, "PHASE1_THETA out of bounds");
static_assert(PHASE2_THETA >= THETA_MIN && PHASE2_THETA <= THETA_MAX, "PHASE2_THETA out of bounds");
static_assert(PHASE1_RHO >= RHO_MIN && PHASE1_RHO <= RHO_MAX, "PHASE1_RHO out of bounds");
static_assert(MIN_PHASE2_KEEP > 0, "MIN_PHASE2_KEEP must be > 0");
