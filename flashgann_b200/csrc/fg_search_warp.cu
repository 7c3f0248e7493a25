// fg_search_warp.cu -- the search with one warp per query.
//
// Same search as fg_search.cu (the reference's QuantizedPrunedBeamSearch,
// SophiaSun18/FlashGANN src/adaptive_search.cuh:5-466, bit for bit), laid out
// for throughput instead of per-query latency: each warp of a CTA is an
// independent worker that pulls query ids from the global counter and runs
// the whole iteration on its own, with no block barrier anywhere.  A CTA
// holds 1, 2 or 4 queries (the planner picks the shape with the most resident
// queries per SM); the per-warp state (beam, visited set, bit planes,
// candidate buffer) is a private slice of shared memory.
//
// Per iteration the warp
//   * merges the pending candidates into the beam in place: candidate m lands
//     at pos[m] = m + #{beam <= cand[m]} (the stable, beam-first merge), and
//     the beam tail is shifted chunk by chunk from the end.  The reference's
//     merge path differs from the stable merge only where a beam entry and a
//     candidate have equal distances at one of its segment boundaries: the
//     segments next to such a boundary are replayed with the reference's
//     splits before the shift and written over it (a full replay covers more
//     than the fix-up list holds);
//   * picks the expanders and runs the adaptive controller (warp-uniform
//     registers);
//   * expands one parent per step, lane l holding neighbour l, while the next
//     parent's block loads: visited lookups (all before any insert of the
//     iteration), bit-plane RaBitQ estimates and the keep rule;
//   * compacts the kept children (first parent wins a shared child) with
//     __match_any_sync, inserts them into the visited set and computes their
//     exact distances G rows at a time: every lane accumulates its strided
//     dimensions of each row in the reference's order, then the reference's
//     shuffle tree runs transposed (lanes split the rows), which gives the
//     same sums with G-1+log2(32/G) shuffles instead of 5 per row.
// The visited set is exact and two-choice (see w_insert), which keeps it
// small enough for 5 CTAs of 4 queries per SM up to beam 640 at D = 128.
#include <cfloat>
#include <cstdint>
#include <cstdio>
#include <cstdlib>

#include <cuda_runtime.h>

#include "fg_config.h"
#include "fg_device.cuh"
#include "fg_internal.h"

static_assert(BUFFER_BOUND <= 32, "the warp kernel keeps at most 32 candidates per iteration");
static_assert(SEARCH_WIDTH <= 32, "expanders are picked by one warp");

namespace fg {
namespace {

constexpr int kWarpsPerCta = 4;  // largest CTA; the planner may launch 1 or 2 warps per CTA
// Register budgets: 4 CTAs per SM (128 registers per thread) or, when the
// query slices of 5 CTAs fit the SM's shared memory, 5 (96 registers).
constexpr int kCtasLarge = 4;
constexpr int kCtasSmall = 5;
// The staged variant (3 CTAs per SM, 168 registers): every parent block of a
// speculative iteration is copied into a shared-memory ring with cp.async at
// once, instead of one block ahead in registers, and exact distances run 16
// rows per round.  On a B200 it was no faster than the register pipeline at
// any batch size (a lone query's time is set by its chain of instructions,
// not by the parent loads) and slower at full batches (12 instead of 20
// resident queries per SM), so the planner never picks it; FG_KERNEL=staged
// selects it.
constexpr int kCtasStaged = 3;
// Kernel modes: one warp per query, the staged variant of it, or a pair of
// warps per query (the pair mode, for batches that fill few warp slots).
constexpr int kModeWarp = 0;
constexpr int kModeStaged = 1;
constexpr int kModePair = 2;
// The pair mode's register budget: 5 CTAs of 4 warps (10 queries) per SM.
constexpr int kCtasPair = 5;

struct WPlan {
    uint32_t padded, cbs, collect_cap;
    uint32_t slots;  // visited-set slots, a multiple of 32
    float phase2_rho;
    int max_iter;
    int mp_active;
    uint32_t slice;  // shared-memory bytes per warp
    uint32_t blk;    // staged variant: bytes of a parent block (codes, factors, ids), a multiple of 16
};

// One warp's slice of the CTA's dynamic shared memory.
struct WSlice {
    uint32_t* bidx;
    float* bdist;
    uint32_t* hash;
    uint32_t* planes;
    uint32_t* wrap;
    uint32_t* cidx;   // candidate buffer (32 entries)
    float* cdist;
    uint32_t* pos;    // merge path with ties: stable positions of the candidates
    uint32_t* stage;  // kept children in (parent, rank) order, or the evaluation list
    uint32_t* eslot;  // single-expander path: candidate slot of each evaluation
    uint32_t* pnode;  // expanders of the iteration
    float* pdist;
    unsigned char* ring;  // staged variant: SEARCH_WIDTH parent blocks
    // stage and eslot (256 contiguous bytes) double as the merge's tie fix-up
    // list, and stage as the query factors during set-up
    QueryState* qs;
};

__host__ __device__ inline size_t a16(size_t x) { return (x + 15) & ~static_cast<size_t>(15); }

__host__ __device__ inline size_t slice_layout(uint32_t padded, uint32_t slots, int D, bool mp, WSlice* s,
                                               unsigned char* base, size_t ring_bytes = 0) {
    size_t off = 0;
    auto take = [&](size_t bytes) {
        unsigned char* p = base ? base + off : nullptr;
        off += a16(bytes);
        return p;
    };
    const int W = D / 32;
    unsigned char* p;
    p = take(static_cast<size_t>(slots) * 4); if (s) s->hash = reinterpret_cast<uint32_t*>(p);
    p = take(padded * 4); if (s) s->bidx = reinterpret_cast<uint32_t*>(p);
    p = take(padded * 4); if (s) s->bdist = reinterpret_cast<float*>(p);
    p = take(static_cast<size_t>(kPlanes) * W * 4); if (s) s->planes = reinterpret_cast<uint32_t*>(p);
    p = take(static_cast<size_t>(W) * 4); if (s) s->wrap = reinterpret_cast<uint32_t*>(p);
    p = take(32 * 4); if (s) s->cidx = reinterpret_cast<uint32_t*>(p);
    p = take(32 * 4); if (s) s->cdist = reinterpret_cast<float*>(p);
    p = take(32 * 4); if (s) s->pos = reinterpret_cast<uint32_t*>(p);
    p = take(32 * 4); if (s) s->stage = reinterpret_cast<uint32_t*>(p);
    p = take(32 * 4); if (s) s->eslot = reinterpret_cast<uint32_t*>(p);
    p = take(SEARCH_WIDTH * 4); if (s) s->pnode = reinterpret_cast<uint32_t*>(p);
    p = take(SEARCH_WIDTH * 4); if (s) s->pdist = reinterpret_cast<float*>(p);
    p = ring_bytes ? take(ring_bytes) : nullptr; if (s) s->ring = p;
    if (s) s->qs = reinterpret_cast<QueryState*>(s->stage);
    (void)mp;
    return off;
}

// ---------------------------------------------------------------- visited set
// Exact set of node ids in buckets of 4 slots (one 128-bit shared load per
// bucket), two-choice: a key lives in the emptier of its two buckets, so a
// lookup reads both (independent loads) and a missing key is settled as soon
// as either has an empty slot.  Only when both are full does an insert walk on
// linearly from the second bucket; it first sets the overflow flag of that
// bucket (the MSB of its slot 0: node ids are < 2^31 - 1, so a flagged id
// never reads as the empty value).  A lookup with both buckets full walks the
// same way only if the flag is set -- nothing is removed between resets, so
// the walk meets the key before any empty slot, and with the flag clear no key
// of that bucket was placed elsewhere.  Two choices keep the walks rare at
// loads up to ~93 %; the flag spares the lookups of absent keys (most of the
// walks) that would otherwise have to reach an empty slot.
__device__ __forceinline__ void w_buckets(uint32_t key, uint32_t nb, uint32_t& b1, uint32_t& b2) {
    b1 = __umulhi(key * 0x9E3779B1u, nb);
    b2 = __umulhi((key ^ 0x5bd1e995u) * 0x85EBCA77u, nb);
    if (b2 == b1) b2 = b1 + 1 == nb ? 0 : b1 + 1;
}

__device__ __forceinline__ bool has_key(const uint4& v, uint32_t key) {
    return (v.x & ~kMsb) == key || v.y == key || v.z == key || v.w == key;
}

__device__ __forceinline__ int empties(const uint4& v) {
    return (v.x == kMax) + (v.y == kMax) + (v.z == kMax) + (v.w == kMax);
}

// the linear walk from bucket b + 1 (both of the key's buckets full)
__device__ __noinline__ bool w_walk_contains(const uint32_t* t, uint32_t nb, uint32_t key, uint32_t b) {
    for (uint32_t n = 1; n < nb; ++n) {
        b = b + 1 == nb ? 0 : b + 1;
        const uint4 v = *reinterpret_cast<const uint4*>(t + 4 * b);
        if (has_key(v, key)) return true;
        if (empties(v)) return false;
    }
    return false;
}

__device__ __noinline__ bool w_walk_insert(uint32_t* t, uint32_t nb, uint32_t key, uint32_t b) {
    for (uint32_t n = 1; n < nb; ++n) {
        b = b + 1 == nb ? 0 : b + 1;
        for (int j = 0; j < 4; ++j) {
            const uint32_t cur = t[4 * b + j];
            if ((j == 0 ? (cur & ~kMsb) : cur) == key) return false;
            if (cur == kMax) {
                const uint32_t old = atomicCAS(&t[4 * b + j], kMax, key);
                if (old == kMax) return true;
                if (old == key) return false;
            }
        }
    }
    return false;
}

// true if the key was not in the set (other lanes may insert concurrently)
__device__ __forceinline__ bool w_insert(uint32_t* t, uint32_t slots, uint32_t key) {
    const uint32_t nb = slots >> 2;
    uint32_t b1, b2;
    w_buckets(key, nb, b1, b2);
    for (uint32_t tries = 0; tries < slots; ++tries) {
        const uint4 v1 = *reinterpret_cast<const uint4*>(t + 4 * b1);
        const uint4 v2 = *reinterpret_cast<const uint4*>(t + 4 * b2);
        if (has_key(v1, key) || has_key(v2, key)) return false;
        const int e1 = empties(v1), e2 = empties(v2);
        if (e1 == 0 && e2 == 0) {
            atomicOr(&t[4 * b2], kMsb);  // overflow flag: slot 0 of a full bucket holds an id
            return w_walk_insert(t, nb, key, b2);
        }
        const uint32_t b = e1 >= e2 ? b1 : b2;
        const uint4 v = e1 >= e2 ? v1 : v2;
        const int j = v.x == kMax ? 0 : v.y == kMax ? 1 : v.z == kMax ? 2 : 3;
        const uint32_t old = atomicCAS(&t[4 * b + j], kMax, key);
        if (old == kMax) return true;
        if (old == key) return false;
        // another lane took the slot: look again
    }
    return false;
}

// LAST: test a bucket for an empty slot by its last slot alone -- inserts take
// the first empty slot and nothing is removed between resets, so a bucket
// with an empty slot has an empty last slot.  On a B200 that was 0.5 %
// faster in the one-warp search and 0.5 % slower in the pair mode, which
// keeps the count of empties.
template <bool LAST>
__device__ __forceinline__ bool w_contains(const uint32_t* t, uint32_t slots, uint32_t key) {
    const uint32_t nb = slots >> 2;
    uint32_t b1, b2;
    w_buckets(key, nb, b1, b2);
    const uint4 v1 = *reinterpret_cast<const uint4*>(t + 4 * b1);
    const uint4 v2 = *reinterpret_cast<const uint4*>(t + 4 * b2);
    if (has_key(v1, key) || has_key(v2, key)) return true;
    if constexpr (LAST) {
        if (v1.w == kMax || v2.w == kMax || !(v2.x & kMsb)) return false;
    } else {
        if (empties(v1) || empties(v2) || !(v2.x & kMsb)) return false;
    }
    return w_walk_contains(t, nb, key, b2);
}

__device__ __forceinline__ void w_clear(uint32_t* t, uint32_t slots, int lane) {
    const uint4 e = make_uint4(kMax, kMax, kMax, kMax);
    for (uint32_t i = static_cast<uint32_t>(lane) * 4; i < slots; i += 128) *reinterpret_cast<uint4*>(t + i) = e;
}

// ----------------------------------------------------------- parent blocks
// Read-only loads as volatile inline PTX: they stay where they are written, so
// the next parent's block is in flight while the current one is examined (a
// plain read-only load may legally be sunk to its first use).
__device__ __forceinline__ uint32_t ldg_pinned(const void* p) {
    uint32_t v;
    asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ uint4 ldg_pinned_v4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

// 16-byte global -> shared copies that complete asynchronously (cp.async,
// L2 only), grouped per parent; wait_groups(n) returns once at most n of the
// calling lane's groups are still in flight.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gmem) : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

__device__ __forceinline__ void cp_async_wait_groups(int n) {
    switch (n) {
        case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
        case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
        case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
        case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
        case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
        case 5: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
        case 6: asm volatile("cp.async.wait_group 6;" ::: "memory"); break;
        default: asm volatile("cp.async.wait_group 7;" ::: "memory"); break;
    }
}

// The staged block of parent t (codes | triple_x | f_dq | f_vq | ids, as in
// the codebook row) into lane `lane`'s ParentLane, from shared memory.
template <int W>
__device__ __forceinline__ void parent_from_ring(const unsigned char* blk, int deg, int D, int lane, ParentLane<W>& p) {
    const int cbytes = deg * (D / 8);
    const float* fac = reinterpret_cast<const float*>(blk + cbytes);
    p.child = kMax;
    p.tx = FLT_MAX;
    p.fdq = 0.0f;
    p.fvq = 0.0f;
#pragma unroll
    for (int w = 0; w < W; ++w) p.c[w] = 0;
    if (lane < deg) {
        p.child = reinterpret_cast<const uint32_t*>(fac + 3 * deg)[lane];
        p.tx = fac[lane];
        p.fdq = fac[deg + lane];
        p.fvq = fac[2 * deg + lane];
        const uint32_t* code = reinterpret_cast<const uint32_t*>(blk) + static_cast<size_t>(lane) * W;
        if constexpr (W % 4 == 0) {
#pragma unroll
            for (int w = 0; w < W; w += 4) {
                const uint4 x = *reinterpret_cast<const uint4*>(code + w);
                p.c[w] = x.x;
                p.c[w + 1] = x.y;
                p.c[w + 2] = x.z;
                p.c[w + 3] = x.w;
            }
        } else {
#pragma unroll
            for (int w = 0; w < W; ++w) p.c[w] = code[w];
        }
    }
}

// load_parent (fg_device.cuh) with pinned loads: neighbour id, the three
// factors and the packed code words of neighbour `lane` of the parent row.
template <int W>
__device__ __forceinline__ void load_parent_pinned(const float* __restrict__ prow, const SearchArgs& a, int limit,
                                                   bool vec, int lane, ParentLane<W>& p) {
    const uint32_t* ids = reinterpret_cast<const uint32_t*>(prow + a.nbr_off);
    const float* fac = prow + a.factor_off;
    if constexpr (W == 4) {
        if (limit >= 32 && vec) {
            // every lane holds a neighbour: no default values to set first
            // (0.3-0.9 % faster on a B200)
            p.child = ldg_pinned(ids + lane);
            p.tx = __uint_as_float(ldg_pinned(fac + lane));
            p.fdq = __uint_as_float(ldg_pinned(fac + a.degree + lane));
            p.fvq = __uint_as_float(ldg_pinned(fac + 2 * a.degree + lane));
            const uint4 x = ldg_pinned_v4(reinterpret_cast<const uint32_t*>(prow + a.code_off) + 4 * lane);
            p.c[0] = x.x;
            p.c[1] = x.y;
            p.c[2] = x.z;
            p.c[3] = x.w;
            return;
        }
    }
    p.child = kMax;
    p.tx = FLT_MAX;
    p.fdq = 0.0f;
    p.fvq = 0.0f;
#pragma unroll
    for (int w = 0; w < W; ++w) p.c[w] = 0;
    if (lane < limit) {
        p.child = ldg_pinned(ids + lane);
        p.tx = __uint_as_float(ldg_pinned(fac + lane));
        p.fdq = __uint_as_float(ldg_pinned(fac + a.degree + lane));
        p.fvq = __uint_as_float(ldg_pinned(fac + 2 * a.degree + lane));
        const uint32_t* code = reinterpret_cast<const uint32_t*>(prow + a.code_off) + static_cast<size_t>(lane) * W;
        if constexpr (W % 4 == 0) {
            if (vec) {
#pragma unroll
                for (int w = 0; w < W; w += 4) {
                    const uint4 x = ldg_pinned_v4(code + w);
                    p.c[w] = x.x;
                    p.c[w + 1] = x.y;
                    p.c[w + 2] = x.z;
                    p.c[w + 3] = x.w;
                }
                return;
            }
        }
#pragma unroll
        for (int w = 0; w < W; ++w) p.c[w] = ldg_pinned(code + w);
    }
}

// ------------------------------------------------------------ exact distances
// Distance of one row, query dimensions lane, lane+32, ... in registers:
// the reference's lane-strided fused accumulation and shfl_down tree
// (include/utils.cuh:270-305).
template <int W, bool IP>
__device__ __forceinline__ float dist_one(const float* __restrict__ r, const float (&q)[W], int dim, int lane) {
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < W; ++k) {
        const int d = lane + 32 * k;
        if (d < dim) {
            const float x = __ldg(r + d);
            if (IP) {
                acc = __fmaf_rn(q[k], x, acc);
            } else {
                const float df = __fsub_rn(q[k], x);
                acc = __fmaf_rn(df, df, acc);
            }
        }
    }
    const float s = tree_sum(acc);
    return IP ? -s : s;
}

// Exact distances of G rows nd[0..G) (the last rows of a short round repeat
// a valid row and are not written).  Lane l accumulates dimensions l, l+32,
// ... of every row (every load is issued before the first multiply-add; a
// dimension >= dim adds fma(0, 0, acc) = acc); then the reference's shuffle
// tree runs transposed: the level with offset o adds the partial of virtual
// lane v+o to that of v, and while a lane still holds several rows it keeps
// half of them and trades the other half with lane l^o.  Every sum is formed
// from the same two operands as in the reference's tree.
template <int W, int G, bool IP>
__device__ __forceinline__ void eval_round(const float* __restrict__ rows, uint64_t rowf, int dim, const float (&q)[W],
                                           const uint32_t (&nd)[G], int valid, float* out,
                                           const uint32_t* slot, int e0, int lane) {
    constexpr int LG = G == 32 ? 5 : G == 16 ? 4 : G == 8 ? 3 : G == 4 ? 2 : G == 2 ? 1 : 0;
    static_assert((1 << LG) == G, "G must be a power of two <= 32");
    float x[G][W];
#pragma unroll
    for (int r = 0; r < G; ++r) {
        const float* p = rows + static_cast<uint64_t>(nd[r]) * rowf + lane;
#pragma unroll
        for (int k = 0; k < W; ++k) x[r][k] = (lane + 32 * k < dim) ? __ldg(p + 32 * k) : 0.0f;
    }
    float acc[G];
#pragma unroll
    for (int r = 0; r < G; ++r) {
        acc[r] = 0.0f;
#pragma unroll
        for (int k = 0; k < W; ++k) {
            const float df = __fsub_rn(q[k], x[r][k]);
            acc[r] = IP ? __fmaf_rn(q[k], x[r][k], acc[r]) : __fmaf_rn(df, df, acc[r]);
        }
    }
#pragma unroll
    for (int lvl = 0; lvl < 5; ++lvl) {
        const int o = 16 >> lvl;
        const int nr = G >> lvl;
        if (nr > 1) {
            const bool up = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < nr / 2; ++i) {
                const float send = up ? acc[i] : acc[i + nr / 2];
                const float keep = up ? acc[i + nr / 2] : acc[i];
                acc[i] = __fadd_rn(keep, __shfl_xor_sync(kFull, send, o));
            }
        } else {
            acc[0] = __fadd_rn(acc[0], __shfl_xor_sync(kFull, acc[0], o));
        }
    }
    const int r = lane >> (5 - LG);
    if ((lane & ((1 << (5 - LG)) - 1)) == 0 && r < valid) {
        const int e = e0 + r;
        out[slot ? slot[e] : e] = IP ? -acc[0] : acc[0];
    }
}

// Exact distances of nodes[0..n) into out[slot ? slot[e] : e], GB rows per round
// (one round shape keeps the loop small for the instruction cache).
template <int W, int GB, bool IP>
__device__ __forceinline__ void eval_nodes(const float* __restrict__ rows, uint64_t rowf, int dim, const float (&q)[W],
                                           const uint32_t* nodes, int n, float* out, const uint32_t* slot,
                                           int lane, int first = 0, int stride = GB) {
    int e0 = first;
    for (; e0 < n; e0 += stride) {
        uint32_t nd[GB];
#pragma unroll
        for (int r = 0; r < GB; ++r) nd[r] = nodes[e0 + r < n ? e0 + r : n - 1];
        eval_round<W, GB, IP>(rows, rowf, dim, q, nd, n - e0, out, slot, e0, lane);
    }
}

// min(rho keep, BUFFER_BOUND / theta budget) of keep_for, before its cutoff clamp.
__device__ __forceinline__ int keep_cap(uint32_t active, int theta, float rho) {
    const int ac = static_cast<int>(active);
    const int rho_keep = static_cast<int>(keep_per_parent(active, rho));
    const int budget = clamp_i(static_cast<int>(c_bound[theta]), 1, ac);
    return rho_keep < budget ? rho_keep : budget;
}

// raw_sum (fg_device.cuh) reading the bit planes and the wrap mask with
// 128-bit shared loads (the slice keeps them 16-byte aligned; W % 4 == 0).
template <int W>
__device__ __forceinline__ uint32_t raw_sum_v(const uint32_t (&c)[W], const uint32_t* planes, const uint32_t* wrap,
                                              bool wrap_any) {
    static_assert(W % 4 == 0, "128-bit plane words");
    const uint4* pl = reinterpret_cast<const uint4*>(planes);
    uint32_t raw = 0;
#pragma unroll
    for (int p = 0; p < kPlanes; ++p) {
        uint32_t sum = 0;
#pragma unroll
        for (int w = 0; w < W; w += 4) {
            const uint4 v = pl[(p * W + w) / 4];
            sum += __popc(c[w] & v.x) + __popc(c[w + 1] & v.y) + __popc(c[w + 2] & v.z) + __popc(c[w + 3] & v.w);
        }
        raw += sum << p;
    }
    if (wrap_any) {
        const uint4* wr = reinterpret_cast<const uint4*>(wrap);
#pragma unroll
        for (int w = 0; w < W; w += 4) {
            const uint4 v = wr[w / 4];
            const uint32_t m[4] = {c[w] & v.x, c[w + 1] & v.y, c[w + 2] & v.z, c[w + 3] & v.w};
#pragma unroll
            for (int j = 0; j < 4; ++j)
                raw -= 256u * static_cast<uint32_t>(__popc(m[j] & (m[j] >> 1) & (m[j] >> 2) & (m[j] >> 3) & 0x11111111u));
        }
    }
    return raw;
}

// ------------------------------------------------------------ merge path
// Merge of the candidate buffer (cidx/cdist[0..cbs)) into the beam
// (bidx/bdist[0..P)) with the reference's merge-path result
// (include/utils.cuh:618-680): sorts the candidates with the 32-lane network
// and returns p0 = #{beam < cand[0]}, the first position that can change.
// Stable (beam-first) merge in place: output o >= p0 is candidate m if
// pos[m] == o, else beam[o - #{pos < o}].  Chunks of 32 positions are
// rewritten from the end, two per step (all reads of a step before its
// writes; every source index is <= its output, so lower chunks are intact).
// UNIFORM: chunks past the last landing candidate take the uniform shift
// first (output o = beam[o - m_in], no per-chunk candidate masks).  Fewer
// instructions, more code: on a B200 the pair mode (latency-bound, few warps
// per SM) ran 3.5 % faster with it, the one-warp search at full residency 7 %
// slower, so only the pair mode uses it.
template <bool UNIFORM>
__device__ __forceinline__ void stable_shift(uint32_t* bidx, float* bdist, float k, uint32_t v, uint32_t pos, uint32_t P,
                                             uint32_t p0, int lane) {
    const int first = static_cast<int>(p0 & ~31u);
    int top = static_cast<int>((P - 1) & ~31u);
    if constexpr (UNIFORM) {
        // the candidates that land (pos < P) are lanes 0 .. m_in - 1, positions increasing
        const int m_in = __popc(__ballot_sync(kFull, pos < P));
        if (m_in == 0) return;  // the merged beam is the beam
        const uint32_t pmax = __shfl_sync(kFull, pos, m_in - 1);
        const int ustop = static_cast<int>((pmax + 32u) & ~31u) > first ? static_cast<int>((pmax + 32u) & ~31u) : first;
        while (top >= ustop) {
            const bool two = top - 32 >= ustop;
            const uint32_t o0 = static_cast<uint32_t>(top) + lane, o1 = o0 - 32u;
            const bool a0 = o0 < P;
            float d0 = 0.0f, d1 = 0.0f;
            uint32_t i0 = 0, i1 = 0;
            if (a0) {
                d0 = bdist[o0 - m_in];
                i0 = bidx[o0 - m_in];
            }
            if (two) {
                d1 = bdist[o1 - m_in];
                i1 = bidx[o1 - m_in];
            }
            __syncwarp();
            if (a0) {
                bdist[o0] = d0;
                bidx[o0] = i0;
            }
            if (two) {
                bdist[o1] = d1;
                bidx[o1] = i1;
            }
            __syncwarp();
            top -= two ? 64 : 32;
        }
    }
    for (int g = top; g >= first; g -= 64) {
        float od[2];
        uint32_t ov[2];
        bool act[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int c0 = g - 32 * u;
            act[u] = false;
            od[u] = 0.0f;
            ov[u] = 0;
            if (c0 >= first) {
                const uint32_t uc0 = static_cast<uint32_t>(c0);
                const uint32_t below = __popc(__ballot_sync(kFull, pos < uc0));
                const uint32_t rel = pos - uc0;
                const uint32_t hit = __reduce_or_sync(kFull, (pos >= uc0 && rel < 32u) ? (1u << rel) : 0u);
                const uint32_t o = uc0 + lane;
                const uint32_t cnt = below + __popc(hit & lanemask_lt(lane));
                const float ck = __shfl_sync(kFull, k, cnt & 31u);
                const uint32_t cv = __shfl_sync(kFull, v, cnt & 31u);
                act[u] = o < P && o >= p0;
                if (act[u]) {
                    if ((hit >> lane) & 1u) {
                        od[u] = ck;
                        ov[u] = cv;
                    } else {
                        od[u] = bdist[o - cnt];
                        ov[u] = bidx[o - cnt];
                    }
                }
            }
        }
        __syncwarp();
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            if (act[u]) {
                const uint32_t o = static_cast<uint32_t>(g - 32 * u) + lane;
                bdist[o] = od[u];
                bidx[o] = ov[u];
            }
        }
        __syncwarp();
    }
}

// Fix-up list in the slice's stage and eslot bytes, which the merge does not
// otherwise use (more flagged segments than it holds take the full replay).
constexpr int kMaxFixSegments = 4;
constexpr int kFixBytes = 2 * 32 * 4;  // stage, eslot
struct FixArea {
    uint32_t* mask;  // segment flags, (BLOCK_SIZE + 32) / 32 words
    uint32_t* list;  // flagged segment ids
    uint32_t* idx;   // 4 * kMaxFixSegments outputs
    float* dist;
    uint16_t* at;    // output position, 0xFFFF = unused
};
__device__ __forceinline__ FixArea fix_area(unsigned char* b) {
    FixArea f;
    f.mask = reinterpret_cast<uint32_t*>(b);
    f.list = reinterpret_cast<uint32_t*>(b + 48);
    f.idx = reinterpret_cast<uint32_t*>(b + 64);
    f.dist = reinterpret_cast<float*>(b + 64 + 4 * 4 * kMaxFixSegments);
    f.at = reinterpret_cast<uint16_t*>(b + 64 + 8 * 4 * kMaxFixSegments);
    return f;
}
static_assert((BLOCK_SIZE + 32) / 32 <= 12 && kMaxFixSegments <= 4, "flags fit in 48 bytes, ids in 16");
static_assert(64 + 10 * 4 * kMaxFixSegments <= kFixBytes, "fix-ups fit in stage and eslot");

__device__ __noinline__ int tie_fixups(uint32_t* s_bidx, float* s_bdist, uint32_t* s_cidx, float* s_cdist,
                                       uint32_t* s_pos, unsigned char* s_fix, uint32_t cbs, uint32_t P, int active,
                                       const uint16_t* bnd, uint32_t p0, uint32_t lb, uint32_t ub, bool tie, int lane);
__device__ __noinline__ void merge_path_ties(uint32_t* s_bidx, float* s_bdist, uint32_t* s_cidx, float* s_cdist,
                                             uint32_t* s_pos, uint32_t cbs, uint32_t P, int active, const uint16_t* bnd,
                                             uint32_t p0, int lane);

// Merge of the candidate buffer (cidx/cdist[0..cbs)) into the beam
// (bidx/bdist[0..P)) with the reference's merge-path result
// (include/utils.cuh:618-680): sorts the candidates with the 32-lane network
// and returns p0 = #{beam < cand[0]}, the first position that can change.
// The merge path equals the stable merge except at a segment boundary where a
// beam entry and a candidate tie: those segments are replayed with the
// reference's splits before the stable shift and written over it.
template <bool UNIFORM>
__device__ __forceinline__ uint32_t merge_path_warp(const WSlice& s, uint32_t cbs, uint32_t P, int active, const uint16_t* bnd,
                                    int lane) {
    uint32_t* bidx = s.bidx;
    float* bdist = s.bdist;
    const bool valid = lane < static_cast<int>(cbs);
    float k = valid ? s.cdist[lane] : FLT_MAX;
    uint32_t v = valid ? s.cidx[lane] : kMax;
    sort32(k, v, lane);
    __syncwarp();
    if (valid) {
        s.cdist[lane] = k;
        s.cidx[lane] = v;
    }
    const uint32_t lb = lower_bound(bdist, P, k);
    uint32_t ub = lb;
    if (k == FLT_MAX) ub = P;
    else if (lb < P && bdist[lb] == k) ub = upper_bound(bdist, P, k);
    const uint32_t pos = valid ? static_cast<uint32_t>(lane) + ub : kMax;
    const uint32_t p0 = __shfl_sync(kFull, lb, 0);
    const bool tie = valid && k != FLT_MAX && lb < ub;
    __syncwarp();
    // nothing enters the beam: no candidate before position P, and none ties
    // the beam (a tie at diagonal P can swap the last entry for a candidate)
    if (__ballot_sync(kFull, pos < P || tie) == 0) return p0;
    int nfix = 0;
    if (__ballot_sync(kFull, tie) != 0) {
        if (valid) s.pos[lane] = pos;
        __syncwarp();
        nfix = tie_fixups(s.bidx, s.bdist, s.cidx, s.cdist, s.pos, reinterpret_cast<unsigned char*>(s.stage), cbs, P,
                          active, bnd, p0, lb, ub, tie, lane);
        if (nfix < 0) {
            merge_path_ties(s.bidx, s.bdist, s.cidx, s.cdist, s.pos, cbs, P, active, bnd, p0, lane);
            return p0;
        }
    }
    stable_shift<UNIFORM>(bidx, bdist, k, v, pos, P, p0, lane);
    if (nfix > 0) {
        const FixArea f = fix_area(reinterpret_cast<unsigned char*>(s.stage));
        if (lane < 4 * nfix && f.at[lane] != 0xFFFFu) {
            bidx[f.at[lane]] = f.idx[lane];
            bdist[f.at[lane]] = f.dist[lane];
        }
        __syncwarp();
    }
    return p0;
}

__device__ __forceinline__ int count_lt(const uint32_t* a, int n, uint32_t x) {
    int lo = 0, hi = n;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (a[mid] < x) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

// Flags the segments next to a boundary whose reference split differs from
// the stable one (only diagonals lb+m+1 .. ub+m of a tied candidate m can),
// and replays each flagged segment with the reference's splits into the
// fix-up list.  Returns the number of flagged segments, or -1 if they do not
// fit the list.
__device__ __noinline__ int tie_fixups(uint32_t* s_bidx, float* s_bdist, uint32_t* s_cidx, float* s_cdist,
                                       uint32_t* s_pos, unsigned char* s_fix, uint32_t cbs, uint32_t P, int active,
                                       const uint16_t* bnd, uint32_t p0, uint32_t lb, uint32_t ub, bool tie, int lane) {
    WSlice s;
    s.bidx = s_bidx;
    s.bdist = s_bdist;
    s.cidx = s_cidx;
    s.cdist = s_cdist;
    s.pos = s_pos;
    if (P > 4u * static_cast<uint32_t>(active)) return -1;  // segments longer than the list's 4 outputs
    const FixArea f = fix_area(s_fix);
    constexpr int kWords = (BLOCK_SIZE + 32) / 32;
    if (lane < kWords) f.mask[lane] = 0;
    __syncwarp();
    if (tie) {
        const uint32_t lo0 = lb + lane + 1, hi0 = ub + lane;
        const uint32_t lo = lo0 > p0 + 1 ? lo0 : p0 + 1;
        const uint32_t hi = hi0 < P ? hi0 : P;
        if (lo <= hi) {
            for (uint32_t sg = (lo * static_cast<uint32_t>(active) + P - 1) / P;
                 sg <= static_cast<uint32_t>(active) && bnd[sg] <= hi; ++sg) {
                const int d = bnd[sg];
                const int stable = d - count_lt(s.pos, static_cast<int>(cbs), static_cast<uint32_t>(d));
                const int ref = split_at(d, p0, s.pos, s.bdist, static_cast<int>(P), s.cdist, static_cast<int>(cbs));
                if (ref != stable) {
                    atomicOr(&f.mask[(sg - 1) >> 5], 1u << ((sg - 1) & 31));
                    if (sg < static_cast<uint32_t>(active)) atomicOr(&f.mask[sg >> 5], 1u << (sg & 31));
                }
            }
        }
    }
    __syncwarp();
    const uint32_t w = lane < kWords ? f.mask[lane] : 0u;
    uint32_t incl = __popc(w);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += y;
    }
    const int total = static_cast<int>(__shfl_sync(kFull, incl, 31));
    if (total == 0 || total > kMaxFixSegments) return total == 0 ? 0 : -1;
    // segment ids in flag order, one per lane (j < total)
    __syncwarp();
    uint32_t* list = f.list;
    {
        uint32_t m = w, at = incl - __popc(w);
        while (m) {
            const int b = __ffs(m) - 1;
            m &= m - 1;
            list[at++] = static_cast<uint32_t>(lane * 32 + b);
        }
    }
    __syncwarp();
    if (lane < 4 * total) f.at[lane] = 0xFFFFu;
    __syncwarp();
    if (lane < total) {
        const int sg = static_cast<int>(list[lane]);
        const int ob = bnd[sg], oe = bnd[sg + 1];
        int ti = split_at(ob, p0, s.pos, s.bdist, static_cast<int>(P), s.cdist, static_cast<int>(cbs));
        const int te = split_at(oe, p0, s.pos, s.bdist, static_cast<int>(P), s.cdist, static_cast<int>(cbs));
        int ci = ob - ti;
        const int ce = oe - te;
        for (int o = ob; o < oe; ++o) {
            const int e = 4 * lane + (o - ob);
            const bool take = (ci >= ce) || (ti < te && s.bdist[ti] <= s.cdist[ci]);
            f.at[e] = static_cast<uint16_t>(o);
            if (take) {
                f.idx[e] = s.bidx[ti];
                f.dist[e] = s.bdist[ti];
                ++ti;
            } else {
                f.idx[e] = s.cidx[ci];
                f.dist[e] = s.cdist[ci];
                ++ci;
            }
        }
    }
    __syncwarp();
    return total;
}

// More flagged segments than the fix-up list holds: every output position
// from p0 on replays its segment's beam-first merge between the reference's
// splits at the segment's two boundaries (split_at, which runs the
// reference's binary search where the split is ambiguous), all computed from
// the unmodified beam; positions are rewritten from the end and every source
// index is <= its output.
__device__ __noinline__ void merge_path_ties(uint32_t* s_bidx, float* s_bdist, uint32_t* s_cidx, float* s_cdist,
                                             uint32_t* s_pos, uint32_t cbs, uint32_t P, int active, const uint16_t* bnd,
                                             uint32_t p0, int lane) {
    uint32_t* bidx = s_bidx;
    float* bdist = s_bdist;
    const uint32_t first_chunk = p0 & ~31u;
    for (int c0 = static_cast<int>((P - 1) & ~31u); c0 >= static_cast<int>(first_chunk); c0 -= 32) {
        const uint32_t o = static_cast<uint32_t>(c0) + lane;
        const bool act = o < P && o >= p0;
        float od = 0.0f;
        uint32_t ov = 0;
        if (act) {
            uint32_t sg = (o * static_cast<uint32_t>(active)) / P;  // o * active < 2^18
            if (bnd[sg + 1] <= o) ++sg;
            const int ob = bnd[sg], oe = bnd[sg + 1];
            int ti = split_at(ob, p0, s_pos, bdist, static_cast<int>(P), s_cdist, static_cast<int>(cbs));
            const int te = split_at(oe, p0, s_pos, bdist, static_cast<int>(P), s_cdist, static_cast<int>(cbs));
            int ci = ob - ti;
            const int ce = oe - te;
            for (int j = ob;; ++j) {
                const bool take = (ci >= ce) || (ti < te && bdist[ti] <= s_cdist[ci]);
                if (j == static_cast<int>(o)) {
                    if (take) {
                        od = bdist[ti];
                        ov = bidx[ti];
                    } else {
                        od = s_cdist[ci];
                        ov = s_cidx[ci];
                    }
                    break;
                }
                if (take) ++ti;
                else ++ci;
            }
        }
        __syncwarp();
        if (act) {
            bdist[o] = od;
            bidx[o] = ov;
        }
        __syncwarp();
    }
}

// -------------------------------------------------------------- the search
// Visited-set reset to the beam's nodes (src/adaptive_search.cuh:129-133).
__device__ __noinline__ void restore_visited(uint32_t* hash, const uint32_t* bidx, uint32_t slots, int beam, int lane) {
    w_clear(hash, slots, lane);
    __syncwarp();
    for (int i = lane; i < beam; i += 32) w_insert(hash, slots, bidx[i] & ~kMsb);
    __syncwarp();
}

template <int W, int MERGE, bool IP, bool STAGED>
__device__ __forceinline__ void search_query(const SearchArgs& a, const WPlan& pl, const WSlice& s,
                                             const uint16_t* bnd, uint32_t qid, bool vec, int lane) {
    constexpr bool mp = MERGE == 0;
    constexpr int G = STAGED && W <= 4 ? 16 : 8;  // rows per exact-distance round
    const int dim = a.dim, deg = a.degree, beam = a.beam;
    const uint32_t P = pl.padded, cbs = pl.cbs, slots = pl.slots;
    const float* __restrict__ rows = a.rows;
    const uint64_t rowf = a.row;
    uint32_t* bidx = s.bidx;
    float* bdist = s.bdist;

    // ---------------------------------------------------------------- init
    const float* q = a.queries + static_cast<size_t>(qid) * dim;
    float qr[W];
#pragma unroll
    for (int k = 0; k < W; ++k) {
        const int d = lane + 32 * k;
        qr[k] = d < dim ? __ldg(q + d) : 0.0f;
    }
    {
        // rotation + quantisation, with the visited table as scratch
        float* qv = reinterpret_cast<float*>(s.hash);
        uint8_t* quant = reinterpret_cast<uint8_t*>(qv + ((dim + 3) & ~3));
        for (int i = lane; i < dim; i += 32) qv[i] = q[i];
        __syncwarp();
        prep_warp<W>(qv, a.signs, dim, quant, nullptr, s.qs, lane);
        build_planes(quant, 32 * W, s.planes, s.wrap, s.qs, lane);
        __syncwarp();
    }
    const QueryState qsl = *s.qs;
    __syncwarp();
    w_clear(s.hash, slots, lane);
    for (uint32_t i = lane; i < P; i += 32) {
        bidx[i] = kMax;
        bdist[i] = FLT_MAX;
    }
    s.cidx[lane] = kMax;
    s.cdist[lane] = FLT_MAX;
    __syncwarp();
    // entry point into candidate slot 0 (src/adaptive_search.cuh:110-118)
    const float ed = dist_one<W, IP>(rows + static_cast<uint64_t>(a.entry) * rowf, qr, dim, lane);
    if (lane == 0) {
        s.cidx[0] = a.entry;
        s.cdist[0] = ed;
        w_insert(s.hash, slots, a.entry);
    }
    __syncwarp();
    CtlRegs c;
    c.theta = PHASE1_THETA;
    c.rho = PHASE1_RHO;
    c.policy_iters = 0;
    c.top1 = kMax;
    c.stall = 0;
    c.warmup_done = false;
    c.entry_d = ed;
    c.last_d = FLT_MAX;
    c.cur_d = FLT_MAX;
    c.scan = 0;
    uint32_t c_iters = 0, c_exp = 0, c_eval = 1, n_est = 0;

    // ---------------------------------------------------------------- loop
    for (int iter = 0; iter < MAX_ITERATIONS; ++iter) {
        if ((iter + 1) % SMALL_HASH_RESET_INTERVAL == 0) restore_visited(s.hash, s.bidx, slots, beam, lane);
        if (iter >= pl.max_iter) break;

        // merge the previous iteration's candidates (:142-145)
        uint32_t p0 = 0;
        if constexpr (mp) {
            p0 = merge_path_warp<false>(s, cbs, P, pl.mp_active, bnd, lane);
        } else {
            merge_bitonic<MERGE>(bidx, bdist, s.cidx, s.cdist, cbs, iter == 0, lane);
            for (uint32_t i = static_cast<uint32_t>(beam) + lane; i < P; i += 32) {
                bidx[i] = kMax;
                bdist[i] = FLT_MAX;
            }
            __syncwarp();
        }
        ++c_iters;

        // control (src/adaptive_search.cuh:147-217)
        const float cutoff = bidx[beam - 1] == kMax ? FLT_MAX : bdist[(a.K < beam ? a.K : beam) - 1];
        const uint32_t b0 = bidx[0];
        __syncwarp();
        s.cidx[lane] = kMax;
        s.cdist[lane] = FLT_MAX;
        controller_update(c, b0, iter, pl.phase2_rho);
        uint32_t start = 0;
        if constexpr (mp) {
            if (p0 < c.scan) c.scan = p0;
            start = c.scan & ~31u;
        }
        // pick_expanders (include/utils.cuh:752-787)
        const uint32_t theta = static_cast<uint32_t>(c.theta);
        uint32_t num = 0, last_pick = 0;
        const uint32_t lim = (static_cast<uint32_t>(beam) + 31u) & ~31u;
        for (uint32_t j0 = start; j0 < lim; j0 += 32) {
            const uint32_t j = j0 + lane;
            uint32_t e = 0;
            const bool np = j < static_cast<uint32_t>(beam) && ((e = bidx[j]) & kMsb) == 0;
            const uint32_t b = __ballot_sync(kFull, np);
            const uint32_t i = __popc(b & lanemask_lt(lane)) + num;
            if (np && i < theta) {
                s.pnode[i] = e & 0x7fffffffu;
                s.pdist[i] = bdist[j];
                bidx[j] = e | kMsb;
            }
            if (num + __popc(b) >= theta) {
                const uint32_t sel = __ballot_sync(kFull, np && i == theta - 1);
                last_pick = j0 + (__ffs(sel) - 1);
                num = theta;
                break;
            }
            num += __popc(b);
        }
        __syncwarp();
        if constexpr (mp) c.scan = num == theta ? last_pick + 1 : static_cast<uint32_t>(beam);
        if (num) {
            // record_selected_expander_dist (adaptive_search_utils.cuh:41-49)
            c.last_d = finite_lt_max(c.cur_d) ? c.cur_d : c.entry_d;
            c.cur_d = s.pdist[num - 1];
        }
        if (a.trace && iter < a.trace_cap) {
            const size_t base = static_cast<size_t>(qid) * a.trace_cap + iter;
            if (lane < SEARCH_WIDTH) a.trace[base * SEARCH_WIDTH + lane] = lane < static_cast<int>(num) ? s.pnode[lane] : kMax;
            if (lane == 0) a.trace_count[base] = static_cast<int32_t>(num);
        }
        if (!num) break;
        c_exp += num;
        const int th = c.theta;
        const float rho = c.rho;
        const bool cut_ok = isfinite(cutoff) && cutoff < FLT_MAX;

        // both expansion paths end in one exact-distance call: the rows of
        // ev_nodes[0..ev_n) into s.cdist[ev_slot ? ev_slot[e] : e] (one copy
        // of the distance rounds keeps the loop's code small; warps of an SM
        // run both paths at the same time)
        const uint32_t* ev_nodes;
        const uint32_t* ev_slot;
        int ev_n;
        // the single expander runs in the controller's first phase only (about
        // one iteration in ten): the hint keeps it off the hot path's code
        // layout (0.9 % faster on a B200)
        if (__builtin_expect(!(th > 1), 0)) {
            // ---------------------------- single expander (src/adaptive_search.cuh:221-343)
            const uint32_t work = static_cast<uint32_t>(deg) < cbs ? static_cast<uint32_t>(deg) : cbs;
            const float* prow = rows + static_cast<uint64_t>(s.pnode[0]) * rowf;
            const float pd = s.pdist[0];
            ParentLane<W> p;
            load_parent_pinned<W>(prow, a, static_cast<int>(work), vec, lane, p);
            const bool in_work = static_cast<uint32_t>(lane) < work;
            uint32_t child = p.child;
            if (child != kMax && (child >= a.n || w_contains<true>(s.hash, slots, child))) child = kMax;
            float dist = child == kMax ? FLT_MAX : 0.0f;
            const int keep = keep_for(work, th, rho, false, 0);
            const uint32_t vcount = __popc(__ballot_sync(kFull, in_work && child != kMax));
            int admit = static_cast<int>(work);
            if (keep < static_cast<int>(vcount)) {
                if (child != kMax) {
                    // theta = 1 variant: triple_x == FLT_MAX estimates 0.0 (include/utils.cuh:951-952)
                    float est = 0.0f;
                    if (p.tx != FLT_MAX) {
                        const uint32_t raw = parent_raw<W>(p, prow, a, lane, s.planes, s.wrap, qsl.wrap_any);
                        est = estimate(raw, p.tx, p.fdq, p.fvq, pd, qsl);
                    }
                    if (isfinite(est)) {
                        dist = est;
                    } else {
                        dist = FLT_MAX;
                        child = kMax;
                    }
                }
                n_est += vcount;
                const uint32_t near =
                    cut_ok ? __popc(__ballot_sync(kFull, in_work && child != kMax && isfinite(dist) && dist <= cutoff)) : 0u;
                const int eff = keep_for(work, th, rho, cut_ok, near);
                float kk = lane < static_cast<int>(cbs) ? dist : FLT_MAX;
                uint32_t vv = lane < static_cast<int>(cbs) ? child : kMax;
                sort32(kk, vv, lane);
                if (lane >= eff) {
                    kk = FLT_MAX;
                    vv = kMax;
                }
                dist = kk;
                child = vv;
                admit = eff;
            }
            // insert kept children (first occurrence wins), list them for evaluation
            const bool want = lane < admit && child != kMax && dist < FLT_MAX;
            const uint32_t same = __match_any_sync(kFull, want ? child : kMax);
            const bool first = want && (__ffs(same) - 1) == lane;
            const bool ins = first && w_insert(s.hash, slots, child);
            if (lane < static_cast<int>(cbs)) s.cidx[lane] = ins ? child : kMax;
            const uint32_t ib = __ballot_sync(kFull, ins);
            if (ins) {
                const uint32_t r = __popc(ib & lanemask_lt(lane));
                s.stage[r] = child;
                s.eslot[r] = lane;
            }
            __syncwarp();
            const int ne = __popc(ib);
            c_eval += ne;
            ev_nodes = s.stage;
            ev_slot = s.eslot;
            ev_n = ne;
        } else {
            // ----------------------- speculative expanders (src/adaptive_search.cuh:344-444)
            // degree <= 32: lane l holds neighbour l of every parent; every
            // lookup of the iteration happens before its inserts.
            const uint32_t active = static_cast<uint32_t>(deg) < 32u ? static_cast<uint32_t>(deg) : 32u;
            const int keep0 = keep_for(active, th, rho, false, 0);
            // keep_for(active, th, rho, cut, near) = clamp(cut ? clamp(near, 1, cap) : cap, 1, active)
            const int cap = keep_cap(active, th, rho);
            ParentLane<W> cur;
            if constexpr (STAGED) {
                // every parent's block in flight at once: one cp.async group
                // per parent into its ring slot (blocks are 16-byte aligned)
                const uint32_t chunks = pl.blk >> 4;
                for (uint32_t t = 0; t < num; ++t) {
                    const unsigned char* src = reinterpret_cast<const unsigned char*>(
                        rows + static_cast<uint64_t>(s.pnode[t]) * rowf + a.code_off);
                    unsigned char* dst = s.ring + t * pl.blk;
                    for (uint32_t c = static_cast<uint32_t>(lane); c < chunks; c += 32) cp_async16(dst + 16 * c, src + 16 * c);
                    cp_async_commit();
                }
            } else {
                // one parent per step; the next parent's block is loaded while
                // this one is examined (the last step reloads its own block)
                load_parent_pinned<W>(rows + static_cast<uint64_t>(s.pnode[0]) * rowf, a, deg, vec, lane, cur);
            }
            uint32_t total = 0;
#pragma unroll 1
            for (int t = 0; t < static_cast<int>(num); ++t) {
                ParentLane<W> nxt;
                if constexpr (STAGED) {
                    cp_async_wait_groups(static_cast<int>(num) - 1 - t);
                    __syncwarp();
                    parent_from_ring<W>(s.ring + t * pl.blk, deg, 32 * W, lane, cur);
                } else {
                    const int tn = t + 1 < static_cast<int>(num) ? t + 1 : t;
                    load_parent_pinned<W>(rows + static_cast<uint64_t>(s.pnode[tn]) * rowf, a, deg, vec, lane, nxt);
                }
                const uint32_t child = cur.child;
                bool valid = child != kMax && child < a.n && !w_contains<true>(s.hash, slots, child);
                const uint32_t raw_valid = __popc(__ballot_sync(kFull, valid));
                bool kl;
                if (keep0 >= static_cast<int>(raw_valid)) {
                    kl = valid;
                } else {
                    float est = FLT_MAX;
                    if (valid) {
                        // speculative variant: triple_x == FLT_MAX estimates FLT_MAX
                        if (cur.tx != FLT_MAX) {
                            uint32_t raw;
                            if constexpr (W % 4 == 0) {
                                raw = raw_sum_v<W>(cur.c, s.planes, s.wrap, qsl.wrap_any);
                            } else {
                                const float* prow = rows + static_cast<uint64_t>(s.pnode[t]) * rowf;
                                raw = parent_raw<W>(cur, prow, a, lane, s.planes, s.wrap, qsl.wrap_any);
                            }
                            est = estimate(raw, cur.tx, cur.fdq, cur.fvq, s.pdist[t], qsl);
                        }
                        valid = isfinite(est);
                    }
                    n_est += raw_valid;
                    const int near = __popc(__ballot_sync(kFull, valid && cut_ok && est <= cutoff));
                    int eff = cut_ok ? (near < 1 ? 1 : (near > cap ? cap : near)) : cap;
                    eff = eff < 1 ? 1 : (eff > static_cast<int>(active) ? static_cast<int>(active) : eff);
                    kl = keep_smallest(est, valid, eff, lane);
                }
                const uint32_t kb = __ballot_sync(kFull, kl);
                if (kl) {
                    const uint32_t r = total + __popc(kb & lanemask_lt(lane));
                    if (r < 32u) s.stage[r] = child;
                }
                total += __popc(kb);
                if constexpr (!STAGED) cur = nxt;
            }
            __syncwarp();
            // inserts and compaction in (parent, rank) order; a child kept by
            // two parents goes to the first (include/utils.cuh:187-214)
            const uint32_t child = lane < static_cast<int>(total) ? s.stage[lane] : kMax;
            const uint32_t same = __match_any_sync(kFull, child);
            const bool first = child != kMax && (__ffs(same) - 1) == lane;
            const bool ins = first && w_insert(s.hash, slots, child);
            const uint32_t ib = __ballot_sync(kFull, ins);
            const uint32_t slot = __popc(ib & lanemask_lt(lane));
            const uint32_t compact = __popc(ib);
            const uint32_t ne = compact < pl.collect_cap ? compact : pl.collect_cap;
            if (ins && slot < pl.collect_cap) s.cidx[slot] = child;
            __syncwarp();
            c_eval += ne;
            ev_nodes = s.cidx;
            ev_slot = nullptr;
            ev_n = static_cast<int>(ne);
        }
        eval_nodes<W, G, IP>(rows, rowf, dim, qr, ev_nodes, ev_n, s.cdist, ev_slot, lane);
        __syncwarp();
    }
    // final merge (src/adaptive_search.cuh:448-452)
    if constexpr (mp) {
        merge_path_warp<false>(s, cbs, P, pl.mp_active, bnd, lane);
    } else {
        merge_bitonic<MERGE>(bidx, bdist, s.cidx, s.cdist, cbs, false, lane);
    }
    __syncwarp();
    // results (:455-464): position i < beam holds the beam entry with its MSB
    // cleared; positions >= beam repeat the last one
    for (int i = lane; i < a.K; i += 32) {
        const int sp = i < beam ? i : beam - 1;
        a.out_ids[static_cast<size_t>(qid) * a.K + i] = bidx[sp] & 0x7fffffffu;
        if (a.out_dists) a.out_dists[static_cast<size_t>(qid) * a.K + i] = bdist[sp];
    }
    if (lane == 0 && a.stats) {
        fg_query_stats st;
        st.iterations = c_iters;
        st.expansions = c_exp;
        st.evaluations = c_eval;
        st.estimates = n_est;
        a.stats[qid] = st;
    }
    __syncwarp();
}

// ------------------------------------------------------------ pair mode
// Two warps per query: the leader keeps the query's serial steps (merge,
// controller, expander pick, compaction and inserts, result write) and both
// warps split the parallel ones -- the parents of a speculative iteration
// (the leader takes parents 0, 2, 4, ..., the follower 1, 3, 5, ...) and the
// exact-distance rounds.  Each parent's kept children go to a list of their
// own, so the leader's compaction sees them in (parent, rank) order exactly
// as the one-warp search does, and every visited-set lookup of an iteration
// still precedes its inserts.  The two warps meet at a named barrier (64
// threads, one per pair of the CTA) at points both reach on every
// path: after set-up, after the pick, after the parents, after the
// compaction, after the distances, and at the end of the query.  Results are
// the one-warp search's, bit for bit.
struct PairCtl {
    QueryState qs;
    uint32_t qid;
    int stop;        // the leader found no expander (or hit the iteration limit)
    int th;
    float rho;
    float cutoff;
    uint32_t num;
    int ev_n;
    uint32_t nest_f;  // the follower's estimate count
    uint32_t kc[SEARCH_WIDTH];  // children kept per parent
};

// shared bytes after the slice: the control block, then SEARCH_WIDTH lists of 32 ids
constexpr size_t kPairCtlBytes = (sizeof(PairCtl) + 15) & ~static_cast<size_t>(15);
constexpr size_t kPairExtraBytes = kPairCtlBytes + static_cast<size_t>(SEARCH_WIDTH) * 32 * 4;

// Barrier of the pair with index `pair` in its CTA (ids 1 and 2; 0 is
// __syncthreads).  The ids are immediates: a barrier id in a register makes
// ptxas reserve all 16 barriers of the CTA, which caps the CTAs per SM.
__device__ __forceinline__ void pair_sync(int pair) {
    if (pair == 0) asm volatile("bar.sync 1, 64;" ::: "memory");
    else asm volatile("bar.sync 2, 64;" ::: "memory");
}

template <int W, int MERGE, bool IP>
__device__ __forceinline__ void search_query_pair(const SearchArgs& a, const WPlan& pl, const WSlice& s, PairCtl* ctl,
                                                  uint32_t* kp, const uint16_t* bnd, uint32_t qid, bool vec, int lane,
                                                  int role, int bar) {
    constexpr bool mp = MERGE == 0;
    constexpr int G = 8;  // rows per exact-distance round
    const bool lead = role == 0;
    const int dim = a.dim, deg = a.degree, beam = a.beam;
    const uint32_t P = pl.padded, cbs = pl.cbs, slots = pl.slots;
    const float* __restrict__ rows = a.rows;
    const uint64_t rowf = a.row;
    uint32_t* bidx = s.bidx;
    float* bdist = s.bdist;

    // ---------------------------------------------------------------- init
    const float* q = a.queries + static_cast<size_t>(qid) * dim;
    float qr[W];
#pragma unroll
    for (int k = 0; k < W; ++k) {
        const int d = lane + 32 * k;
        qr[k] = d < dim ? __ldg(q + d) : 0.0f;
    }
    CtlRegs c;
    c.theta = PHASE1_THETA;
    c.rho = PHASE1_RHO;
    c.policy_iters = 0;
    c.top1 = kMax;
    c.stall = 0;
    c.warmup_done = false;
    c.entry_d = FLT_MAX;
    c.last_d = FLT_MAX;
    c.cur_d = FLT_MAX;
    c.scan = 0;
    if (lead) {
        float* qv = reinterpret_cast<float*>(s.hash);
        uint8_t* quant = reinterpret_cast<uint8_t*>(qv + ((dim + 3) & ~3));
        for (int i = lane; i < dim; i += 32) qv[i] = q[i];
        __syncwarp();
        prep_warp<W>(qv, a.signs, dim, quant, nullptr, s.qs, lane);
        build_planes(quant, 32 * W, s.planes, s.wrap, s.qs, lane);
        __syncwarp();
        if (lane == 0) ctl->qs = *s.qs;
        __syncwarp();
        w_clear(s.hash, slots, lane);
        for (uint32_t i = lane; i < P; i += 32) {
            bidx[i] = kMax;
            bdist[i] = FLT_MAX;
        }
        s.cidx[lane] = kMax;
        s.cdist[lane] = FLT_MAX;
        __syncwarp();
        // entry point into candidate slot 0 (src/adaptive_search.cuh:110-118)
        const float ed = dist_one<W, IP>(rows + static_cast<uint64_t>(a.entry) * rowf, qr, dim, lane);
        if (lane == 0) {
            s.cidx[0] = a.entry;
            s.cdist[0] = ed;
            w_insert(s.hash, slots, a.entry);
        }
        __syncwarp();
        c.entry_d = ed;
    }
    pair_sync(bar);
    const QueryState qsl = ctl->qs;
    uint32_t c_iters = 0, c_exp = 0, c_eval = 1, n_est = 0;

    // ---------------------------------------------------------------- loop
    for (int iter = 0; iter < MAX_ITERATIONS; ++iter) {
        if (lead && (iter + 1) % SMALL_HASH_RESET_INTERVAL == 0) restore_visited(s.hash, s.bidx, slots, beam, lane);
        if (iter >= pl.max_iter) break;  // the same on both warps

        if (lead) {
            // merge the previous iteration's candidates (:142-145)
            uint32_t p0 = 0;
            if constexpr (mp) {
                p0 = merge_path_warp<true>(s, cbs, P, pl.mp_active, bnd, lane);
            } else {
                merge_bitonic<MERGE>(bidx, bdist, s.cidx, s.cdist, cbs, iter == 0, lane);
                for (uint32_t i = static_cast<uint32_t>(beam) + lane; i < P; i += 32) {
                    bidx[i] = kMax;
                    bdist[i] = FLT_MAX;
                }
                __syncwarp();
            }
            ++c_iters;
            // control (src/adaptive_search.cuh:147-217)
            const float cutoff = bidx[beam - 1] == kMax ? FLT_MAX : bdist[(a.K < beam ? a.K : beam) - 1];
            const uint32_t b0 = bidx[0];
            __syncwarp();
            s.cidx[lane] = kMax;
            s.cdist[lane] = FLT_MAX;
            controller_update(c, b0, iter, pl.phase2_rho);
            uint32_t start = 0;
            if constexpr (mp) {
                if (p0 < c.scan) c.scan = p0;
                start = c.scan & ~31u;
            }
            // pick_expanders (include/utils.cuh:752-787)
            const uint32_t theta = static_cast<uint32_t>(c.theta);
            uint32_t num = 0, last_pick = 0;
            const uint32_t lim = (static_cast<uint32_t>(beam) + 31u) & ~31u;
            for (uint32_t j0 = start; j0 < lim; j0 += 32) {
                const uint32_t j = j0 + lane;
                uint32_t e = 0;
                const bool np = j < static_cast<uint32_t>(beam) && ((e = bidx[j]) & kMsb) == 0;
                const uint32_t b = __ballot_sync(kFull, np);
                const uint32_t i = __popc(b & lanemask_lt(lane)) + num;
                if (np && i < theta) {
                    s.pnode[i] = e & 0x7fffffffu;
                    s.pdist[i] = bdist[j];
                    bidx[j] = e | kMsb;
                }
                if (num + __popc(b) >= theta) {
                    const uint32_t sel = __ballot_sync(kFull, np && i == theta - 1);
                    last_pick = j0 + (__ffs(sel) - 1);
                    num = theta;
                    break;
                }
                num += __popc(b);
            }
            __syncwarp();
            if constexpr (mp) c.scan = num == theta ? last_pick + 1 : static_cast<uint32_t>(beam);
            if (num) {
                c.last_d = finite_lt_max(c.cur_d) ? c.cur_d : c.entry_d;
                c.cur_d = s.pdist[num - 1];
            }
            if (a.trace && iter < a.trace_cap) {
                const size_t base = static_cast<size_t>(qid) * a.trace_cap + iter;
                if (lane < SEARCH_WIDTH)
                    a.trace[base * SEARCH_WIDTH + lane] = lane < static_cast<int>(num) ? s.pnode[lane] : kMax;
                if (lane == 0) a.trace_count[base] = static_cast<int32_t>(num);
            }
            if (lane == 0) {
                ctl->stop = num == 0;
                ctl->num = num;
                ctl->th = c.theta;
                ctl->rho = c.rho;
                ctl->cutoff = cutoff;
            }
            c_exp += num;
        }
        pair_sync(bar);
        if (ctl->stop) break;  // the same on both warps
        const uint32_t num = ctl->num;
        const int th = ctl->th;
        const float rho = ctl->rho;
        const float cutoff = ctl->cutoff;
        const bool cut_ok = isfinite(cutoff) && cutoff < FLT_MAX;

        if (!(th > 1)) {
            // ---------------------------- single expander (src/adaptive_search.cuh:221-343), leader only
            if (lead) {
                const uint32_t work = static_cast<uint32_t>(deg) < cbs ? static_cast<uint32_t>(deg) : cbs;
                const float* prow = rows + static_cast<uint64_t>(s.pnode[0]) * rowf;
                const float pd = s.pdist[0];
                ParentLane<W> p;
                load_parent_pinned<W>(prow, a, static_cast<int>(work), vec, lane, p);
                const bool in_work = static_cast<uint32_t>(lane) < work;
                uint32_t child = p.child;
                if (child != kMax && (child >= a.n || w_contains<false>(s.hash, slots, child))) child = kMax;
                float dist = child == kMax ? FLT_MAX : 0.0f;
                const int keep = keep_for(work, th, rho, false, 0);
                const uint32_t vcount = __popc(__ballot_sync(kFull, in_work && child != kMax));
                int admit = static_cast<int>(work);
                if (keep < static_cast<int>(vcount)) {
                    if (child != kMax) {
                        // theta = 1 variant: triple_x == FLT_MAX estimates 0.0 (include/utils.cuh:951-952)
                        float est = 0.0f;
                        if (p.tx != FLT_MAX) {
                            const uint32_t raw = parent_raw<W>(p, prow, a, lane, s.planes, s.wrap, qsl.wrap_any);
                            est = estimate(raw, p.tx, p.fdq, p.fvq, pd, qsl);
                        }
                        if (isfinite(est)) {
                            dist = est;
                        } else {
                            dist = FLT_MAX;
                            child = kMax;
                        }
                    }
                    n_est += vcount;
                    const uint32_t near =
                        cut_ok ? __popc(__ballot_sync(kFull, in_work && child != kMax && isfinite(dist) && dist <= cutoff)) : 0u;
                    const int eff = keep_for(work, th, rho, cut_ok, near);
                    float kk = lane < static_cast<int>(cbs) ? dist : FLT_MAX;
                    uint32_t vv = lane < static_cast<int>(cbs) ? child : kMax;
                    sort32(kk, vv, lane);
                    if (lane >= eff) {
                        kk = FLT_MAX;
                        vv = kMax;
                    }
                    dist = kk;
                    child = vv;
                    admit = eff;
                }
                const bool want = lane < admit && child != kMax && dist < FLT_MAX;
                const uint32_t same = __match_any_sync(kFull, want ? child : kMax);
                const bool first = want && (__ffs(same) - 1) == lane;
                const bool ins = first && w_insert(s.hash, slots, child);
                if (lane < static_cast<int>(cbs)) s.cidx[lane] = ins ? child : kMax;
                const uint32_t ib = __ballot_sync(kFull, ins);
                if (ins) {
                    const uint32_t r = __popc(ib & lanemask_lt(lane));
                    s.stage[r] = child;
                    s.eslot[r] = lane;
                }
                __syncwarp();
                const int ne = __popc(ib);
                c_eval += ne;
                if (lane == 0) ctl->ev_n = ne;
            }
        } else {
            // ----------------------- speculative expanders (src/adaptive_search.cuh:344-444)
            // this warp's parents t = role, role + 2, ...; lane l holds neighbour l
            const uint32_t active = static_cast<uint32_t>(deg) < 32u ? static_cast<uint32_t>(deg) : 32u;
            const int keep0 = keep_for(active, th, rho, false, 0);
            const int cap = keep_cap(active, th, rho);
            ParentLane<W> cur;
            if (static_cast<uint32_t>(role) < num)
                load_parent_pinned<W>(rows + static_cast<uint64_t>(s.pnode[role]) * rowf, a, deg, vec, lane, cur);
#pragma unroll 1
            for (int t = role; t < static_cast<int>(num); t += 2) {
                const int tn = t + 2 < static_cast<int>(num) ? t + 2 : t;
                ParentLane<W> nxt;
                load_parent_pinned<W>(rows + static_cast<uint64_t>(s.pnode[tn]) * rowf, a, deg, vec, lane, nxt);
                const uint32_t child = cur.child;
                bool valid = child != kMax && child < a.n && !w_contains<false>(s.hash, slots, child);
                const uint32_t raw_valid = __popc(__ballot_sync(kFull, valid));
                bool kl;
                if (keep0 >= static_cast<int>(raw_valid)) {
                    kl = valid;
                } else {
                    float est = FLT_MAX;
                    if (valid) {
                        // speculative variant: triple_x == FLT_MAX estimates FLT_MAX
                        if (cur.tx != FLT_MAX) {
                            uint32_t raw;
                            if constexpr (W % 4 == 0) {
                                raw = raw_sum_v<W>(cur.c, s.planes, s.wrap, qsl.wrap_any);
                            } else {
                                const float* prow = rows + static_cast<uint64_t>(s.pnode[t]) * rowf;
                                raw = parent_raw<W>(cur, prow, a, lane, s.planes, s.wrap, qsl.wrap_any);
                            }
                            est = estimate(raw, cur.tx, cur.fdq, cur.fvq, s.pdist[t], qsl);
                        }
                        valid = isfinite(est);
                    }
                    n_est += raw_valid;
                    const int near = __popc(__ballot_sync(kFull, valid && cut_ok && est <= cutoff));
                    int eff = cut_ok ? (near < 1 ? 1 : (near > cap ? cap : near)) : cap;
                    eff = eff < 1 ? 1 : (eff > static_cast<int>(active) ? static_cast<int>(active) : eff);
                    kl = keep_smallest(est, valid, eff, lane);
                }
                const uint32_t kb = __ballot_sync(kFull, kl);
                if (kl) kp[t * 32 + __popc(kb & lanemask_lt(lane))] = child;
                if (lane == 0) ctl->kc[t] = __popc(kb);
                cur = nxt;
            }
            pair_sync(bar);
            if (lead) {
                // the kept children in (parent, rank) order, the first 32;
                // a child kept by two parents goes to the first (include/utils.cuh:187-214)
                uint32_t child = kMax;
                uint32_t base = 0;
                for (uint32_t t = 0; t < num; ++t) {
                    const uint32_t k = ctl->kc[t];
                    if (static_cast<uint32_t>(lane) >= base && static_cast<uint32_t>(lane) < base + k)
                        child = kp[t * 32 + (lane - base)];
                    base += k;
                }
                const uint32_t same = __match_any_sync(kFull, child);
                const bool first = child != kMax && (__ffs(same) - 1) == lane;
                const bool ins = first && w_insert(s.hash, slots, child);
                const uint32_t ib = __ballot_sync(kFull, ins);
                const uint32_t slot = __popc(ib & lanemask_lt(lane));
                const uint32_t compact = __popc(ib);
                const uint32_t ne = compact < pl.collect_cap ? compact : pl.collect_cap;
                if (ins && slot < pl.collect_cap) s.cidx[slot] = child;
                __syncwarp();
                c_eval += ne;
                if (lane == 0) ctl->ev_n = static_cast<int>(ne);
            }
        }
        pair_sync(bar);
        // exact distances, rounds split between the two warps
        const int ev_n = ctl->ev_n;
        if (th > 1) eval_nodes<W, G, IP>(rows, rowf, dim, qr, s.cidx, ev_n, s.cdist, nullptr, lane, role * G, 2 * G);
        else eval_nodes<W, G, IP>(rows, rowf, dim, qr, s.stage, ev_n, s.cdist, s.eslot, lane, role * G, 2 * G);
        pair_sync(bar);
    }
    if (!lead && lane == 0) ctl->nest_f = n_est;
    pair_sync(bar);
    if (!lead) return;
    // final merge (src/adaptive_search.cuh:448-452)
    if constexpr (mp) {
        merge_path_warp<true>(s, cbs, P, pl.mp_active, bnd, lane);
    } else {
        merge_bitonic<MERGE>(bidx, bdist, s.cidx, s.cdist, cbs, false, lane);
    }
    __syncwarp();
    for (int i = lane; i < a.K; i += 32) {
        const int sp = i < beam ? i : beam - 1;
        a.out_ids[static_cast<size_t>(qid) * a.K + i] = bidx[sp] & 0x7fffffffu;
        if (a.out_dists) a.out_dists[static_cast<size_t>(qid) * a.K + i] = bdist[sp];
    }
    if (lane == 0 && a.stats) {
        fg_query_stats st;
        st.iterations = c_iters;
        st.expansions = c_exp;
        st.evaluations = c_eval;
        st.estimates = n_est + ctl->nest_f;
        a.stats[qid] = st;
    }
    __syncwarp();
}

template <int W, int MERGE, bool IP, int MINB, int MODE>
__global__ void __launch_bounds__(kWarpsPerCta * 32, MINB) search_warp_kernel(const SearchArgs a, const WPlan pl,
                                                                                  int vec_codes) {
    constexpr bool kStaged = MODE == kModeStaged;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    // merge-path output segment boundaries s * itopk / active (launch constants)
    __shared__ uint16_t bnd[MERGE == 0 ? BLOCK_SIZE + 1 : 1];
    if constexpr (MERGE == 0) {
        for (int sg = threadIdx.x; sg <= pl.mp_active; sg += blockDim.x)
            bnd[sg] = static_cast<uint16_t>((static_cast<uint32_t>(sg) * pl.padded) / static_cast<uint32_t>(pl.mp_active));
    }
    __syncthreads();  // the only block-wide barrier: warps (or pairs of warps) are independent from here on
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if constexpr (MODE == kModePair) {
        const int pair = warp >> 1, role = warp & 1, bar = pair;
        WSlice s;
        slice_layout(pl.padded, pl.slots, 32 * W, MERGE == 0, &s, smem_raw + static_cast<size_t>(pair) * pl.slice,
                     kPairExtraBytes);
        PairCtl* ctl = reinterpret_cast<PairCtl*>(s.ring);
        uint32_t* kp = reinterpret_cast<uint32_t*>(s.ring + kPairCtlBytes);
        for (;;) {
            if (role == 0 && lane == 0) ctl->qid = atomicAdd(a.work_counter, 1u);
            pair_sync(bar);
            const uint32_t qid = ctl->qid;
            if (qid >= static_cast<uint32_t>(a.nq)) break;  // the same on both warps
            search_query_pair<W, MERGE, IP>(a, pl, s, ctl, kp, bnd, qid, vec_codes != 0, lane, role, bar);
        }
    } else {
        WSlice s;
        slice_layout(pl.padded, pl.slots, 32 * W, MERGE == 0, &s, smem_raw + static_cast<size_t>(warp) * pl.slice,
                     kStaged ? static_cast<size_t>(SEARCH_WIDTH) * pl.blk : 0);
        for (;;) {
            uint32_t qid = 0;
            if (lane == 0) qid = atomicAdd(a.work_counter, 1u);
            qid = __shfl_sync(kFull, qid, 0);
            if (qid >= static_cast<uint32_t>(a.nq)) break;
            search_query<W, MERGE, IP, kStaged>(a, pl, s, bnd, qid, vec_codes != 0, lane);
        }
    }
}

template <int W, bool IP, int MINB, int MODE>
const void* pick_merge_w(int merge) {
    switch (merge) {
        case 1: return reinterpret_cast<const void*>(search_warp_kernel<W, 1, IP, MINB, MODE>);
        case 2: return reinterpret_cast<const void*>(search_warp_kernel<W, 2, IP, MINB, MODE>);
        case 4: return reinterpret_cast<const void*>(search_warp_kernel<W, 4, IP, MINB, MODE>);
        default: return reinterpret_cast<const void*>(search_warp_kernel<W, 0, IP, MINB, MODE>);
    }
}

template <bool IP, int MINB, int MODE>
const void* pick_w(int W, int merge) {
    switch (W) {
        case 1: return pick_merge_w<1, IP, MINB, MODE>(merge);
        case 2: return pick_merge_w<2, IP, MINB, MODE>(merge);
        case 4: return pick_merge_w<4, IP, MINB, MODE>(merge);
        default: return pick_merge_w<8, IP, MINB, MODE>(merge);
    }
}

template <int MINB, int MODE>
const void* pick_ip(int W, int merge, bool ip) {
    return ip ? pick_w<true, MINB, MODE>(W, merge) : pick_w<false, MINB, MODE>(W, merge);
}

// kernel for W = padded dim / 32, the beam merge, the metric, the register
// budget and the mode (one warp per query; staged; a pair of warps per query)
const void* warp_kernel_for(int W, int merge, bool ip, int minb, int mode) {
    if (mode == kModePair) return pick_ip<kCtasPair, kModePair>(W, merge, ip);
    if (mode == kModeStaged) return pick_ip<kCtasStaged, kModeStaged>(W, merge, ip);
    if (minb == kCtasSmall) return pick_ip<kCtasSmall, kModeWarp>(W, merge, ip);
    return pick_ip<kCtasLarge, kModeWarp>(W, merge, ip);
}

}  // namespace

bool warp_kernel_supports(int padded_dim) { return padded_dim >= 32 && padded_dim <= 256; }

// Bytes of a parent's expansion block (codes, three factors, ids); the staged
// variant needs it 16-byte aligned and a multiple of 16 bytes.
static uint32_t parent_block_bytes(const SearchArgs& a) {
    return static_cast<uint32_t>(a.degree) * static_cast<uint32_t>(a.padded_dim / 8 + 16);
}

bool warp_staged_supported(const SearchArgs& a, const SearchPlan& p) {
    return p.vec_codes && (parent_block_bytes(a) % 16) == 0;
}

// mode: kModeWarp (one warp per query), kModeStaged (falls back to kModeWarp
// where the blocks are not 16-byte aligned) or kModePair (two warps per query).
int plan_search_warp(const SearchArgs& a, SearchPlan* p, int device, char* err, size_t errlen, int mode) {
    const int D = a.padded_dim;
    uint32_t req = p->padded + p->cbs * SMALL_HASH_RESET_INTERVAL;
    uint32_t slots = req + (req + 11) / 12;  // ~93 % at the bound (two-choice buckets)
    // the table doubles as the query's scratch during set-up
    const uint32_t scratch = (static_cast<uint32_t>((a.dim + 3) & ~3) * 4 + static_cast<uint32_t>(D) + 3) / 4;
    if (slots < scratch) slots = scratch;
    slots = (slots + 31) & ~31u;
    p->kernel = 1;
    p->slots = slots;
    if (mode == kModeStaged && !warp_staged_supported(a, *p)) mode = kModeWarp;
    p->warp_mode = mode;
    p->blk = mode == kModeStaged ? parent_block_bytes(a) : 0;
    const size_t extra = mode == kModeStaged ? static_cast<size_t>(SEARCH_WIDTH) * p->blk
                         : mode == kModePair ? kPairExtraBytes : 0;
    // bytes per query (per warp, or per pair of warps in the pair mode)
    p->slice_bytes = slice_layout(p->padded, slots, D, p->merge_n2 == 0, nullptr, nullptr, extra);
    const int warps_per_query = mode == kModePair ? 2 : 1;
    int sms = 0, max_smem = 0;
    cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    if (e != cudaSuccess) {
        snprintf(err, errlen, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
        return FG_ERR_CUDA;
    }
    if (p->slice_bytes > static_cast<size_t>(max_smem)) {
        snprintf(err, errlen, "shared memory %zu exceeds the device limit %d", p->slice_bytes, max_smem);
        return FG_ERR_UNSUPPORTED;
    }
    // resident queries per SM for every register budget and CTA size (queries
    // per CTA), as the occupancy calculator counts them; the most wins, ties
    // go to the larger CTA
    const void* best = nullptr;
    int best_q = 0;
    // FG_CTA_WARPS=1|2|4 restricts the CTA size (a tuning knob; results do not depend on it)
    const char* cw = getenv("FG_CTA_WARPS");
    const int cta_warps = cw ? atoi(cw) : 0;
    int budgets[2] = {kCtasSmall, kCtasLarge};
    int nbudgets = 2;
    if (mode == kModeStaged) budgets[0] = kCtasStaged, nbudgets = 1;
    if (mode == kModePair) budgets[0] = kCtasPair, nbudgets = 1;
    for (int bi = 0; bi < nbudgets; ++bi) {
        const int minb = budgets[bi];
        const void* fn = warp_kernel_for(D / 32, p->merge_n2, a.use_ip != 0, minb, mode);
        for (int wpc : {kWarpsPerCta, 2, 1}) {
            if (wpc % warps_per_query) continue;
            if (cta_warps && wpc != cta_warps) continue;
            const int qpc = wpc / warps_per_query;
            const size_t smem = p->slice_bytes * static_cast<size_t>(qpc);
            if (smem > static_cast<size_t>(max_smem)) continue;
            e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
            int per_sm = 0;
            if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, wpc * 32, smem);
            if (e != cudaSuccess) {
                snprintf(err, errlen, "occupancy query failed: %s", cudaGetErrorString(e));
                return FG_ERR_CUDA;
            }
            if (per_sm * qpc > best_q) {
                best_q = per_sm * qpc;
                best = fn;
                p->min_ctas = minb;
                p->threads = wpc * 32;
                p->smem_bytes = smem;
                p->blocks_per_sm = per_sm;
            }
        }
    }
    if (!best) {
        snprintf(err, errlen, "no launch shape fits: %zu bytes of shared memory per query", p->slice_bytes);
        return FG_ERR_UNSUPPORTED;
    }
    e = cudaFuncSetAttribute(best, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(p->smem_bytes));
    if (e != cudaSuccess) {
        snprintf(err, errlen, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        return FG_ERR_CUDA;
    }
    const int qpc = p->threads / 32 / warps_per_query;
    const int resident = p->blocks_per_sm * sms;
    const int need = (a.nq + qpc - 1) / qpc;
    p->grid = need < resident ? need : resident;
    if (p->grid < 1) p->grid = 1;
    p->resident_queries = resident * qpc;
    return FG_OK;
}

cudaError_t launch_search_warp(const SearchArgs& a, const SearchPlan& p, cudaStream_t stream) {
    WPlan pl;
    pl.padded = p.padded;
    pl.cbs = p.cbs;
    pl.collect_cap = p.collect_cap;
    pl.slots = p.slots;
    pl.phase2_rho = p.phase2_rho;
    pl.max_iter = p.max_iter;
    pl.mp_active = p.mp_active;
    pl.slice = static_cast<uint32_t>(p.slice_bytes);
    pl.blk = p.blk;
    cudaError_t e = cudaMemsetAsync(a.work_counter, 0, sizeof(uint32_t), stream);
    if (e != cudaSuccess) return e;
    const void* fn = warp_kernel_for(a.padded_dim / 32, p.merge_n2, a.use_ip != 0, p.min_ctas, p.warp_mode);
    SearchArgs args = a;
    int vec = p.vec_codes;
    void* params[] = {&args, &pl, &vec};
    return cudaLaunchKernel(fn, dim3(p.grid), dim3(p.threads), params, p.smem_bytes, stream);
}

}  // namespace fg
