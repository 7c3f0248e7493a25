// fg_search.cu -- the one-CTA-per-query search kernel, the planner and the
// launchers (the planner hands batches of more than 4 queries per SM with a
// padded dimension <= 256 to the warp-per-query kernel, fg_search_warp.cu).
//
// One persistent kernel runs the reference's whole per-query search
// (SophiaSun18/FlashGANN src/adaptive_search.cuh:5-466): each CTA of NW warps
// pulls queries from an atomic counter and keeps the query's state in shared
// memory (beam, candidates, visited set, quantised query bit planes).
//
// Per iteration: visited-set reset/restore every SMALL_HASH_RESET_INTERVAL
// iterations -> beam merge -> control in warp 0 (k-th cutoff, adaptive
// controller, expander pick) -> expansion -> exact distances.  Compared with
// the reference's one-CTA-per-query loop (about 18 block barriers per
// iteration) this design:
//   * issues a parent's neighbour ids, RaBitQ factors and packed codes
//     together (128-bit code loads), for all parents a warp owns, before any
//     of them is examined: one dependent global round trip per expansion;
//   * in speculative iterations lets each warp evaluate the exact distances of
//     the children it kept right away, before the CTA-wide insert/compaction;
//   * runs the insert/compaction (first parent wins a shared child) in one
//     warp with __match_any_sync, and has that warp also sort the new
//     candidates and rank them against the beam for the next merge (for
//     beams <= 128 it performs the whole register merge there);
//   * merges ping-pong between two beam buffers;
//   * keeps the adaptive controller's state in warp-0 registers and picks
//     expanders from the first beam position that can hold an unexpanded
//     entry, prefetching the next likely parents' blocks into L2;
//   * needs 3 (beam <= 128) or 4 block barriers per speculative iteration.
#include <cfloat>
#include <cstdint>
#include <cstdio>
#include <cstdlib>

#include <cuda_runtime.h>

#include "fg_config.h"
#include "fg_device.cuh"
#include "fg_internal.h"

namespace fg {
namespace {

struct Plan {
    uint32_t padded, cbs, collect_cap;
    int hbits;
    float phase2_rho;
    int max_iter;
    int merge_n2;
    int mp_active;
    int lshift;  // log2 of the 128-byte lines per raw vector, rounded up
};

struct Smem {
    uint32_t* beam_idx;
    float* beam_dist;
    uint32_t* beam_idx2;   // merge path: the second beam buffer
    float* beam_dist2;
    uint32_t* cand_idx;
    float* cand_dist;
    uint32_t* hash;
    float* qvec;
    uint32_t* planes;
    uint32_t* wrap;
    uint8_t* quant;
    uint32_t* stage;       // kept children, SEARCH_WIDTH x 32
    float* stage_dist;     // their exact distances
    uint32_t* pos;         // merge path: stable positions of the candidates
    uint32_t* eval_slot;   // single-expander path: candidate slot of each evaluation
    uint32_t* eval_node;
    uint32_t* wlist;       // per warp: stage slots of the children it kept (NW x 32)
    float* rot;            // rotation scratch for D outside [32, 256]
};

// Values warp 0 publishes to the CTA each iteration.
struct Shared {
    int theta;
    float rho;
    float cutoff;
    uint32_t keep_exp;
    uint32_t p0;      // merge path: first beam position the pending merge can change
    uint32_t n_eval;
    uint32_t n_est;
    uint32_t query;
};

__host__ __device__ inline size_t align16(size_t x) { return (x + 15) & ~static_cast<size_t>(15); }

__host__ __device__ inline size_t smem_layout(uint32_t padded, int hbits, int dim, int D, int nw, bool mp, Smem* s,
                                              unsigned char* base) {
    size_t off = 0;
    auto take = [&](size_t bytes) {
        unsigned char* p = base ? base + off : nullptr;
        off += align16(bytes);
        return p;
    };
    unsigned char* p;
    p = take(padded * 4); if (s) s->beam_idx = reinterpret_cast<uint32_t*>(p);
    p = take(padded * 4); if (s) s->beam_dist = reinterpret_cast<float*>(p);
    p = take(mp ? padded * 4 : 0); if (s) s->beam_idx2 = reinterpret_cast<uint32_t*>(p);
    p = take(mp ? padded * 4 : 0); if (s) s->beam_dist2 = reinterpret_cast<float*>(p);
    p = take(32 * 4); if (s) s->cand_idx = reinterpret_cast<uint32_t*>(p);
    p = take(32 * 4); if (s) s->cand_dist = reinterpret_cast<float*>(p);
    p = take((size_t(1) << hbits) * 4); if (s) s->hash = reinterpret_cast<uint32_t*>(p);
    p = take(static_cast<size_t>(dim) * 4); if (s) s->qvec = reinterpret_cast<float*>(p);
    const int W = D / 32;
    p = take(static_cast<size_t>(kPlanes) * W * 4); if (s) s->planes = reinterpret_cast<uint32_t*>(p);
    p = take(static_cast<size_t>(W) * 4); if (s) s->wrap = reinterpret_cast<uint32_t*>(p);
    p = take(static_cast<size_t>(D)); if (s) s->quant = p;
    p = take(static_cast<size_t>(SEARCH_WIDTH) * 32 * 4); if (s) s->stage = reinterpret_cast<uint32_t*>(p);
    p = take(static_cast<size_t>(SEARCH_WIDTH) * 32 * 4); if (s) s->stage_dist = reinterpret_cast<float*>(p);
    p = take(32 * 4); if (s) s->pos = reinterpret_cast<uint32_t*>(p);
    p = take(32 * 4); if (s) s->eval_slot = reinterpret_cast<uint32_t*>(p);
    p = take(32 * 4); if (s) s->eval_node = reinterpret_cast<uint32_t*>(p);
    p = take(static_cast<size_t>(nw) * 32 * 4); if (s) s->wlist = reinterpret_cast<uint32_t*>(p);
    const bool warp_prep = D >= 32 && D <= 256;
    p = take(warp_prep ? 0 : static_cast<size_t>(D) * 4); if (s) s->rot = reinterpret_cast<float*>(p);
    return off;
}

// Exact distances of list entries first, first+STRIDE, ... (< n) in batches
// of kEvalBatch rows per warp; node(e) / write(e, d) supply and store them.
// lshift = log2 of the 128-byte lines per row rounded up to a power of two.
template <int STRIDE, typename NodeF, typename OutF>
__device__ __forceinline__ void eval_list(const SearchArgs& a, const float* qvec, int first, int n, int lshift,
                                          NodeF node, OutF write, int lane) {
    if (n <= first) return;
    const int cnt = (n - first + STRIDE - 1) / STRIDE;
    if (cnt > kEvalBatch) {
        // one L2 prefetch per lane per 128-byte line of every row this warp reads
        const int lpr = (a.dim * 4 + 127) >> 7;
        for (int j = lane; j < (cnt << lshift); j += 32) {
            const int line = j & ((1 << lshift) - 1);
            if (line < lpr) {
                const int e = first + (j >> lshift) * STRIDE;
                const char* p = reinterpret_cast<const char*>(a.rows + static_cast<uint64_t>(node(e)) * a.row) + line * 128;
                asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
            }
        }
    }
    for (int base = first; base < n; base += STRIDE * kEvalBatch) {
        uint32_t nodes[kEvalBatch];
        int cnt = 0;
#pragma unroll
        for (int b = 0; b < kEvalBatch; ++b) {
            const int e = base + b * STRIDE;
            nodes[b] = e < n ? node(e) : 0u;
            cnt += e < n;
        }
        float d[kEvalBatch];
        eval_rows<kEvalBatch>(a.rows, a.row, a.dim, qvec, nodes, cnt, a.use_ip, d, lane);
        if (lane == 0) {
#pragma unroll
            for (int b = 0; b < kEvalBatch; ++b)
                if (b < cnt) write(base + b * STRIDE, d[b]);
        }
    }
}

template <int NW, int W, int MERGE>
__device__ void search_one(const SearchArgs& a, const Plan& pl, const Smem& sm, Shared& sh, QueryState& qs,
                           uint32_t* s_pnode, float* s_pdist, uint32_t* s_stage_cnt, float* red_f, int* red_i,
                           const uint16_t* bnd, uint32_t qid, int vec_codes) {
    constexpr int kThreads = Cfg<NW>::kThreads;
    constexpr int kTPW = Cfg<NW>::kTasksPerWarp;
    constexpr bool mp = MERGE == 0;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int dim = a.dim, D = a.padded_dim, deg = a.degree, beam = a.beam;
    const uint32_t padded = pl.padded, cbs = pl.cbs;
    const int hbits = pl.hbits;
    const float* __restrict__ rows = a.rows;
    const uint64_t rowf = a.row;
    const bool vec = vec_codes != 0;
    uint32_t* bidx = sm.beam_idx;
    float* bdist = sm.beam_dist;
    uint32_t* oidx = sm.beam_idx2;
    float* odist = sm.beam_dist2;

    // ---------------------------------------------------------------- init
    const float* q = a.queries + static_cast<size_t>(qid) * dim;
    for (int i = tid; i < dim; i += kThreads) sm.qvec[i] = q[i];
    for (int i = tid; i < (1 << hbits); i += kThreads) sm.hash[i] = kMax;
    for (uint32_t i = tid; i < padded; i += kThreads) {
        bidx[i] = kMax;
        bdist[i] = FLT_MAX;
    }
    if (tid < 32) {
        sm.cand_idx[tid] = kMax;
        sm.cand_dist[tid] = FLT_MAX;
    }
    __syncthreads();
    uint32_t c_iters = 0, c_exp = 0, c_eval = 1;
    CtlRegs c;
    if (warp == 0) {
        // entry point into candidate slot 0 (src/adaptive_search.cuh:110-118)
        const float ed = warp_dist(rows + static_cast<uint64_t>(a.entry) * rowf, sm.qvec, dim, a.use_ip, lane);
        if (lane == 0) {
            sm.cand_idx[0] = a.entry;
            sm.cand_dist[0] = ed;
            h_insert(sm.hash, hbits, a.entry);
            sh.n_est = 0;
        }
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
    }
    const bool warp_prep = D >= 32 && D <= 256;
    if (warp_prep) {
        if (warp == (NW > 1 ? 1 : 0)) {
            if constexpr (W >= 1 && W <= 8) {
                prep_warp<W>(sm.qvec, a.signs, dim, sm.quant, nullptr, &qs, lane);
            } else {
                switch (D) {
                    case 32: prep_warp<1>(sm.qvec, a.signs, dim, sm.quant, nullptr, &qs, lane); break;
                    case 64: prep_warp<2>(sm.qvec, a.signs, dim, sm.quant, nullptr, &qs, lane); break;
                    case 128: prep_warp<4>(sm.qvec, a.signs, dim, sm.quant, nullptr, &qs, lane); break;
                    default: prep_warp<8>(sm.qvec, a.signs, dim, sm.quant, nullptr, &qs, lane); break;
                }
            }
            build_planes(sm.quant, D, sm.planes, sm.wrap, &qs, lane);
        }
    } else {
        prep_block<NW>(sm.qvec, a.signs, dim, D, sm.rot, sm.quant, &qs, red_f, red_i);
        if (warp == 0) build_planes(sm.quant, D, sm.planes, sm.wrap, &qs, lane);
    }
    __syncthreads();
    const QueryState qsl = qs;

    // pending candidates already ranked against the beam (merge path) or
    // already merged (register merge) by the previous iteration's compaction
    bool prepared = false;
    bool merged = false;

    // ---------------------------------------------------------------- loop
    for (int iter = 0; iter < MAX_ITERATIONS; ++iter) {
        __syncthreads();  // the previous iteration is complete
        if ((iter + 1) % SMALL_HASH_RESET_INTERVAL == 0) {
            // src/adaptive_search.cuh:129-133
            for (int i = tid; i < (1 << hbits); i += kThreads) sm.hash[i] = kMax;
            __syncthreads();
            for (int i = tid; i < beam; i += kThreads) h_insert(sm.hash, hbits, bidx[i] & ~kMsb);
            __syncthreads();
        }
        if (iter >= pl.max_iter) break;

        // merge the previous iteration's candidates into the beam (:142-145)
        if constexpr (mp) {
            if (!prepared) {
                if (warp == 0) mp_prepare(bdist, sm.cand_idx, sm.cand_dist, cbs, padded, sm.pos, &sh.p0, lane);
                __syncthreads();
            }
            mp_apply<NW>(bidx, bdist, oidx, odist, sm.cand_idx, sm.cand_dist, cbs, padded, pl.mp_active, bnd, sm.pos,
                         sh.p0);
            uint32_t* ti = bidx; bidx = oidx; oidx = ti;
            float* td = bdist; bdist = odist; odist = td;
            prepared = false;
            __syncthreads();
        } else {
            if (warp == 0 && !merged) merge_bitonic<MERGE>(bidx, bdist, sm.cand_idx, sm.cand_dist, cbs, iter == 0, lane);
            merged = false;
        }
        ++c_iters;

        // control in warp 0 (src/adaptive_search.cuh:147-217)
        if (warp == 0) {
            if constexpr (!mp) {
                for (uint32_t i = static_cast<uint32_t>(beam) + lane; i < padded; i += 32) {
                    bidx[i] = kMax;
                    bdist[i] = FLT_MAX;
                }
                __syncwarp();
            }
            const float cutoff = bidx[beam - 1] == kMax ? FLT_MAX : bdist[(a.K < beam ? a.K : beam) - 1];
            if (lane < static_cast<int>(cbs)) {
                sm.cand_idx[lane] = kMax;
                sm.cand_dist[lane] = FLT_MAX;
            }
            controller_update(c, bidx[0], iter, pl.phase2_rho);
            uint32_t start = 0;
            if constexpr (mp) {
                // entries before the merge's first change are still expanded
                if (sh.p0 < c.scan) c.scan = sh.p0;
                start = c.scan & ~31u;
            }
            // pick_expanders (include/utils.cuh:752-787)
            const uint32_t theta = static_cast<uint32_t>(c.theta);
            uint32_t num = 0, last_pick = 0;
            const uint32_t lim = (static_cast<uint32_t>(beam) + 31u) & ~31u;
            uint32_t j0 = start;
            for (; j0 < lim; j0 += 32) {
                const uint32_t j = j0 + lane;
                uint32_t e = 0;
                const bool np = j < static_cast<uint32_t>(beam) && ((e = bidx[j]) & kMsb) == 0;
                const uint32_t b = __ballot_sync(kFull, np);
                const uint32_t i = __popc(b & lanemask_lt(lane)) + num;
                if (np && i < theta) {
                    s_pnode[i] = e & 0x7fffffffu;
                    s_pdist[i] = bdist[j];
                    bidx[j] = e | kMsb;
                }
                if (num + __popc(b) >= theta) {
                    // position of the theta-th pick: lane holding rank theta-1
                    const uint32_t sel = __ballot_sync(kFull, np && i == theta - 1);
                    last_pick = j0 + (__ffs(sel) - 1);
                    num = theta;
                    // prefetch the blocks of the next unexpanded entries of this chunk
                    const uint32_t later = b & ~((sel << 1) - 1u);
                    if ((later >> lane) & 1u) {
                        const char* blk = reinterpret_cast<const char*>(rows + static_cast<uint64_t>(e & 0x7fffffffu) * rowf +
                                                                        a.code_off);
#pragma unroll
                        for (int l = 0; l < 8; ++l) asm volatile("prefetch.global.L2 [%0];" ::"l"(blk + 128 * l));
                    }
                    break;
                }
                num += __popc(b);
            }
            __syncwarp();
            if constexpr (mp) c.scan = num == theta ? last_pick + 1 : static_cast<uint32_t>(beam);
            if (num) {
                // record_selected_expander_dist (adaptive_search_utils.cuh:41-49)
                c.last_d = finite_lt_max(c.cur_d) ? c.cur_d : c.entry_d;
                c.cur_d = s_pdist[num - 1];
            }
            if (lane == 0) {
                sh.keep_exp = num;
                sh.theta = c.theta;
                sh.rho = c.rho;
                sh.cutoff = cutoff;
            }
            if (a.trace && iter < a.trace_cap) {
                const size_t base = static_cast<size_t>(qid) * a.trace_cap + iter;
                if (lane < SEARCH_WIDTH) a.trace[base * SEARCH_WIDTH + lane] = lane < static_cast<int>(num) ? s_pnode[lane] : kMax;
                if (lane == 0) a.trace_count[base] = static_cast<int32_t>(num);
            }
        }
        __syncthreads();
        const uint32_t keep_exp = sh.keep_exp;
        if (!keep_exp) break;
        c_exp += keep_exp;
        const int theta = sh.theta;
        const float rho = sh.rho;
        const float cutoff = sh.cutoff;
        const bool cut_ok = isfinite(cutoff) && cutoff < FLT_MAX;

        if (!(theta > 1)) {
            // ------------------------ single expander (src/adaptive_search.cuh:221-343)
            if (warp == 0) {
                const uint32_t work = static_cast<uint32_t>(deg) < cbs ? static_cast<uint32_t>(deg) : cbs;
                const float* prow = rows + static_cast<uint64_t>(s_pnode[0]) * rowf;
                ParentLane<W> p;
                load_parent<W>(prow, a, static_cast<int>(work), vec, lane, p);
                const bool in_work = static_cast<uint32_t>(lane) < work;
                uint32_t child = p.child;
                if (child != kMax && (child >= a.n || h_contains(sm.hash, hbits, child))) child = kMax;
                float dist = child == kMax ? FLT_MAX : 0.0f;
                const int keep = keep_for(work, theta, rho, false, 0);
                const uint32_t vcount = __popc(__ballot_sync(kFull, in_work && child != kMax));
                const bool keep_all = keep >= static_cast<int>(vcount);
                int admit = static_cast<int>(work);
                if (!keep_all) {
                    if (child != kMax) {
                        // theta = 1 variant: triple_x == FLT_MAX estimates 0.0 (include/utils.cuh:951-952)
                        float est = 0.0f;
                        if (p.tx != FLT_MAX) {
                            const uint32_t raw = parent_raw<W>(p, prow, a, lane, sm.planes, sm.wrap, qsl.wrap_any);
                            est = estimate(raw, p.tx, p.fdq, p.fvq, s_pdist[0], qsl);
                        }
                        if (isfinite(est)) {
                            dist = est;
                        } else {
                            dist = FLT_MAX;
                            child = kMax;
                        }
                    }
                    if (lane == 0) sh.n_est += vcount;
                    const uint32_t near = cut_ok ? __popc(__ballot_sync(kFull, in_work && child != kMax && isfinite(dist) && dist <= cutoff)) : 0u;
                    const int eff = keep_for(work, theta, rho, cut_ok, near);
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
                const bool ins = first && h_insert(sm.hash, hbits, child);
                if (lane < static_cast<int>(cbs)) {
                    sm.cand_idx[lane] = ins ? child : kMax;
                    sm.cand_dist[lane] = FLT_MAX;
                }
                const uint32_t ib = __ballot_sync(kFull, ins);
                if (ins) {
                    const uint32_t r = __popc(ib & lanemask_lt(lane));
                    sm.eval_slot[r] = lane;
                    sm.eval_node[r] = child;
                }
                if (lane == 0) sh.n_eval = __popc(ib);
            }
            __syncthreads();
            const int ne = static_cast<int>(sh.n_eval);
            c_eval += ne;
            eval_list<NW>(a, sm.qvec, warp, ne, pl.lshift, [&](int e) { return sm.eval_node[e]; },
                          [&](int e, float d) { sm.cand_dist[sm.eval_slot[e]] = d; }, lane);
        } else {
            // ------------------- speculative expanders (src/adaptive_search.cuh:344-444)
            // degree <= 32: one neighbour tile per parent; every lookup of the
            // iteration happens before its inserts.
            const uint32_t active = static_cast<uint32_t>(deg) < 32u ? static_cast<uint32_t>(deg) : 32u;
            ParentLane<W> pr[kTPW];
#pragma unroll
            for (int k = 0; k < kTPW; ++k) {
                const int t = warp + k * NW;
                if (t < static_cast<int>(keep_exp))
                    load_parent<W>(rows + static_cast<uint64_t>(s_pnode[t]) * rowf, a, deg, vec, lane, pr[k]);
            }
            int nkept = 0;
#pragma unroll
            for (int k = 0; k < kTPW; ++k) {
                const int t = warp + k * NW;
                if (t >= static_cast<int>(keep_exp)) break;
                const float* prow = rows + static_cast<uint64_t>(s_pnode[t]) * rowf;
                const uint32_t child = pr[k].child;
                bool valid = child != kMax && child < a.n && !h_contains(sm.hash, hbits, child);
                const int keep = keep_for(active, theta, rho, false, 0);
                const uint32_t raw_valid = __popc(__ballot_sync(kFull, valid));
                const bool keep_all = keep >= static_cast<int>(raw_valid);
                bool kl;
                if (keep_all) {
                    kl = valid;
                } else {
                    float est = FLT_MAX;
                    if (valid) {
                        // speculative variant: triple_x == FLT_MAX estimates FLT_MAX
                        if (pr[k].tx != FLT_MAX) {
                            const uint32_t raw = parent_raw<W>(pr[k], prow, a, lane, sm.planes, sm.wrap, qsl.wrap_any);
                            est = estimate(raw, pr[k].tx, pr[k].fdq, pr[k].fvq, s_pdist[t], qsl);
                        }
                        valid = isfinite(est);
                    }
                    if (lane == 0) atomicAdd(&sh.n_est, raw_valid);
                    const uint32_t near = __popc(__ballot_sync(kFull, valid && cut_ok && est <= cutoff));
                    const int eff = keep_for(active, theta, rho, cut_ok, near);
                    kl = keep_smallest(est, valid, eff, lane);
                }
                const uint32_t kb = __ballot_sync(kFull, kl);
                if (kl) {
                    const uint32_t r = __popc(kb & lanemask_lt(lane));
                    sm.stage[t * 32 + r] = child;
                    sm.wlist[warp * 32 + nkept + r] = t * 32 + r;
                }
                if (lane == 0) s_stage_cnt[t] = __popc(kb);
                nkept += __popc(kb);
            }
            __syncwarp();
            // exact distances of this warp's kept children, before the barrier
            eval_list<1>(a, sm.qvec, 0, nkept, pl.lshift, [&](int e) { return sm.stage[sm.wlist[warp * 32 + e]]; },
                         [&](int e, float d) { sm.stage_dist[sm.wlist[warp * 32 + e]] = d; }, lane);
            __syncthreads();
            if (warp == 0) {
                // inserts and compaction in (parent, lane) order; a child kept by
                // two parents goes to the first (include/utils.cuh:187-214)
                const uint32_t cnt = lane < static_cast<int>(keep_exp) ? s_stage_cnt[lane] : 0u;
                uint32_t incl = cnt;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t y = __shfl_up_sync(kFull, incl, o);
                    if (lane >= o) incl += y;
                }
                const uint32_t total = __shfl_sync(kFull, incl, 31);
                uint32_t compact = 0;
                for (uint32_t base = 0; base < total; base += 32) {
                    const uint32_t e = base + lane;
                    uint32_t child = kMax, slot_in = 0;
                    // parent of entry e: the number of parents whose inclusive count is <= e
                    uint32_t t = 0, before = 0;
                    for (uint32_t p = 0; p < keep_exp; ++p) {
                        const uint32_t ip = __shfl_sync(kFull, incl, p);
                        if (ip <= e) {
                            t = p + 1;
                            before = ip;
                        }
                    }
                    if (e < total) {
                        slot_in = t * 32 + (e - before);
                        child = sm.stage[slot_in];
                    }
                    const uint32_t same = __match_any_sync(kFull, child);
                    const bool first = child != kMax && (__ffs(same) - 1) == lane;
                    const bool ins = first && h_insert(sm.hash, hbits, child);
                    const uint32_t ib = __ballot_sync(kFull, ins);
                    if (ins) {
                        const uint32_t slot = compact + __popc(ib & lanemask_lt(lane));
                        if (slot < pl.collect_cap) {
                            sm.cand_idx[slot] = child;
                            sm.cand_dist[slot] = sm.stage_dist[slot_in];
                        }
                    }
                    compact += __popc(ib);
                }
                // counted by thread 0, which writes the statistics
                c_eval += compact < pl.collect_cap ? compact : pl.collect_cap;
                __syncwarp();
                // get the next merge ready while the other warps wait at the barrier
                if constexpr (mp) {
                    mp_prepare(bdist, sm.cand_idx, sm.cand_dist, cbs, padded, sm.pos, &sh.p0, lane);
                } else if ((iter + 2) % SMALL_HASH_RESET_INTERVAL != 0) {
                    // not before a visited-set reset, which must restore the unmerged beam
                    merge_bitonic<MERGE>(bidx, bdist, sm.cand_idx, sm.cand_dist, cbs, false, lane);
                    if (lane < static_cast<int>(cbs)) {
                        sm.cand_idx[lane] = kMax;
                        sm.cand_dist[lane] = FLT_MAX;
                    }
                    merged = true;
                }
            }
            if constexpr (mp) prepared = true;
        }
    }
    // final merge (src/adaptive_search.cuh:448-452)
    __syncthreads();
    if constexpr (mp) {
        if (!prepared) {
            if (warp == 0) mp_prepare(bdist, sm.cand_idx, sm.cand_dist, cbs, padded, sm.pos, &sh.p0, lane);
            __syncthreads();
        }
        mp_apply<NW>(bidx, bdist, oidx, odist, sm.cand_idx, sm.cand_dist, cbs, padded, pl.mp_active, bnd, sm.pos, sh.p0);
        uint32_t* ti = bidx; bidx = oidx; oidx = ti;
        float* td = bdist; bdist = odist; odist = td;
    } else if (warp == 0) {
        merge_bitonic<MERGE>(bidx, bdist, sm.cand_idx, sm.cand_dist, cbs, false, lane);
    }
    __syncthreads();
    // results (:455-464): position i < beam holds the beam entry with its MSB
    // cleared; positions >= beam repeat the last one
    for (int i = tid; i < a.K; i += kThreads) {
        const int s = i < beam ? i : beam - 1;
        a.out_ids[static_cast<size_t>(qid) * a.K + i] = bidx[s] & 0x7fffffffu;
        if (a.out_dists) a.out_dists[static_cast<size_t>(qid) * a.K + i] = bdist[s];
    }
    if (tid == 0 && a.stats) {
        fg_query_stats st;
        st.iterations = c_iters;
        st.expansions = c_exp;
        st.evaluations = c_eval;
        st.estimates = sh.n_est;
        a.stats[qid] = st;
    }
    __syncthreads();
}

template <int NW, int MINB, int W, int MERGE>
__global__ void __launch_bounds__(NW * 32, MINB) search_kernel(const SearchArgs a, const Plan pl, int vec_codes) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ Shared sh;
    __shared__ QueryState qs;
    __shared__ uint32_t s_pnode[SEARCH_WIDTH];
    __shared__ float s_pdist[SEARCH_WIDTH];
    __shared__ uint32_t s_stage_cnt[SEARCH_WIDTH];
    __shared__ float red_f[2 * NW];
    __shared__ int red_i[NW];
    // merge-path output segment boundaries s * itopk / active (launch constants)
    __shared__ uint16_t bnd[MERGE == 0 ? BLOCK_SIZE + 1 : 1];
    if constexpr (MERGE == 0) {
        for (int s = threadIdx.x; s <= pl.mp_active; s += NW * 32)
            bnd[s] = static_cast<uint16_t>((static_cast<uint32_t>(s) * pl.padded) / static_cast<uint32_t>(pl.mp_active));
    }
    Smem sm;
    smem_layout(pl.padded, pl.hbits, a.dim, a.padded_dim, NW, MERGE == 0, &sm, smem_raw);
    for (;;) {
        if (threadIdx.x == 0) sh.query = atomicAdd(a.work_counter, 1u);
        __syncthreads();
        const uint32_t qid = sh.query;
        __syncthreads();
        if (qid >= static_cast<uint32_t>(a.nq)) break;
        search_one<NW, W, MERGE>(a, pl, sm, sh, qs, s_pnode, s_pdist, s_stage_cnt, red_f, red_i, bnd, qid, vec_codes);
    }
}

// ------------------------------------------------ standalone query prepare
constexpr int kAuxWarps = 4;

__global__ void __launch_bounds__(kAuxWarps * 32) query_prepare_kernel(const float* queries, int nq, int dim, int D,
                                                                       const float* signs, float* rotated,
                                                                       uint8_t* quant_out, uint8_t* lut, float* factors,
                                                                       int32_t* sum_q) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ QueryState qs;
    __shared__ float red_f[2 * kAuxWarps];
    __shared__ int red_i[kAuxWarps];
    float* qvec = reinterpret_cast<float*>(smem_raw);
    float* rot = qvec + align16(dim * 4) / 4;
    uint8_t* quant = reinterpret_cast<uint8_t*>(rot + D);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int q = blockIdx.x; q < nq; q += gridDim.x) {
        for (int i = tid; i < dim; i += blockDim.x) qvec[i] = queries[static_cast<size_t>(q) * dim + i];
        __syncthreads();
        const bool warp_prep = D >= 32 && D <= 256;
        if (warp_prep) {
            if (warp == 0) {
                switch (D) {
                    case 32: prep_warp<1>(qvec, signs, dim, quant, rot, &qs, lane); break;
                    case 64: prep_warp<2>(qvec, signs, dim, quant, rot, &qs, lane); break;
                    case 128: prep_warp<4>(qvec, signs, dim, quant, rot, &qs, lane); break;
                    default: prep_warp<8>(qvec, signs, dim, quant, rot, &qs, lane); break;
                }
            }
            __syncthreads();
        } else {
            prep_block<kAuxWarps>(qvec, signs, dim, D, rot, quant, &qs, red_f, red_i);
        }
        if (rotated)
            for (int i = tid; i < D; i += blockDim.x) rotated[static_cast<size_t>(q) * D + i] = rot[i];
        if (quant_out)
            for (int i = tid; i < D; i += blockDim.x) quant_out[static_cast<size_t>(q) * D + i] = quant[i];
        if (lut) {
            // the reference's 16-entry nibble LUT (include/utils.cuh:909-917), for checking
            for (int cb = tid; cb < (D >> 2); cb += blockDim.x) {
                uint8_t* c = lut + static_cast<size_t>(q) * 4 * D + (cb << 4);
                for (int m = 0; m < 16; ++m) {
                    uint32_t s = 0;
                    if (m & 8) s += quant[4 * cb];
                    if (m & 4) s += quant[4 * cb + 1];
                    if (m & 2) s += quant[4 * cb + 2];
                    if (m & 1) s += quant[4 * cb + 3];
                    c[m] = static_cast<uint8_t>(s);
                }
            }
        }
        if (tid == 0) {
            factors[q * 3 + 0] = qs.low;
            factors[q * 3 + 1] = qs.high;
            factors[q * 3 + 2] = qs.width;
            if (sum_q) sum_q[q] = qs.sum_q;
        }
        __syncthreads();
    }
}

// ------------------------------------------------------ merge test kernel
__global__ void __launch_bounds__(kAuxWarps * 32) beam_merge_kernel(uint32_t* idx, float* dist, int itopk, int cbs,
                                                                    int first, int merge_n2, int active) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ uint32_t p0;
    __shared__ uint16_t bnd[BLOCK_SIZE + 1];
    const int total = itopk + cbs;
    uint32_t* sidx = reinterpret_cast<uint32_t*>(smem_raw);
    float* sdist = reinterpret_cast<float*>(sidx + total);
    uint32_t* pos = reinterpret_cast<uint32_t*>(sdist + total);
    uint32_t* oidx = pos + 32;
    float* odist = reinterpret_cast<float*>(oidx + itopk);
    const size_t off = static_cast<size_t>(blockIdx.x) * total;
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
        sidx[i] = idx[off + i];
        sdist[i] = dist[off + i];
    }
    for (int s = threadIdx.x; s <= active; s += blockDim.x)
        bnd[s] = static_cast<uint16_t>((static_cast<uint32_t>(s) * itopk) / static_cast<uint32_t>(active));
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t* ridx = sidx;
    const float* rdist = sdist;
    if (merge_n2 == 0) {
        if (warp == 0) mp_prepare(sdist, sidx + itopk, sdist + itopk, cbs, itopk, pos, &p0, lane);
        __syncthreads();
        mp_apply<kAuxWarps>(sidx, sdist, oidx, odist, sidx + itopk, sdist + itopk, cbs, itopk, active, bnd, pos, p0);
        ridx = oidx;
        rdist = odist;
    } else if (warp == 0) {
        if (merge_n2 == 1) merge_bitonic<1>(sidx, sdist, sidx + itopk, sdist + itopk, cbs, first != 0, lane);
        else if (merge_n2 == 2) merge_bitonic<2>(sidx, sdist, sidx + itopk, sdist + itopk, cbs, first != 0, lane);
        else merge_bitonic<4>(sidx, sdist, sidx + itopk, sdist + itopk, cbs, first != 0, lane);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < itopk; i += blockDim.x) {
        idx[off + i] = ridx[i];
        dist[off + i] = rdist[i];
    }
}

// ---------------------------------------------------------- kernel variants
// (warps per query, minimum resident CTAs per SM for the register budget)
struct Variant {
    int nw, minb;
};
constexpr Variant kVariants[] = {{8, 4}, {4, 8}, {8, 5}, {4, 10}};
constexpr int kNumVariants = sizeof(kVariants) / sizeof(kVariants[0]);
constexpr int kDefaultVariant = 0;

template <int NW, int MINB, int W>
const void* pick_merge(int merge) {
    switch (merge) {
        case 1: return reinterpret_cast<const void*>(search_kernel<NW, MINB, W, 1>);
        case 2: return reinterpret_cast<const void*>(search_kernel<NW, MINB, W, 2>);
        case 4: return reinterpret_cast<const void*>(search_kernel<NW, MINB, W, 4>);
        default: return reinterpret_cast<const void*>(search_kernel<NW, MINB, W, 0>);
    }
}

template <int NW, int MINB>
const void* pick_w(int W, int merge) {
    return W == 4 ? pick_merge<NW, MINB, 4>(merge) : pick_merge<NW, MINB, 0>(merge);
}

const void* kernel_for(int variant, int W, int merge) {
    switch (variant) {
        case 0: return pick_w<8, 4>(W, merge);
        case 1: return pick_w<4, 8>(W, merge);
        case 2: return pick_w<8, 5>(W, merge);
        default: return pick_w<4, 10>(W, merge);
    }
}

int variant_from_env() {
    const char* v = getenv("FG_KERNEL_VARIANT");
    if (!v || !*v) return kDefaultVariant;
    const int x = atoi(v);
    return (x >= 0 && x < kNumVariants) ? x : kDefaultVariant;
}

// Kernel choice where all apply (padded dim <= 256; they return identical
// results), by queries per SM, from batch sweeps on a B200.  For the
// shortest time of one batch (FG_GOAL_LATENCY): up to 4 the CTA kernel (8
// warps per query: the shortest time per query), up to what the pair mode
// holds resident (10) the warp kernel's pair mode (2 warps per query), above
// that one warp per query (20 resident queries per SM at beam <= 640 and
// D = 128).  For batches kept in flight on several streams
// (FG_GOAL_THROUGHPUT) each batch shares the SMs with the next one: the pair
// mode while two batches are resident at once, one warp per query above
// (c2_1m, beam 640, two streams: 592 queries 0.95 ms per batch in the pair
// mode against 1.36 in the CTA kernel, 1,250 queries 1.45 ms with one warp per
// query against 1.55 in the pair mode).  FG_KERNEL=cta, =pair, =warp or
// =staged (the warp kernel's staged variant) forces one.
enum class Choice { kCta, kWarp, kStaged, kPair, kAuto };

Choice kernel_choice(int nq, int device, int goal) {
    const char* v = getenv("FG_KERNEL");
    if (v && v[0] == 'c') return Choice::kCta;
    if (v && v[0] == 'w') return Choice::kWarp;
    if (v && v[0] == 's') return Choice::kStaged;
    if (v && v[0] == 'p') return Choice::kPair;
    if (goal == FG_GOAL_THROUGHPUT) return Choice::kAuto;
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) sms = 148;
    return nq > 4 * sms ? Choice::kAuto : Choice::kCta;
}

int merge_width(uint32_t itopk) {
    uint32_t n2 = (itopk + 31) / 32;
    if (n2 > 32) n2 = 4;
    return (itopk % 32 == 0 && (n2 == 1 || n2 == 2 || n2 == 4)) ? static_cast<int>(n2) : 0;
}

int merge_active(uint32_t itopk) {
    int active = static_cast<int>((itopk + 3) / 4);
    active = ((active + 31) / 32) * 32;
    return active < BLOCK_SIZE ? active : BLOCK_SIZE;
}

}  // namespace

// --------------------------------------------------------------- host side
uint32_t effective_sort_beam(uint32_t beam) {
    if (beam == 0) return 0;
    uint32_t r = 1;
    while (r < beam) r <<= 1;
    if (r <= 128) return r < 32 ? 32 : r;
    return beam;
}

uint32_t candidate_buffer_size(int degree) {
    uint32_t cap = BUFFER_BOUND;
    const uint32_t mx = static_cast<uint32_t>(THETA_MAX) * static_cast<uint32_t>(degree);
    if (cap > mx) cap = mx;
    uint32_t r = 1;
    while (r < cap) r <<= 1;
    return r;
}

// Visited-table bits: the reference's load rule (include/utils.cuh:137-151)
// from a floor of 2^FG_HASH_BASE_BITLEN slots.
int hash_bits(uint32_t padded, uint32_t cbs) {
    const uint64_t req = static_cast<uint64_t>(padded) + static_cast<uint64_t>(cbs) * SMALL_HASH_RESET_INTERVAL;
    const uint64_t target = (req * 4 + 2) / 3;
    int b = FG_HASH_BASE_BITLEN;
    while ((uint64_t(1) << b) < target) ++b;
    return b;
}

int plan_search(const SearchArgs& a, SearchPlan* p, int device, char* err, size_t errlen) {
    if (a.degree < 1 || a.degree > FG_MAX_DEGREE) {
        snprintf(err, errlen, "degree %d outside the supported range [1, %d]", a.degree, FG_MAX_DEGREE);
        return FG_ERR_UNSUPPORTED;
    }
    if (a.beam < 1 || a.beam > FG_MAX_BEAM) {
        snprintf(err, errlen, "beam %d outside the supported range [1, %d]", a.beam, FG_MAX_BEAM);
        return FG_ERR_UNSUPPORTED;
    }
    if (a.K < 1) {
        snprintf(err, errlen, "K must be >= 1 (got %d)", a.K);
        return FG_ERR_ARG;
    }
    if (a.dim < 32 || a.dim > FG_MAX_DIM) {
        snprintf(err, errlen, "dim %d outside the supported range [32, %d]", a.dim, FG_MAX_DIM);
        return FG_ERR_UNSUPPORTED;
    }
    p->padded = effective_sort_beam(static_cast<uint32_t>(a.beam));
    p->cbs = candidate_buffer_size(a.degree);
    p->collect_cap = BUFFER_BOUND < p->cbs ? BUFFER_BOUND : p->cbs;
    p->hbits = hash_bits(p->padded, p->cbs);
    p->phase2_rho = (static_cast<uint32_t>(a.degree) <= static_cast<uint32_t>(MIN_PHASE2_KEEP))
                        ? RHO_MIN
                        : 1.0f - static_cast<float>(MIN_PHASE2_KEEP) / static_cast<float>(a.degree);
    p->max_iter = (a.beam * 11 + 9) / 10;
    p->merge_n2 = merge_width(p->padded);
    p->mp_active = merge_active(p->padded);
    const uintptr_t base = reinterpret_cast<uintptr_t>(a.rows);
    p->vec_codes = ((base % 16) == 0 && ((a.row * 4) % 16) == 0 && ((a.code_off * 4) % 16) == 0) ? 1 : 0;
    if (warp_kernel_supports(a.padded_dim)) {
        const Choice c = kernel_choice(a.nq, device, a.goal);
        if (c == Choice::kAuto) {
            // the pair mode while the whole batch (two batches, for throughput) is resident at
            // once, else one warp per query (a pair-mode shape that does not fit, e.g. under
            // FG_CTA_WARPS=1, also falls back)
            const int rc = plan_search_warp(a, p, device, err, errlen, 2);
            const long long need = a.goal == FG_GOAL_THROUGHPUT ? 2LL * a.nq : static_cast<long long>(a.nq);
            if (rc == FG_OK && need <= p->resident_queries) return rc;
            return plan_search_warp(a, p, device, err, errlen, 0);
        }
        if (c != Choice::kCta)
            return plan_search_warp(a, p, device, err, errlen, c == Choice::kStaged ? 1 : c == Choice::kPair ? 2 : 0);
    }
    p->kernel = 0;
    p->variant = variant_from_env();
    const int nw = kVariants[p->variant].nw;
    p->smem_bytes = smem_layout(p->padded, p->hbits, a.dim, a.padded_dim, nw, p->merge_n2 == 0, nullptr, nullptr);
    p->threads = nw * 32;
    int sms = 0;
    cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) {
        snprintf(err, errlen, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
        return FG_ERR_CUDA;
    }
    int max_smem = 0;
    cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    if (p->smem_bytes > static_cast<size_t>(max_smem)) {
        snprintf(err, errlen, "shared memory %zu exceeds the device limit %d", p->smem_bytes, max_smem);
        return FG_ERR_UNSUPPORTED;
    }
    const void* fn = kernel_for(p->variant, a.padded_dim / 32, p->merge_n2);
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(p->smem_bytes));
    if (e != cudaSuccess) {
        snprintf(err, errlen, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        return FG_ERR_CUDA;
    }
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, p->threads, p->smem_bytes);
    if (e != cudaSuccess || per_sm < 1) {
        snprintf(err, errlen, "occupancy query failed: %s", cudaGetErrorString(e));
        return FG_ERR_CUDA;
    }
    p->blocks_per_sm = per_sm;
    const int resident = per_sm * sms;
    p->grid = a.nq < resident ? a.nq : resident;
    if (p->grid < 1) p->grid = 1;
    return FG_OK;
}

cudaError_t launch_search(const SearchArgs& a, const SearchPlan& p, cudaStream_t stream) {
    if (p.kernel == 1) return launch_search_warp(a, p, stream);
    Plan pl;
    pl.padded = p.padded;
    pl.cbs = p.cbs;
    pl.collect_cap = p.collect_cap;
    pl.hbits = p.hbits;
    pl.phase2_rho = p.phase2_rho;
    pl.max_iter = p.max_iter;
    pl.merge_n2 = p.merge_n2;
    pl.mp_active = p.mp_active;
    const int lpr = (a.dim * 4 + 127) / 128;
    pl.lshift = 0;
    while ((1 << pl.lshift) < lpr) ++pl.lshift;
    cudaError_t e = cudaMemsetAsync(a.work_counter, 0, sizeof(uint32_t), stream);
    if (e != cudaSuccess) return e;
    const void* fn = kernel_for(p.variant, a.padded_dim / 32, p.merge_n2);
    SearchArgs args = a;
    int vec = p.vec_codes;
    void* params[] = {&args, &pl, &vec};
    return cudaLaunchKernel(fn, dim3(p.grid), dim3(p.threads), params, p.smem_bytes, stream);
}

cudaError_t launch_query_prepare(const float* queries, int nq, int dim, const float* signs, float* rotated,
                                 uint8_t* quant, uint8_t* lut, float* factors, int32_t* sum_q, cudaStream_t stream) {
    int D = 1;
    while (D < dim) D <<= 1;
    const size_t sm = align16(static_cast<size_t>(dim) * 4) + static_cast<size_t>(D) * 4 + D;
    if (sm > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(query_prepare_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(sm));
        if (e != cudaSuccess) return e;
    }
    const int grid = nq < 4096 ? nq : 4096;
    if (grid < 1) return cudaSuccess;
    query_prepare_kernel<<<grid, kAuxWarps * 32, sm, stream>>>(queries, nq, dim, D, signs, rotated, quant, lut, factors,
                                                               sum_q);
    return cudaGetLastError();
}

cudaError_t launch_beam_merge(uint32_t* idx, float* dist, int ncase, int itopk, int cbs, int first, cudaStream_t stream) {
    if (ncase < 1) return cudaSuccess;
    const size_t sm = static_cast<size_t>(itopk + cbs) * 8 + 32 * 4 + static_cast<size_t>(itopk) * 8;
    if (sm > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(beam_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(sm));
        if (e != cudaSuccess) return e;
    }
    beam_merge_kernel<<<ncase, kAuxWarps * 32, sm, stream>>>(idx, dist, itopk, cbs, first,
                                                              merge_width(static_cast<uint32_t>(itopk)),
                                                              merge_active(static_cast<uint32_t>(itopk)));
    return cudaGetLastError();
}

}  // namespace fg
