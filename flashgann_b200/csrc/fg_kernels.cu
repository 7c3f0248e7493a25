// fg_kernels.cu -- the B200 search path: query preparation, beam search with
// RaBitQ-pruned expansion and the adaptive controller, all in one persistent
// kernel (one CTA of FG_WARPS_PER_QUERY warps per query in flight).
//
// What is computed is the reference's search (SophiaSun18/FlashGANN,
// src/adaptive_search.cuh:5-466 and the helpers it calls); how it is computed
// is this file's own design:
//   * persistent CTAs pull queries from an atomic counter instead of one CTA
//     per query;
//   * all per-query state lives in shared memory, but the iteration uses about
//     a third of the reference's block barriers: control (controller, expander
//     pick) runs warp-synchronously in warp 0, each warp scans whole parent
//     lists, and the candidate insert/compaction runs in one warp;
//   * a parent's neighbour ids, factors and packed codes are loaded together
//     (128-bit code loads) as soon as the parent is known;
//   * RaBitQ estimates use bit-plane popcounts of the quantised query instead
//     of the byte LUT walk; the integer sums are identical (including the
//     uint8 wrap of the reference LUT, which is corrected for explicitly);
//   * exact distances issue every load of a warp's candidates before reducing,
//     keeping the reference's lane-strided fused accumulation order and
//     shuffle tree so float results are bit-identical;
//   * the merge-path beam merge computes the reference's segment partitions
//     from stable ranks and only runs the reference's binary search at
//     boundaries where a beam entry ties a candidate.
// Every float operation whose rounding matters is spelled out with __f*_rn
// intrinsics so the compiler cannot contract it differently.
#include <cfloat>
#include <cstdint>
#include <cstdio>

#include <cuda_runtime.h>

#include "fg_config.h"
#include "fg_internal.h"

namespace fg {
namespace {

constexpr uint32_t kMax = 0xFFFFFFFFu;
constexpr uint32_t kMsb = 0x80000000u;
constexpr unsigned kFull = 0xFFFFFFFFu;
constexpr int kPlanes = 7;  // quantised query values are in [0, 64]
constexpr int kNW = FG_WARPS_PER_QUERY;
constexpr int kThreads = kNW * 32;
// merge-path segments per thread: at most ceil(256 / threads) (BLOCK_SIZE caps segments)
constexpr int kMaxSegPerThread = (BLOCK_SIZE + kThreads - 1) / kThreads;
constexpr int kEvalBatch = (32 + kNW - 1) / kNW;  // candidates per warp per iteration

__device__ __forceinline__ uint32_t lanemask_lt(int lane) { return (1u << lane) - 1u; }

// ------------------------------------------------------------------ bitonic
// The reference's warp bitonic network (include/utils.cuh:307-414): N
// registers per lane in blocked layout, compare-exchange never swaps equal keys.
__device__ __forceinline__ void cx_shfl(float& k, uint32_t& v, int c, bool asc) {
    const float k1 = __shfl_xor_sync(kFull, k, c);
    const uint32_t v1 = __shfl_xor_sync(kFull, v, c);
    if ((k != k1) && ((k < k1) != asc)) {
        k = k1;
        v = v1;
    }
}

__device__ __forceinline__ void cx_reg(float& k0, uint32_t& v0, float& k1, uint32_t& v1, bool asc) {
    if ((k0 != k1) && ((k0 < k1) != asc)) {
        const float tk = k0;
        k0 = k1;
        k1 = tk;
        const uint32_t tv = v0;
        v0 = v1;
        v1 = tv;
    }
}

template <int N>
__device__ __forceinline__ void net_merge(float (&k)[N], uint32_t (&v)[N], int range, int lane) {
    if constexpr (N == 1) {
        if (range == 1) return;
#pragma unroll
        for (int c = 16; c >= 1; c >>= 1) {
            if (c >= range) continue;
            const bool asc = ((lane & range) != 0) == ((lane & c) != 0);
            cx_shfl(k[0], v[0], c, asc);
        }
    } else if constexpr (N == 2) {
        if (range == 1) {
            cx_reg(k[0], v[0], k[1], v[1], (lane & 1) == 0);
            return;
        }
#pragma unroll
        for (int c = 16; c >= 1; c >>= 1) {
            if (c >= range) continue;
            const bool asc = ((lane & range) != 0) == ((lane & c) != 0);
            cx_shfl(k[0], v[0], c, asc);
            cx_shfl(k[1], v[1], c, asc);
        }
        cx_reg(k[0], v[0], k[1], v[1], (lane & range) == 0);
    } else {
        if (range == 1) {
#pragma unroll
            for (int b = 2; b <= N; b <<= 1)
#pragma unroll
                for (int c = b >> 1; c >= 1; c >>= 1)
#pragma unroll
                    for (int i = 0; i < N; ++i) {
                        const int j = i ^ c;
                        if (i < j) {
                            const int line = i + N * lane;
                            cx_reg(k[i], v[i], k[j], v[j], ((line & b) != 0) == ((line & c) != 0));
                        }
                    }
            return;
        }
#pragma unroll
        for (int c = 16; c >= 1; c >>= 1) {
            if (c >= range) continue;
            const bool asc = ((lane & range) != 0) == ((lane & c) != 0);
#pragma unroll
            for (int i = 0; i < N; ++i) cx_shfl(k[i], v[i], c, asc);
        }
        const bool asc = (lane & range) == 0;
#pragma unroll
        for (int c = N >> 1; c >= 1; c >>= 1)
#pragma unroll
            for (int i = 0; i < N; ++i) {
                const int j = i ^ c;
                if (i < j) cx_reg(k[i], v[i], k[j], v[j], asc);
            }
    }
}

template <int N>
__device__ __forceinline__ void net_sort(float (&k)[N], uint32_t (&v)[N], int lane) {
#pragma unroll
    for (int range = 1; range <= 32; range <<= 1) net_merge<N>(k, v, range, lane);
}

// 32-entry candidate sort (include/utils.cuh:417-457 with N_1 = 1), in registers.
__device__ __forceinline__ void sort32(float& k, uint32_t& v, int lane) {
    float kk[1] = {k};
    uint32_t vv[1] = {v};
    net_sort<1>(kk, vv, lane);
    k = kk[0];
    v = vv[0];
}

// -------------------------------------------------------------- visited set
// An exact set of node ids with linear probing; Fibonacci hashing spreads the
// consecutive ids of one mixture component.  Membership answers equal the
// reference table's (include/utils.cuh:683-750) because neither table ever
// fills: at most beam + 32 * SMALL_HASH_RESET_INTERVAL keys live between
// resets and the capacity is >= 4/3 of that.
__device__ __forceinline__ uint32_t h_slot(uint32_t key, int hbits) { return (key * 0x9E3779B1u) >> (32 - hbits); }

__device__ __forceinline__ bool h_insert(uint32_t* t, int hbits, uint32_t key) {
    const uint32_t mask = (1u << hbits) - 1u;
    uint32_t i = h_slot(key, hbits);
    for (uint32_t n = 0; n <= mask; ++n) {
        const uint32_t old = atomicCAS(&t[i], kMax, key);
        if (old == kMax) return true;
        if (old == key) return false;
        i = (i + 1) & mask;
    }
    return false;
}

__device__ __forceinline__ bool h_contains(const uint32_t* t, int hbits, uint32_t key) {
    const uint32_t mask = (1u << hbits) - 1u;
    uint32_t i = h_slot(key, hbits);
    for (uint32_t n = 0; n <= mask; ++n) {
        const uint32_t old = t[i];
        if (old == key) return true;
        if (old == kMax) return false;
        i = (i + 1) & mask;
    }
    return false;
}

// ------------------------------------------------------- query preparation
// Query factors live in shared memory next to the bit planes.
struct QueryState {
    float low, high, width;
    int32_t sum_q;
    int wrap_any;
};

// code bit t of a neighbour's packed code (byte t/8, bit t%8) holds the sign
// bit of dimension code_bit_dim(t): chunk cb = 2*(t/8) + (t%8)/4 sits in the
// low (even cb) or high nibble, nibble bits 8,4,2,1 map to dims 4cb..4cb+3
// (include/utils.cuh:836-837, 911-917).
__device__ __forceinline__ int code_bit_dim(int t) {
    const int byte = t >> 3, r = t & 7;
    const int cb = 2 * byte + (r >> 2);
    return 4 * cb + (3 - (r & 3));
}

// Quantise one rotated value: q = lroundf((x - low) * (1/width) + 0.5)
// (include/utils.cuh:894-906), with the fused multiply-add nvcc emits there.
__device__ __forceinline__ uint8_t quantize(float x, float low, float inv_w) {
    return static_cast<uint8_t>(lroundf(__fmaf_rn(__fsub_rn(x, low), inv_w, 0.5f)));
}

__device__ __forceinline__ float width_of(float lo, float hi) {
    constexpr float kInv = 1.0f / static_cast<float>((1 << FG_QG_BQUERY) - 1);
    return __fmul_rn(__fsub_rn(hi, lo), kInv);
}

// Bit planes and wrap mask from the 6-bit codes in quant[D] (one warp).
__device__ void build_planes(const uint8_t* quant, int D, uint32_t* planes, uint32_t* wrap, QueryState* qs, int lane) {
    const int W = D >> 5;
    int any = 0;
    for (int w = 0; w < W; ++w) {
        const int t = 32 * w + lane;
        const int d = code_bit_dim(t);
        const uint32_t qv = quant[d];
#pragma unroll
        for (int p = 0; p < kPlanes; ++p) {
            const uint32_t b = __ballot_sync(kFull, (qv >> p) & 1u);
            if (lane == 0) planes[p * W + w] = b;
        }
        const int cb = d >> 2;
        const bool wr = quant[4 * cb] == 64 && quant[4 * cb + 1] == 64 && quant[4 * cb + 2] == 64 && quant[4 * cb + 3] == 64;
        const uint32_t wb = __ballot_sync(kFull, wr);
        if (lane == 0) wrap[w] = wb;
        any |= (wb != 0);
    }
    if (lane == 0) qs->wrap_any = any;
}

// Rotation + quantisation for 32 <= D <= 256 in one warp: lane l holds
// elements l*E .. l*E+E-1.  Butterfly stages run len = 1, 2, ..., D/2 with
// the same additions as the reference's in-place FWHT (include/utils.cuh:790-821).
template <int E>
__device__ void prep_warp(const float* qvec, const float* __restrict__ signs, int dim, uint8_t* quant,
                          float* rot_out, QueryState* qs, int lane) {
    constexpr int D = 32 * E;
    float r[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int i = lane * E + e;
        r[e] = i < dim ? __fmul_rn(qvec[i], signs[i]) : 0.0f;
    }
#pragma unroll
    for (int len = 1; len < D; len <<= 1) {
        if (len < E) {
#pragma unroll
            for (int e = 0; e < E; ++e) {
                if ((e & len) == 0) {
                    const float u = r[e], v = r[e + len];
                    r[e] = __fadd_rn(u, v);
                    r[e + len] = __fsub_rn(u, v);
                }
            }
        } else {
            const int j = len / E;
#pragma unroll
            for (int e = 0; e < E; ++e) {
                const float o = __shfl_xor_sync(kFull, r[e], j);
                r[e] = (lane & j) ? __fsub_rn(o, r[e]) : __fadd_rn(r[e], o);
            }
        }
    }
    float lo = FLT_MAX, hi = -FLT_MAX;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        lo = fminf(lo, r[e]);
        hi = fmaxf(hi, r[e]);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        lo = fminf(lo, __shfl_xor_sync(kFull, lo, o));
        hi = fmaxf(hi, __shfl_xor_sync(kFull, hi, o));
    }
    const float width = width_of(lo, hi);
    const float inv_w = __fdiv_rn(1.0f, width);
    int sum = 0;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const uint8_t qv = quantize(r[e], lo, inv_w);
        quant[lane * E + e] = qv;
        sum += qv;
        if (rot_out) rot_out[lane * E + e] = r[e];
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) sum += __shfl_xor_sync(kFull, sum, o);
    if (lane == 0) {
        qs->low = lo;
        qs->high = hi;
        qs->width = width;
        qs->sum_q = sum;
    }
    __syncwarp();
}

// Generic rotation + quantisation with the whole CTA (any power-of-two D),
// using rot[D] in shared memory.  Same stage order and arithmetic.
__device__ void prep_block(const float* qvec, const float* __restrict__ signs, int dim, int D, float* rot,
                           uint8_t* quant, QueryState* qs, float* red_f, int* red_i) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < D; i += blockDim.x) rot[i] = i < dim ? __fmul_rn(qvec[i], signs[i]) : 0.0f;
    __syncthreads();
    for (int len = 1; len < D; len <<= 1) {
        for (int pi = tid; pi < (D >> 1); pi += blockDim.x) {
            const int blk = pi / len, j = pi % len;
            const int i1 = blk * (len << 1) + j, i2 = i1 + len;
            const float u = rot[i1], v = rot[i2];
            rot[i1] = __fadd_rn(u, v);
            rot[i2] = __fsub_rn(u, v);
        }
        __syncthreads();
    }
    float lo = FLT_MAX, hi = -FLT_MAX;
    for (int i = tid; i < D; i += blockDim.x) {
        lo = fminf(lo, rot[i]);
        hi = fmaxf(hi, rot[i]);
    }
    for (int o = 16; o >= 1; o >>= 1) {
        lo = fminf(lo, __shfl_xor_sync(kFull, lo, o));
        hi = fmaxf(hi, __shfl_xor_sync(kFull, hi, o));
    }
    if (lane == 0) {
        red_f[warp] = lo;
        red_f[kNW + warp] = hi;
    }
    __syncthreads();
    lo = FLT_MAX;
    hi = -FLT_MAX;
    for (int w = 0; w < kNW; ++w) {
        lo = fminf(lo, red_f[w]);
        hi = fmaxf(hi, red_f[kNW + w]);
    }
    const float width = width_of(lo, hi);
    const float inv_w = __fdiv_rn(1.0f, width);
    int sum = 0;
    for (int i = tid; i < D; i += blockDim.x) {
        const uint8_t qv = quantize(rot[i], lo, inv_w);
        quant[i] = qv;
        sum += qv;
    }
    for (int o = 16; o >= 1; o >>= 1) sum += __shfl_xor_sync(kFull, sum, o);
    if (lane == 0) red_i[warp] = sum;
    __syncthreads();
    if (tid == 0) {
        int s = 0;
        for (int w = 0; w < kNW; ++w) s += red_i[w];
        qs->low = lo;
        qs->high = hi;
        qs->width = width;
        qs->sum_q = s;
    }
    __syncthreads();
}

// ------------------------------------------------------------- estimation
// Integer part of the RaBitQ estimate: sum over code bits b_d * q_d, computed
// as sum_p 2^p popc(code & plane_p) (W code words per neighbour).
template <int W>
__device__ __forceinline__ uint32_t raw_sum(const uint32_t (&c)[W], const uint32_t* planes, const uint32_t* wrap,
                                            bool wrap_any) {
    uint32_t raw = 0;
#pragma unroll
    for (int p = 0; p < kPlanes; ++p) {
        uint32_t s = 0;
#pragma unroll
        for (int w = 0; w < W; ++w) s += __popc(c[w] & planes[p * W + w]);
        raw += s << p;
    }
    if (wrap_any) {
        // a chunk whose four codes are all 64 sums to 256 in the reference's
        // uint8 LUT entry 15, which wraps to 0
#pragma unroll
        for (int w = 0; w < W; ++w) {
            const uint32_t m = c[w] & wrap[w];
            const uint32_t full = m & (m >> 1) & (m >> 2) & (m >> 3) & 0x11111111u;
            raw -= 256u * static_cast<uint32_t>(__popc(full));
        }
    }
    return raw;
}

__device__ __forceinline__ uint32_t raw_sum_dyn(const uint32_t* __restrict__ code, int W, const uint32_t* planes,
                                                const uint32_t* wrap, bool wrap_any) {
    uint32_t raw = 0;
    for (int w = 0; w < W; ++w) {
        const uint32_t c = __ldg(code + w);
#pragma unroll
        for (int p = 0; p < kPlanes; ++p) raw += static_cast<uint32_t>(__popc(c & planes[p * W + w])) << p;
        if (wrap_any) {
            const uint32_t m = c & wrap[w];
            raw -= 256u * static_cast<uint32_t>(__popc(m & (m >> 1) & (m >> 2) & (m >> 3) & 0x11111111u));
        }
    }
    return raw;
}

// est = triple_x + d_parent + f_dq * width * (2 raw - sum_q) + f_vq * low
// (include/utils.cuh:989-993, 1022-1026), in the reference build's rounding.
__device__ __forceinline__ float estimate(uint32_t raw, float tx, float fdq, float fvq, float pdist,
                                          const QueryState& qs) {
    const float rf = static_cast<float>(static_cast<int32_t>(raw << 1) - qs.sum_q);
    float est = __fadd_rn(tx, pdist);
    est = __fmaf_rn(__fmul_rn(fdq, qs.width), rf, est);
    est = __fmaf_rn(fvq, qs.low, est);
    return est;
}

// -------------------------------------------------------- exact distances
__device__ __forceinline__ float tree_sum(float s) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) s = __fadd_rn(s, __shfl_down_sync(kFull, s, o));
    return __shfl_sync(kFull, s, 0);
}

// One warp computes up to kEvalBatch distances at once: every row load is
// issued before any reduction.  Per lane the accumulation runs over dims
// lane, lane+32, ... with fused multiply-adds, then the shfl_down tree
// (include/utils.cuh:270-305).
__device__ void eval_rows(const float* __restrict__ rows, uint64_t row, int dim, const float* qvec,
                          const uint32_t* nodes, int count, int use_ip, float* out, int lane) {
    float acc[kEvalBatch];
#pragma unroll
    for (int b = 0; b < kEvalBatch; ++b) acc[b] = 0.0f;
    for (int d0 = 0; d0 < dim; d0 += 128) {
        float v[kEvalBatch][4];
#pragma unroll
        for (int b = 0; b < kEvalBatch; ++b) {
            const float* r = rows + static_cast<uint64_t>(b < count ? nodes[b] : nodes[0]) * row;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int d = d0 + lane + 32 * k;
                v[b][k] = (b < count && d < dim) ? __ldg(r + d) : 0.0f;
            }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int d = d0 + lane + 32 * k;
            if (d < dim) {
                const float qd = qvec[d];
#pragma unroll
                for (int b = 0; b < kEvalBatch; ++b) {
                    if (use_ip) {
                        acc[b] = __fmaf_rn(qd, v[b][k], acc[b]);
                    } else {
                        const float df = __fsub_rn(qd, v[b][k]);
                        acc[b] = __fmaf_rn(df, df, acc[b]);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int b = 0; b < kEvalBatch; ++b) {
        const float s = tree_sum(acc[b]);
        if (b < count && lane == 0) out[b] = use_ip ? -s : s;
    }
}

__device__ __forceinline__ float warp_dist(const float* __restrict__ r, const float* qvec, int dim, int use_ip,
                                           int lane) {
    float acc = 0.0f;
    for (int d = lane; d < dim; d += 32) {
        const float x = __ldg(r + d);
        if (use_ip) {
            acc = __fmaf_rn(qvec[d], x, acc);
        } else {
            const float df = __fsub_rn(qvec[d], x);
            acc = __fmaf_rn(df, df, acc);
        }
    }
    const float s = tree_sum(acc);
    return use_ip ? -s : s;
}

// ----------------------------------------------------- adaptive controller
// src/adaptive_search_utils.cuh:8-135 and the call site at
// src/adaptive_search.cuh:166-217.
struct Ctl {
    int theta;
    float rho;
    int policy_iters;
    uint32_t top1;
    int stall;
    int warmup_done;
    float entry_d, last_d, cur_d;
    uint32_t keep_exp;
    float cutoff;
    uint32_t scan_start;
    uint32_t merge_p0;
    uint32_t n_eval;
    uint32_t n_est;
    uint32_t query;
};

__device__ __forceinline__ bool finite_lt_max(float x) { return isfinite(x) && x < FLT_MAX; }

__device__ __forceinline__ int clamp_i(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

__device__ __forceinline__ float clamp_f(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

__device__ __forceinline__ uint32_t keep_per_parent(uint32_t maxdeg, float rho) {
    float kf = __fsub_rn(1.0f, rho);
    if (kf < 0.0f) kf = 0.0f;
    if (kf > 1.0f) kf = 1.0f;
    uint32_t kc = static_cast<uint32_t>(ceilf(__fmul_rn(static_cast<float>(maxdeg), kf)));
    if (kc < 1) kc = 1;
    if (kc > maxdeg) kc = maxdeg;
    return kc;
}

__device__ __forceinline__ int keep_for(uint32_t active, int theta, float rho, bool cut_valid, uint32_t near) {
    const int ac = static_cast<int>(active);
    const int rho_keep = static_cast<int>(keep_per_parent(active, rho));
    const uint32_t bound = static_cast<uint32_t>(BUFFER_BOUND) / static_cast<uint32_t>(theta);
    const int budget = clamp_i(static_cast<int>(bound), 1, ac);
    int mk = rho_keep < budget ? rho_keep : budget;
    if (cut_valid) mk = clamp_i(static_cast<int>(near), 1, mk);
    return clamp_i(mk, 1, ac);
}

__device__ void controller_step(Ctl& c, uint32_t beam0, int iter, float phase2_rho) {
    const uint32_t top1 = beam0 & 0x7fffffffu;
    const int stall = (c.policy_iters > 0 && top1 == c.top1) ? c.stall + 1 : 0;
    const bool changed = c.warmup_done || stall >= TOP1_WARMUP_STALL_ITERS;
    // update_expander_progress
    const float e = c.entry_d;
    const float last = finite_lt_max(c.last_d) ? c.last_d : e;
    const float cur = finite_lt_max(c.cur_d) ? c.cur_d : last;
    float rate = 0.0f;
    const float denom = fabsf(e);
    if (isfinite(last) && isfinite(cur) && isfinite(e) && !(denom <= 1.0e-20f)) {
        const float prog = __fdiv_rn(__fsub_rn(last, cur), denom);
        if (isfinite(prog) && prog > 0.0f) rate = prog < 1.0f ? prog : 1.0f;
    }
    c.top1 = top1;
    c.stall = stall;
    c.last_d = last;
    c.cur_d = cur;
    if (changed) {
        c.warmup_done = 1;
        c.theta = PHASE2_THETA;
        c.rho = phase2_rho;
        c.policy_iters += 1;
    } else if (iter == 0 || (iter % CHECK_INTERVAL) == 0) {
        const float span = phase2_rho > PHASE1_RHO ? __fsub_rn(phase2_rho, PHASE1_RHO) : __fsub_rn(RHO_MAX, RHO_MIN);
        const float base = c.policy_iters == 0 ? PHASE1_RHO : c.rho;
        const float cap = phase2_rho > PHASE1_RHO ? phase2_rho : RHO_MAX;
        c.warmup_done = 0;
        c.theta = PHASE1_THETA;
        c.rho = clamp_f(__fmaf_rn(span, rate, base), RHO_MIN, cap);
        c.policy_iters += 1;
    }
}

// smallest `eff` valid lanes by (estimate, lane) -- the rank rule of
// include/utils.cuh:251-267 -- by repeated warp minimum on order-preserving keys.
__device__ __forceinline__ uint32_t fkey(float f) {
    const uint32_t u = __float_as_uint(__fadd_rn(f, 0.0f));  // -0 -> +0: equal floats, equal keys
    return (u & kMsb) ? ~u : (u | kMsb);
}

__device__ __forceinline__ bool keep_smallest(float est, bool valid, int eff, int lane) {
    uint32_t key = valid ? fkey(est) : kMax;
    bool sel = false;
    for (int r = 0; r < eff; ++r) {
        const uint32_t m = __reduce_min_sync(kFull, key);
        if (m == kMax) break;
        const uint32_t cand = __ballot_sync(kFull, key == m);
        if (lane == __ffs(cand) - 1) {
            sel = true;
            key = kMax;
        }
    }
    return sel;
}

// ------------------------------------------------------------ beam merges
// Register bitonic merge for itopk = 32*N2 <= 128 (include/utils.cuh:490-586),
// run by warp 0.
template <int N2>
__device__ void merge_bitonic(uint32_t* bidx, float* bdist, uint32_t* cidx, float* cdist, uint32_t cbs, bool first,
                              int lane) {
    constexpr uint32_t itopk = 32u * N2;
    float k1 = lane < static_cast<int>(cbs) ? cdist[lane] : FLT_MAX;
    uint32_t v1 = lane < static_cast<int>(cbs) ? cidx[lane] : kMax;
    sort32(k1, v1, lane);
    if (lane < static_cast<int>(cbs)) {
        cdist[lane] = k1;
        cidx[lane] = v1;
    }
    __syncwarp();
    float k[N2];
    uint32_t v[N2];
    if (first) {
#pragma unroll
        for (int i = 0; i < N2; ++i) {
            k[i] = bdist[lane + 32 * i];
            v[i] = bidx[lane + 32 * i];
        }
        net_sort<N2>(k, v, lane);
    } else {
#pragma unroll
        for (int i = 0; i < N2; ++i) {
            k[i] = bdist[N2 * lane + i];
            v[i] = bidx[N2 * lane + i];
        }
    }
#pragma unroll
    for (int i = 0; i < N2; ++i) {
        const uint32_t j = static_cast<uint32_t>(N2 * lane + i);
        const uint32_t kk = itopk - 1u - j;
        if (kk < cbs) {
            const float ck = cdist[kk];
            if (k[i] > ck) {
                k[i] = ck;
                v[i] = cidx[kk];
            }
        }
    }
    net_merge<N2>(k, v, 32, lane);
    __syncwarp();
#pragma unroll
    for (int i = 0; i < N2; ++i) {
        bdist[N2 * lane + i] = k[i];
        bidx[N2 * lane + i] = v[i];
    }
    __syncwarp();
}

// number of a[0..n) <= x (upper bound) / < x (lower bound); a ascending
__device__ __forceinline__ uint32_t upper_bound(const float* a, uint32_t n, float x) {
    uint32_t lo = 0, hi = n;
    while (lo < hi) {
        const uint32_t mid = (lo + hi) >> 1;
        if (a[mid] <= x) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

__device__ __forceinline__ uint32_t lower_bound(const float* a, uint32_t n, float x) {
    uint32_t lo = 0, hi = n;
    while (lo < hi) {
        const uint32_t mid = (lo + hi) >> 1;
        if (a[mid] < x) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

// The reference's merge-path partition (include/utils.cuh:588-616).
__device__ __forceinline__ int mp_search(const float* a, int an, const float* b, int bn, int diag) {
    int lo = max(0, diag - bn), hi = min(diag, an);
    while (lo <= hi) {
        const int ai = (lo + hi) >> 1, bi = diag - ai;
        const float al = ai > 0 ? a[ai - 1] : -FLT_MAX;
        const float ar = ai < an ? a[ai] : FLT_MAX;
        const float bl = bi > 0 ? b[bi - 1] : -FLT_MAX;
        const float br = bi < bn ? b[bi] : FLT_MAX;
        if (al > br) hi = ai - 1;
        else if (bl > ar) lo = ai + 1;
        else return ai;
    }
    return lo;
}

// Beam elements taken before output diagonal d, exactly as the reference's
// merge path decides it.  Without a beam/candidate tie at the split the
// partition is unique and equals the stable (beam-first) rank split;
// otherwise the reference's own binary search picks among the valid splits.
__device__ __forceinline__ int split_at(int d, uint32_t p0, const uint32_t* pos, const float* a, int an,
                                        const float* b, int bn) {
    if (d <= static_cast<int>(p0)) return d;
    // candidates placed before d in the stable merge
    int lo = 0, hi = bn;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (pos[mid] < static_cast<uint32_t>(d)) lo = mid + 1;
        else hi = mid;
    }
    const int ai = d - lo, bi = lo;
    if (ai > 0 && bi < bn && a[ai - 1] == b[bi] && a[ai - 1] != FLT_MAX) return mp_search(a, an, b, bn, d);
    return ai;
}

// Merge-path beam merge (include/utils.cuh:618-680) for itopk > 128 or
// itopk % 32 != 0.  Output segment s covers [s*itopk/active, (s+1)*itopk/active)
// and is merged beam-first between the reference's partitions.
// Ends with the merged beam visible to the whole CTA.
__device__ void merge_path(uint32_t* bidx, float* bdist, uint32_t* cidx, float* cdist, uint32_t cbs, uint32_t itopk,
                           int active, uint32_t* pos, Ctl& ctl) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (warp == 0) {
        float k = lane < static_cast<int>(cbs) ? cdist[lane] : FLT_MAX;
        uint32_t v = lane < static_cast<int>(cbs) ? cidx[lane] : kMax;
        sort32(k, v, lane);
        if (lane < static_cast<int>(cbs)) {
            cdist[lane] = k;
            cidx[lane] = v;
            pos[lane] = static_cast<uint32_t>(lane) + upper_bound(bdist, itopk, k);
        }
        if (lane == 0) ctl.merge_p0 = lower_bound(bdist, itopk, k);
    }
    __syncthreads();
    const uint32_t p0 = ctl.merge_p0;
    float od[kMaxSegPerThread * 4];
    uint32_t oi[kMaxSegPerThread * 4];
    const int s_begin = tid * kMaxSegPerThread;
    int nout = 0;
    int out_begin = -1;
#pragma unroll
    for (int sj = 0; sj < kMaxSegPerThread; ++sj) {
        const int s = s_begin + sj;
        if (s >= active) break;
        const int ob = static_cast<int>((static_cast<uint32_t>(s) * itopk) / static_cast<uint32_t>(active));
        const int oe = static_cast<int>((static_cast<uint32_t>(s + 1) * itopk) / static_cast<uint32_t>(active));
        if (oe <= static_cast<int>(p0)) continue;  // identical prefix
        if (out_begin < 0) out_begin = ob;
        const int tb = split_at(ob, p0, pos, bdist, static_cast<int>(itopk), cdist, static_cast<int>(cbs));
        const int te = split_at(oe, p0, pos, bdist, static_cast<int>(itopk), cdist, static_cast<int>(cbs));
        int ti = tb, ci = ob - tb;
        const int ce = oe - te;
        for (int o = ob; o < oe; ++o) {
            const bool take = (ci >= ce) || (ti < te && bdist[ti] <= cdist[ci]);
            if (take) {
                od[nout] = bdist[ti];
                oi[nout] = bidx[ti];
                ++ti;
            } else {
                od[nout] = cdist[ci];
                oi[nout] = cidx[ci];
                ++ci;
            }
            ++nout;
        }
    }
    __syncthreads();
    for (int i = 0; i < nout; ++i) {
        bdist[out_begin + i] = od[i];
        bidx[out_begin + i] = oi[i];
    }
    __syncthreads();
}

// ------------------------------------------------------------- the search
struct Plan {
    uint32_t padded, cbs, collect_cap;
    int hbits;
    float phase2_rho;
    int max_iter;
    int merge_n2;
    int mp_active;
};

struct Smem {
    uint32_t* beam_idx;
    float* beam_dist;
    uint32_t* cand_idx;
    float* cand_dist;
    uint32_t* hash;
    float* qvec;
    uint32_t* planes;
    uint32_t* wrap;
    uint8_t* quant;
    uint32_t* stage;
    uint32_t* pos;
    uint32_t* eval_slot;
    uint32_t* eval_node;
    float* rot;
};

__host__ __device__ inline size_t align16(size_t x) { return (x + 15) & ~static_cast<size_t>(15); }

__host__ __device__ inline size_t smem_layout(uint32_t padded, int hbits, int dim, int D, Smem* s, unsigned char* base) {
    size_t off = 0;
    auto take = [&](size_t bytes) {
        unsigned char* p = base ? base + off : nullptr;
        off += align16(bytes);
        return p;
    };
    unsigned char* p;
    p = take(padded * 4); if (s) s->beam_idx = reinterpret_cast<uint32_t*>(p);
    p = take(padded * 4); if (s) s->beam_dist = reinterpret_cast<float*>(p);
    p = take(32 * 4); if (s) s->cand_idx = reinterpret_cast<uint32_t*>(p);
    p = take(32 * 4); if (s) s->cand_dist = reinterpret_cast<float*>(p);
    p = take((size_t(1) << hbits) * 4); if (s) s->hash = reinterpret_cast<uint32_t*>(p);
    p = take(static_cast<size_t>(dim) * 4); if (s) s->qvec = reinterpret_cast<float*>(p);
    const int W = D >= 32 ? D / 32 : 1;
    p = take(static_cast<size_t>(kPlanes) * W * 4); if (s) s->planes = reinterpret_cast<uint32_t*>(p);
    p = take(static_cast<size_t>(W) * 4); if (s) s->wrap = reinterpret_cast<uint32_t*>(p);
    p = take(static_cast<size_t>(D < 32 ? 32 : D)); if (s) s->quant = p;
    p = take(static_cast<size_t>(SEARCH_WIDTH) * 32 * 4); if (s) s->stage = reinterpret_cast<uint32_t*>(p);
    p = take(32 * 4); if (s) s->pos = reinterpret_cast<uint32_t*>(p);
    p = take(32 * 4); if (s) s->eval_slot = reinterpret_cast<uint32_t*>(p);
    p = take(32 * 4); if (s) s->eval_node = reinterpret_cast<uint32_t*>(p);
    const bool warp_prep = D >= 32 && D <= 256;
    p = take(warp_prep ? 0 : static_cast<size_t>(D < 32 ? 32 : D) * 4); if (s) s->rot = reinterpret_cast<float*>(p);
    return off;
}

template <int W>
__device__ __forceinline__ void load_codes(const float* prow, uint64_t code_off, int ni, bool vec, uint32_t (&c)[W]) {
    const uint32_t* base = reinterpret_cast<const uint32_t*>(prow + code_off) + static_cast<size_t>(ni) * W;
    if constexpr (W % 4 == 0) {
        if (vec) {
#pragma unroll
            for (int w = 0; w < W; w += 4) {
                const uint4 x = __ldg(reinterpret_cast<const uint4*>(base + w));
                c[w] = x.x;
                c[w + 1] = x.y;
                c[w + 2] = x.z;
                c[w + 3] = x.w;
            }
            return;
        }
    }
#pragma unroll
    for (int w = 0; w < W; ++w) c[w] = __ldg(base + w);
}

// Estimate of neighbour `ni` of parent row `prow` for this lane.
template <int W>
__device__ __forceinline__ uint32_t lane_raw(const float* prow, uint64_t code_off, int ni, bool vec, int D,
                                             const uint32_t* planes, const uint32_t* wrap, bool wrap_any) {
    if constexpr (W > 0) {
        uint32_t c[W];
        load_codes<W>(prow, code_off, ni, vec, c);
        return raw_sum<W>(c, planes, wrap, wrap_any);
    } else {
        const int Wd = D >> 5;
        return raw_sum_dyn(reinterpret_cast<const uint32_t*>(prow + code_off) + static_cast<size_t>(ni) * Wd, Wd, planes,
                           wrap, wrap_any);
    }
}

template <int W, bool TRACE>
__device__ void search_one(const SearchArgs& a, const Plan& pl, const Smem& sm, Ctl& ctl, QueryState& qs,
                           uint32_t* s_pnode, float* s_pdist, uint32_t* s_ppos, uint32_t* s_stage_cnt,
                           float* red_f, int* red_i, uint32_t qid, int vec_codes) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int dim = a.dim, D = a.padded_dim, deg = a.degree, beam = a.beam;
    const uint32_t padded = pl.padded, cbs = pl.cbs;
    const int hbits = pl.hbits;
    const float* __restrict__ rows = a.rows;
    const uint64_t rowf = a.row;
    const bool vec = vec_codes != 0;

    // ---------------------------------------------------------------- init
    const float* q = a.queries + static_cast<size_t>(qid) * dim;
    for (int i = tid; i < dim; i += kThreads) sm.qvec[i] = q[i];
    for (int i = tid; i < (1 << hbits); i += kThreads) sm.hash[i] = kMax;
    for (uint32_t i = tid; i < padded; i += kThreads) {
        sm.beam_idx[i] = kMax;
        sm.beam_dist[i] = FLT_MAX;
    }
    if (tid < 32) {
        sm.cand_idx[tid] = kMax;
        sm.cand_dist[tid] = FLT_MAX;
    }
    __syncthreads();
    uint32_t c_iters = 0, c_exp = 0, c_eval = 1;
    if (warp == 0) {
        const float ed = warp_dist(rows + static_cast<uint64_t>(a.entry) * rowf, sm.qvec, dim, a.use_ip, lane);
        if (lane == 0) {
            sm.cand_idx[0] = a.entry;
            sm.cand_dist[0] = ed;
            h_insert(sm.hash, hbits, a.entry);
            ctl.theta = PHASE1_THETA;
            ctl.rho = PHASE1_RHO;
            ctl.policy_iters = 0;
            ctl.top1 = kMax;
            ctl.stall = 0;
            ctl.warmup_done = 0;
            ctl.entry_d = ed;
            ctl.last_d = FLT_MAX;
            ctl.cur_d = FLT_MAX;
            ctl.scan_start = 0;
            ctl.n_est = 0;
        }
    }
    const bool warp_prep = D >= 32 && D <= 256;
    if (warp_prep) {
        const int pw = kNW > 1 ? 1 : 0;
        if (warp == pw) {
            switch (D) {
                case 32: prep_warp<1>(sm.qvec, a.signs, dim, sm.quant, nullptr, &qs, lane); break;
                case 64: prep_warp<2>(sm.qvec, a.signs, dim, sm.quant, nullptr, &qs, lane); break;
                case 128: prep_warp<4>(sm.qvec, a.signs, dim, sm.quant, nullptr, &qs, lane); break;
                default: prep_warp<8>(sm.qvec, a.signs, dim, sm.quant, nullptr, &qs, lane); break;
            }
            build_planes(sm.quant, D, sm.planes, sm.wrap, &qs, lane);
        }
    } else {
        prep_block(sm.qvec, a.signs, dim, D, sm.rot, sm.quant, &qs, red_f, red_i);
        if (warp == 0) build_planes(sm.quant, D < 32 ? 32 : D, sm.planes, sm.wrap, &qs, lane);
    }
    __syncthreads();

    // ---------------------------------------------------------------- loop
    const bool mp = pl.merge_n2 == 0;
    const QueryState qsl = qs;
    for (int iter = 0; iter < MAX_ITERATIONS; ++iter) {
        if ((iter + 1) % SMALL_HASH_RESET_INTERVAL == 0) {
            for (int i = tid; i < (1 << hbits); i += kThreads) sm.hash[i] = kMax;
            __syncthreads();
            for (int i = tid; i < beam; i += kThreads) h_insert(sm.hash, hbits, sm.beam_idx[i] & ~kMsb);
        }
        __syncthreads();
        if (iter >= pl.max_iter) break;

        // merge the candidates of the previous iteration into the beam
        if (mp) {
            merge_path(sm.beam_idx, sm.beam_dist, sm.cand_idx, sm.cand_dist, cbs, padded, pl.mp_active, sm.pos, ctl);
        } else if (warp == 0) {
            if (pl.merge_n2 == 1) merge_bitonic<1>(sm.beam_idx, sm.beam_dist, sm.cand_idx, sm.cand_dist, cbs, iter == 0, lane);
            else if (pl.merge_n2 == 2) merge_bitonic<2>(sm.beam_idx, sm.beam_dist, sm.cand_idx, sm.cand_dist, cbs, iter == 0, lane);
            else merge_bitonic<4>(sm.beam_idx, sm.beam_dist, sm.cand_idx, sm.cand_dist, cbs, iter == 0, lane);
        }
        ++c_iters;

        // control: warp 0 (src/adaptive_search.cuh:147-217)
        if (warp == 0) {
            for (uint32_t i = static_cast<uint32_t>(beam) + lane; i < padded; i += 32) {
                sm.beam_idx[i] = kMax;
                sm.beam_dist[i] = FLT_MAX;
            }
            if (lane < static_cast<int>(cbs)) {
                sm.cand_idx[lane] = kMax;
                sm.cand_dist[lane] = FLT_MAX;
            }
            uint32_t start = 0;
            if (lane == 0) {
                ctl.cutoff = sm.beam_idx[beam - 1] == kMax ? FLT_MAX : sm.beam_dist[(a.K < beam ? a.K : beam) - 1];
                controller_step(ctl, sm.beam_idx[0], iter, pl.phase2_rho);
                if (mp) {
                    if (ctl.merge_p0 < ctl.scan_start) ctl.scan_start = ctl.merge_p0;
                    start = ctl.scan_start & ~31u;
                }
            }
            const int theta = __shfl_sync(kFull, ctl.theta, 0);
            start = __shfl_sync(kFull, start, 0);
            // pick_expanders (include/utils.cuh:752-787); entries before
            // `start` are known to be expanded already
            uint32_t num = 0;
            const uint32_t lim = (static_cast<uint32_t>(beam) + 31u) & ~31u;
            for (uint32_t j0 = start; j0 < lim; j0 += 32) {
                const uint32_t j = j0 + lane;
                uint32_t e = 0;
                const bool np = j < static_cast<uint32_t>(beam) && ((e = sm.beam_idx[j]) & kMsb) == 0;
                const uint32_t b = __ballot_sync(kFull, np);
                if (np) {
                    const uint32_t i = __popc(b & lanemask_lt(lane)) + num;
                    if (i < static_cast<uint32_t>(theta)) {
                        s_ppos[i] = j;
                        s_pnode[i] = e & 0x7fffffffu;
                        s_pdist[i] = sm.beam_dist[j];
                        sm.beam_idx[j] = e | kMsb;
                    }
                }
                num += __popc(b);
                if (num >= static_cast<uint32_t>(theta)) {
                    num = theta;
                    break;
                }
            }
            __syncwarp();
            if (lane == 0) {
                ctl.keep_exp = num;
                if (mp) ctl.scan_start = num == static_cast<uint32_t>(theta) ? s_ppos[num - 1] + 1 : static_cast<uint32_t>(beam);
                if (num) {
                    // record_selected_expander_dist
                    ctl.last_d = finite_lt_max(ctl.cur_d) ? ctl.cur_d : ctl.entry_d;
                    ctl.cur_d = s_pdist[num - 1];
                }
            }
            if (TRACE && a.trace && iter < a.trace_cap) {
                const size_t base = (static_cast<size_t>(qid) * a.trace_cap + iter);
                if (lane < SEARCH_WIDTH) a.trace[base * SEARCH_WIDTH + lane] = lane < static_cast<int>(num) ? s_pnode[lane] : kMax;
                if (lane == 0) a.trace_count[base] = static_cast<int32_t>(num);
            }
        }
        __syncthreads();
        const uint32_t keep_exp = ctl.keep_exp;
        if (!keep_exp) break;
        c_exp += keep_exp;
        const int theta = ctl.theta;
        const float rho = ctl.rho;
        const float cutoff = ctl.cutoff;
        const bool cut_ok = isfinite(cutoff) && cutoff < FLT_MAX;

        if (!(theta > 1)) {
            // ------------------------ single expander (src/adaptive_search.cuh:221-343)
            if (warp == 0) {
                const uint32_t work = static_cast<uint32_t>(deg) < cbs ? static_cast<uint32_t>(deg) : cbs;
                const float* prow = rows + static_cast<uint64_t>(s_pnode[0]) * rowf;
                const bool in_work = static_cast<uint32_t>(lane) < work;
                uint32_t child = in_work ? __ldg(reinterpret_cast<const uint32_t*>(prow + a.nbr_off) + lane) : kMax;
                float tx = 0.0f, fdq = 0.0f, fvq = 0.0f;
                if (in_work) {
                    tx = __ldg(prow + a.factor_off + lane);
                    fdq = __ldg(prow + a.factor_off + deg + lane);
                    fvq = __ldg(prow + a.factor_off + 2 * deg + lane);
                }
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
                        if (tx != FLT_MAX) {
                            const uint32_t raw = lane_raw<W>(prow, a.code_off, lane, vec, D, sm.planes, sm.wrap, qsl.wrap_any);
                            est = estimate(raw, tx, fdq, fvq, s_pdist[0], qsl);
                        }
                        if (isfinite(est)) dist = est;
                        else {
                            dist = FLT_MAX;
                            child = kMax;
                        }
                    }
                    if (lane == 0) ctl.n_est += vcount;
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
                if (lane == 0) ctl.n_eval = __popc(ib);
            }
        } else {
            // ------------------- speculative expanders (src/adaptive_search.cuh:344-444)
            // deg <= 32: one neighbour tile per parent, every lookup of the
            // round precedes its inserts.
            const uint32_t active = static_cast<uint32_t>(deg) < 32u ? static_cast<uint32_t>(deg) : 32u;
            for (int t = warp; t < static_cast<int>(keep_exp); t += kNW) {
                const float* prow = rows + static_cast<uint64_t>(s_pnode[t]) * rowf;
                const bool in_deg = lane < deg;
                uint32_t child = in_deg ? __ldg(reinterpret_cast<const uint32_t*>(prow + a.nbr_off) + lane) : kMax;
                float tx = FLT_MAX, fdq = 0.0f, fvq = 0.0f;
                if (in_deg) {
                    tx = __ldg(prow + a.factor_off + lane);
                    fdq = __ldg(prow + a.factor_off + deg + lane);
                    fvq = __ldg(prow + a.factor_off + 2 * deg + lane);
                }
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
                        if (tx != FLT_MAX) {
                            const uint32_t raw = lane_raw<W>(prow, a.code_off, lane, vec, D, sm.planes, sm.wrap, qsl.wrap_any);
                            est = estimate(raw, tx, fdq, fvq, s_pdist[t], qsl);
                        }
                        valid = isfinite(est);
                    }
                    if (lane == 0) atomicAdd(&ctl.n_est, raw_valid);
                    const uint32_t near = __popc(__ballot_sync(kFull, valid && cut_ok && est <= cutoff));
                    const int eff = keep_for(active, theta, rho, cut_ok, near);
                    kl = keep_smallest(est, valid, eff, lane);
                }
                const uint32_t kb = __ballot_sync(kFull, kl);
                if (kl) sm.stage[t * 32 + __popc(kb & lanemask_lt(lane))] = child;
                if (lane == 0) s_stage_cnt[t] = __popc(kb);
            }
            __syncthreads();
            if (warp == 0) {
                // inserts and compaction in (parent, lane) order; a child kept by
                // two parents goes to the first (include/utils.cuh:187-214)
                uint32_t compact = 0;
                uint32_t carry = 0;  // entries consumed before this chunk
                uint32_t total = 0;
                for (uint32_t t = 0; t < keep_exp; ++t) total += s_stage_cnt[t];
                for (uint32_t base = 0; base < total; base += 32) {
                    const uint32_t e = base + lane;
                    uint32_t child = kMax;
                    if (e < total) {
                        uint32_t acc = 0, t = 0;
                        while (acc + s_stage_cnt[t] <= e) acc += s_stage_cnt[t++];
                        child = sm.stage[t * 32 + (e - acc)];
                    }
                    const uint32_t same = __match_any_sync(kFull, child);
                    const bool first = child != kMax && (__ffs(same) - 1) == lane;
                    const bool ins = first && h_insert(sm.hash, hbits, child);
                    const uint32_t ib = __ballot_sync(kFull, ins);
                    if (ins) {
                        const uint32_t slot = compact + __popc(ib & lanemask_lt(lane));
                        if (slot < pl.collect_cap) {
                            sm.cand_idx[slot] = child;
                            sm.cand_dist[slot] = FLT_MAX;
                            sm.eval_slot[slot] = slot;
                            sm.eval_node[slot] = child;
                        }
                    }
                    compact += __popc(ib);
                    carry += 32;
                }
                if (lane == 0) ctl.n_eval = compact < pl.collect_cap ? compact : pl.collect_cap;
            }
        }
        __syncthreads();
        // ------------------------------- exact distances of accepted children
        {
            const uint32_t ne = ctl.n_eval;
            c_eval += ne;
            // warp w evaluates list entries w, w + kNW, ...
            uint32_t nodes[kEvalBatch];
            int cnt = 0;
#pragma unroll
            for (int b = 0; b < kEvalBatch; ++b) {
                const uint32_t e = static_cast<uint32_t>(warp) + static_cast<uint32_t>(b * kNW);
                nodes[b] = e < ne ? sm.eval_node[e] : 0u;
                cnt += e < ne;
            }
            if (cnt > 0) {
                float d[kEvalBatch];
                eval_rows(rows, rowf, dim, sm.qvec, nodes, cnt, a.use_ip, d, lane);
                if (lane == 0) {
                    for (int b = 0; b < cnt; ++b) sm.cand_dist[sm.eval_slot[warp + b * kNW]] = d[b];
                }
            }
        }
    }
    // final merge (src/adaptive_search.cuh:448-452)
    __syncthreads();
    if (mp) {
        merge_path(sm.beam_idx, sm.beam_dist, sm.cand_idx, sm.cand_dist, cbs, padded, pl.mp_active, sm.pos, ctl);
    } else if (warp == 0) {
        if (pl.merge_n2 == 1) merge_bitonic<1>(sm.beam_idx, sm.beam_dist, sm.cand_idx, sm.cand_dist, cbs, false, lane);
        else if (pl.merge_n2 == 2) merge_bitonic<2>(sm.beam_idx, sm.beam_dist, sm.cand_idx, sm.cand_dist, cbs, false, lane);
        else merge_bitonic<4>(sm.beam_idx, sm.beam_dist, sm.cand_idx, sm.cand_dist, cbs, false, lane);
    }
    __syncthreads();
    // results (src/adaptive_search.cuh:455-464): position i < beam holds the
    // beam entry (MSB cleared); positions >= beam repeat the last one
    for (int i = tid; i < a.K; i += kThreads) {
        const int s = i < beam ? i : beam - 1;
        a.out_ids[static_cast<size_t>(qid) * a.K + i] = sm.beam_idx[s] & 0x7fffffffu;
        if (a.out_dists) a.out_dists[static_cast<size_t>(qid) * a.K + i] = sm.beam_dist[s];
    }
    if (tid == 0 && a.stats) {
        fg_query_stats st;
        st.iterations = c_iters;
        st.expansions = c_exp;
        st.evaluations = c_eval;
        st.estimates = ctl.n_est;
        a.stats[qid] = st;
    }
    __syncthreads();
}

template <int W, bool TRACE>
__global__ void __launch_bounds__(kThreads) search_kernel(const SearchArgs a, const Plan pl, int vec_codes) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ Ctl ctl;
    __shared__ QueryState qs;
    __shared__ uint32_t s_pnode[SEARCH_WIDTH];
    __shared__ float s_pdist[SEARCH_WIDTH];
    __shared__ uint32_t s_ppos[SEARCH_WIDTH];
    __shared__ uint32_t s_stage_cnt[SEARCH_WIDTH];
    __shared__ float red_f[2 * kNW];
    __shared__ int red_i[kNW];
    Smem sm;
    smem_layout(pl.padded, pl.hbits, a.dim, a.padded_dim, &sm, smem_raw);
    for (;;) {
        if (threadIdx.x == 0) ctl.query = atomicAdd(a.work_counter, 1u);
        __syncthreads();
        const uint32_t qid = ctl.query;
        __syncthreads();
        if (qid >= static_cast<uint32_t>(a.nq)) break;
        search_one<W, TRACE>(a, pl, sm, ctl, qs, s_pnode, s_pdist, s_ppos, s_stage_cnt, red_f, red_i, qid, vec_codes);
    }
}

// ------------------------------------------------ standalone query prepare
__global__ void __launch_bounds__(kThreads) query_prepare_kernel(const float* queries, int nq, int dim, int D,
                                                                 const float* signs, float* rotated, uint8_t* quant_out,
                                                                 uint8_t* lut, float* factors, int32_t* sum_q) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ QueryState qs;
    __shared__ float red_f[2 * kNW];
    __shared__ int red_i[kNW];
    float* qvec = reinterpret_cast<float*>(smem_raw);
    float* rot = qvec + align16(dim * 4) / 4;
    uint8_t* quant = reinterpret_cast<uint8_t*>(rot + (D < 32 ? 32 : D));
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
            prep_block(qvec, signs, dim, D, rot, quant, &qs, red_f, red_i);
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
__global__ void __launch_bounds__(kThreads) beam_merge_kernel(uint32_t* idx, float* dist, int itopk, int cbs, int first,
                                                              int merge_n2, int active) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ Ctl ctl;
    const int total = itopk + cbs;
    uint32_t* sidx = reinterpret_cast<uint32_t*>(smem_raw);
    float* sdist = reinterpret_cast<float*>(sidx + total);
    uint32_t* pos = reinterpret_cast<uint32_t*>(sdist + total);
    const size_t off = static_cast<size_t>(blockIdx.x) * total;
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
        sidx[i] = idx[off + i];
        sdist[i] = dist[off + i];
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (merge_n2 == 0) {
        merge_path(sidx, sdist, sidx + itopk, sdist + itopk, cbs, itopk, active, pos, ctl);
    } else if (warp == 0) {
        if (merge_n2 == 1) merge_bitonic<1>(sidx, sdist, sidx + itopk, sdist + itopk, cbs, first != 0, lane);
        else if (merge_n2 == 2) merge_bitonic<2>(sidx, sdist, sidx + itopk, sdist + itopk, cbs, first != 0, lane);
        else merge_bitonic<4>(sidx, sdist, sidx + itopk, sdist + itopk, cbs, first != 0, lane);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < itopk; i += blockDim.x) {
        idx[off + i] = sidx[i];
        dist[off + i] = sdist[i];
    }
}

}  // namespace

// --------------------------------------------------------------- host side
uint32_t effective_sort_beam(uint32_t beam) {
    if (beam == 0) return 0;
    uint32_t x = beam - 1;
    x |= x >> 1; x |= x >> 2; x |= x >> 4; x |= x >> 8; x |= x >> 16;
    const uint32_t r = beam <= 1 ? 1 : x + 1;
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

int hash_bits(uint32_t padded, uint32_t cbs) {
    const uint64_t req = static_cast<uint64_t>(padded) + static_cast<uint64_t>(cbs) * SMALL_HASH_RESET_INTERVAL;
    const uint64_t target = (req * 4 + 2) / 3;
    int b = FG_HASH_BASE_BITLEN;
    while ((uint64_t(1) << b) < target) ++b;
    return b;
}

static int merge_width(uint32_t itopk) {
    uint32_t n2 = (itopk + 31) / 32;
    if (n2 > 32) n2 = 4;
    return (itopk % 32 == 0 && (n2 == 1 || n2 == 2 || n2 == 4)) ? static_cast<int>(n2) : 0;
}

static int merge_active(uint32_t itopk) {
    int active = static_cast<int>((itopk + 3) / 4);
    active = ((active + 31) / 32) * 32;
    return active < BLOCK_SIZE ? active : BLOCK_SIZE;
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
    if (a.dim < 1 || a.dim > FG_MAX_DIM) {
        snprintf(err, errlen, "dim %d outside the supported range [1, %d]", a.dim, FG_MAX_DIM);
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
    p->smem_bytes = smem_layout(p->padded, p->hbits, a.dim, a.padded_dim, nullptr, nullptr);
    p->threads = kThreads;
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
    const int W = a.padded_dim / 32;
    const void* fn = nullptr;
    const bool trace = a.trace != nullptr;
    switch (W) {
        case 4: fn = trace ? (const void*)search_kernel<4, true> : (const void*)search_kernel<4, false>; break;
        case 2: fn = trace ? (const void*)search_kernel<2, true> : (const void*)search_kernel<2, false>; break;
        case 1: fn = trace ? (const void*)search_kernel<1, true> : (const void*)search_kernel<1, false>; break;
        case 8: fn = trace ? (const void*)search_kernel<8, true> : (const void*)search_kernel<8, false>; break;
        default: fn = trace ? (const void*)search_kernel<0, true> : (const void*)search_kernel<0, false>; break;
    }
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(p->smem_bytes));
    if (e != cudaSuccess) {
        snprintf(err, errlen, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        return FG_ERR_CUDA;
    }
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kThreads, p->smem_bytes);
    if (e != cudaSuccess || per_sm < 1) {
        snprintf(err, errlen, "occupancy query failed: %s", cudaGetErrorString(e));
        return FG_ERR_CUDA;
    }
    const int resident = per_sm * sms;
    p->grid = a.nq < resident ? a.nq : resident;
    if (p->grid < 1) p->grid = 1;
    return FG_OK;
}

cudaError_t launch_search(const SearchArgs& a, const SearchPlan& p, cudaStream_t stream) {
    Plan pl;
    pl.padded = p.padded;
    pl.cbs = p.cbs;
    pl.collect_cap = p.collect_cap;
    pl.hbits = p.hbits;
    pl.phase2_rho = p.phase2_rho;
    pl.max_iter = p.max_iter;
    pl.merge_n2 = p.merge_n2;
    pl.mp_active = p.mp_active;
    cudaError_t e = cudaMemsetAsync(a.work_counter, 0, sizeof(uint32_t), stream);
    if (e != cudaSuccess) return e;
    const int W = a.padded_dim / 32;
    const bool trace = a.trace != nullptr;
    dim3 g(p.grid), b(kThreads);
#define FG_LAUNCH(WW)                                                                          \
    do {                                                                                       \
        if (trace) search_kernel<WW, true><<<g, b, p.smem_bytes, stream>>>(a, pl, p.vec_codes);  \
        else search_kernel<WW, false><<<g, b, p.smem_bytes, stream>>>(a, pl, p.vec_codes);      \
    } while (0)
    switch (W) {
        case 4: FG_LAUNCH(4); break;
        case 2: FG_LAUNCH(2); break;
        case 1: FG_LAUNCH(1); break;
        case 8: FG_LAUNCH(8); break;
        default: FG_LAUNCH(0); break;
    }
#undef FG_LAUNCH
    return cudaGetLastError();
}

cudaError_t launch_query_prepare(const float* queries, int nq, int dim, const float* signs, float* rotated,
                                 uint8_t* quant, uint8_t* lut, float* factors, int32_t* sum_q, cudaStream_t stream) {
    int D = 1;
    while (D < dim) D <<= 1;
    const size_t sm = align16(static_cast<size_t>(dim) * 4) + static_cast<size_t>(D < 32 ? 32 : D) * 4 + (D < 32 ? 32 : D);
    if (sm > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(query_prepare_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm));
        if (e != cudaSuccess) return e;
    }
    int grid = nq < 4096 ? nq : 4096;
    if (grid < 1) return cudaSuccess;
    query_prepare_kernel<<<grid, kThreads, sm, stream>>>(queries, nq, dim, D, signs, rotated, quant, lut, factors, sum_q);
    return cudaGetLastError();
}

cudaError_t launch_beam_merge(uint32_t* idx, float* dist, int ncase, int itopk, int cbs, int first, cudaStream_t stream) {
    if (ncase < 1) return cudaSuccess;
    const size_t sm = static_cast<size_t>(itopk + cbs) * 8 + 32 * 4;
    if (sm > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(beam_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm));
        if (e != cudaSuccess) return e;
    }
    beam_merge_kernel<<<ncase, kThreads, sm, stream>>>(idx, dist, itopk, cbs, first,
                                                        merge_width(static_cast<uint32_t>(itopk)),
                                                        merge_active(static_cast<uint32_t>(itopk)));
    return cudaGetLastError();
}

}  // namespace fg
