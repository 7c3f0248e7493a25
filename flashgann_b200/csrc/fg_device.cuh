// fg_device.cuh -- device building blocks of the search (included by both
// kernels, fg_search.cu and fg_search_warp.cu): the warp bitonic network, the
// CTA kernel's visited set, query
// rotation/quantisation, bit-plane RaBitQ estimates, exact distances, the
// adaptive controller and both beam merges.
//
// What is computed is the reference's (SophiaSun18/FlashGANN,
// src/adaptive_search.cuh and include/utils.cuh, cited per function); how is
// this build's own:
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
#pragma once

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

// Per-CTA shape of a kernel variant with NW warps per query.
template <int NW>
struct Cfg {
    static constexpr int kThreads = NW * 32;
    // merge-path segments per thread (BLOCK_SIZE caps the reference's segments)
    static constexpr int kSegPerThread = (BLOCK_SIZE + kThreads - 1) / kThreads;
    // parents of one speculative iteration handled by one warp
    static constexpr int kTasksPerWarp = (SEARCH_WIDTH + NW - 1) / NW;
};

// rows whose exact distance one warp evaluates at once (all of a warp's rows
// are prefetched into L2 first, so later batches do not wait on HBM)
constexpr int kEvalBatch = 4;

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
// An exact set of node ids: Fibonacci hashing (spreads the consecutive ids of
// one mixture component) into buckets of 4 slots probed linearly, one 128-bit
// shared load per bucket.  Membership answers equal the reference table's
// (include/utils.cuh:683-750) because neither table ever fills: at most
// beam + 32 * SMALL_HASH_RESET_INTERVAL keys live between resets and the
// capacity is >= 4/3 of that.  Keys are inserted into the first empty slot
// of their probe order, so a lookup may stop at the first empty slot.
__device__ __forceinline__ uint32_t h_bucket(uint32_t key, int hbits) {
    return ((key * 0x9E3779B1u) >> (32 - hbits)) & ~3u;
}

__device__ __forceinline__ bool h_insert(uint32_t* t, int hbits, uint32_t key) {
    const uint32_t mask = (1u << hbits) - 1u;
    uint32_t b = h_bucket(key, hbits);
    for (uint32_t n = 0; n <= mask; n += 4) {
        const uint4 v = *reinterpret_cast<const uint4*>(t + b);
        const uint32_t s[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (s[j] == key) return false;
            if (s[j] == kMax) {
                const uint32_t old = atomicCAS(&t[b + j], kMax, key);
                if (old == kMax) return true;
                if (old == key) return false;
            }
        }
        b = (b + 4) & mask;
    }
    return false;
}

__device__ __forceinline__ bool h_contains(const uint32_t* t, int hbits, uint32_t key) {
    const uint32_t mask = (1u << hbits) - 1u;
    uint32_t b = h_bucket(key, hbits);
    for (uint32_t n = 0; n <= mask; n += 4) {
        const uint4 v = *reinterpret_cast<const uint4*>(t + b);
        if (v.x == key || v.y == key || v.z == key || v.w == key) return true;
        if (v.x == kMax || v.y == kMax || v.z == kMax || v.w == kMax) return false;
        b = (b + 4) & mask;
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
template <int NW>
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
        red_f[NW + warp] = hi;
    }
    __syncthreads();
    lo = FLT_MAX;
    hi = -FLT_MAX;
    for (int w = 0; w < NW; ++w) {
        lo = fminf(lo, red_f[w]);
        hi = fmaxf(hi, red_f[NW + w]);
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
        for (int w = 0; w < NW; ++w) s += red_i[w];
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

// One warp computes up to B distances at once: every row load is
// issued before any reduction.  Per lane the accumulation runs over dims
// lane, lane+32, ... with fused multiply-adds, then the shfl_down tree
// (include/utils.cuh:270-305).
template <int B>
__device__ void eval_rows(const float* __restrict__ rows, uint64_t row, int dim, const float* qvec,
                          const uint32_t* nodes, int count, int use_ip, float* out, int lane) {
    float acc[B];
#pragma unroll
    for (int b = 0; b < B; ++b) acc[b] = 0.0f;
    for (int d0 = 0; d0 < dim; d0 += 128) {
        float v[B][4];
#pragma unroll
        for (int b = 0; b < B; ++b) {
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
                for (int b = 0; b < B; ++b) {
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
    for (int b = 0; b < B; ++b) {
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

// BUFFER_BOUND / theta for theta in [1, 32] (theta <= THETA_MAX <= SEARCH_WIDTH <= 32)
__constant__ uint8_t c_bound[33] = {
    0, BUFFER_BOUND / 1, BUFFER_BOUND / 2, BUFFER_BOUND / 3, BUFFER_BOUND / 4, BUFFER_BOUND / 5,
    BUFFER_BOUND / 6, BUFFER_BOUND / 7, BUFFER_BOUND / 8, BUFFER_BOUND / 9, BUFFER_BOUND / 10, BUFFER_BOUND / 11,
    BUFFER_BOUND / 12, BUFFER_BOUND / 13, BUFFER_BOUND / 14, BUFFER_BOUND / 15, BUFFER_BOUND / 16,
    BUFFER_BOUND / 17, BUFFER_BOUND / 18, BUFFER_BOUND / 19, BUFFER_BOUND / 20, BUFFER_BOUND / 21,
    BUFFER_BOUND / 22, BUFFER_BOUND / 23, BUFFER_BOUND / 24, BUFFER_BOUND / 25, BUFFER_BOUND / 26,
    BUFFER_BOUND / 27, BUFFER_BOUND / 28, BUFFER_BOUND / 29, BUFFER_BOUND / 30, BUFFER_BOUND / 31,
    BUFFER_BOUND / 32};

__device__ __forceinline__ int keep_for(uint32_t active, int theta, float rho, bool cut_valid, uint32_t near) {
    const int ac = static_cast<int>(active);
    const int rho_keep = static_cast<int>(keep_per_parent(active, rho));
    const uint32_t bound = c_bound[theta];
    const int budget = clamp_i(static_cast<int>(bound), 1, ac);
    int mk = rho_keep < budget ? rho_keep : budget;
    if (cut_valid) mk = clamp_i(static_cast<int>(near), 1, mk);
    return clamp_i(mk, 1, ac);
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
// itopk % 32 != 0, in two steps.
//
// mp_prepare (warp 0): sorts the candidate buffer with the reference's
// 32-lane network and records, for candidate m, its position in the stable
// (beam-first) merge, pos[m] = m + #{beam entries <= cand[m]}, and the first
// position the merge can change, *p0 = #{beam entries < cand[0]}.
__device__ __forceinline__ void mp_prepare(const float* bdist, uint32_t* cidx, float* cdist, uint32_t cbs,
                                           uint32_t itopk, uint32_t* pos, uint32_t* p0, int lane) {
    float k = lane < static_cast<int>(cbs) ? cdist[lane] : FLT_MAX;
    uint32_t v = lane < static_cast<int>(cbs) ? cidx[lane] : kMax;
    sort32(k, v, lane);
    if (lane < static_cast<int>(cbs)) {
        cdist[lane] = k;
        cidx[lane] = v;
        pos[lane] = static_cast<uint32_t>(lane) + upper_bound(bdist, itopk, k);
    }
    if (lane == 0) *p0 = lower_bound(bdist, itopk, k);
}

// mp_apply (whole CTA): output segment s covers [bnd[s], bnd[s+1]) with
// bnd[s] = s*itopk/active and is merged beam-first between the reference's
// partitions, reading the beam from (sidx, sdist) and writing the merged
// beam to (didx, ddist).  The caller synchronises afterwards.
template <int NW>
__device__ __forceinline__ void mp_apply(const uint32_t* sidx, const float* sdist, uint32_t* didx, float* ddist,
                                         const uint32_t* cidx, const float* cdist, uint32_t cbs, uint32_t itopk,
                                         int active, const uint16_t* bnd, const uint32_t* pos, uint32_t p0) {
    constexpr int S = Cfg<NW>::kSegPerThread;
    const int s0 = threadIdx.x * S;
#pragma unroll
    for (int sj = 0; sj < S; ++sj) {
        const int s = s0 + sj;
        if (s < active) {
            const int ob = bnd[s], oe = bnd[s + 1];
            if (oe <= static_cast<int>(p0)) {
                for (int o = ob; o < oe; ++o) {
                    ddist[o] = sdist[o];
                    didx[o] = sidx[o];
                }
            } else {
                int ti = split_at(ob, p0, pos, sdist, static_cast<int>(itopk), cdist, static_cast<int>(cbs));
                const int te = split_at(oe, p0, pos, sdist, static_cast<int>(itopk), cdist, static_cast<int>(cbs));
                int ci = ob - ti;
                const int ce = oe - te;
                for (int o = ob; o < oe; ++o) {
                    const bool take = (ci >= ce) || (ti < te && sdist[ti] <= cdist[ci]);
                    if (take) {
                        ddist[o] = sdist[ti];
                        didx[o] = sidx[ti];
                        ++ti;
                    } else {
                        ddist[o] = cdist[ci];
                        didx[o] = cidx[ci];
                        ++ci;
                    }
                }
            }
        }
    }
}

// ------------------------------------------------------- parent expansion
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

// One lane's slice of a parent's expansion block (neighbour `lane`).
template <int W>
struct ParentLane {
    uint32_t child;
    float tx, fdq, fvq;
    uint32_t c[W > 0 ? W : 1];
};

// Issue every load of a parent's block for this lane: id, the three factors
// and (for W > 0) the packed code words; nothing waits on them here.
template <int W>
__device__ __forceinline__ void load_parent(const float* __restrict__ prow, const SearchArgs& a, int limit, bool vec,
                                            int lane, ParentLane<W>& p) {
    const bool in = lane < limit;
    const uint32_t* ids = reinterpret_cast<const uint32_t*>(prow + a.nbr_off);
    const float* fac = prow + a.factor_off;
    p.child = in ? __ldg(ids + lane) : kMax;
    p.tx = in ? __ldg(fac + lane) : FLT_MAX;
    p.fdq = in ? __ldg(fac + a.degree + lane) : 0.0f;
    p.fvq = in ? __ldg(fac + 2 * a.degree + lane) : 0.0f;
    if constexpr (W > 0) {
        if (in) {
            load_codes<W>(prow, a.code_off, lane, vec, p.c);
        } else {
#pragma unroll
            for (int w = 0; w < W; ++w) p.c[w] = 0;
        }
    }
}

template <int W>
__device__ __forceinline__ uint32_t parent_raw(const ParentLane<W>& p, const float* __restrict__ prow,
                                               const SearchArgs& a, int lane, const uint32_t* planes,
                                               const uint32_t* wrap, bool wrap_any) {
    if constexpr (W > 0) {
        return raw_sum<W>(p.c, planes, wrap, wrap_any);
    } else {
        const int Wd = a.padded_dim >> 5;
        return raw_sum_dyn(reinterpret_cast<const uint32_t*>(prow + a.code_off) + static_cast<size_t>(lane) * Wd, Wd,
                           planes, wrap, wrap_any);
    }
}

// The adaptive controller's state (src/adaptive_search_utils.cuh:8-18), held
// in warp-0 registers: every lane computes the same (warp-uniform) values.
struct CtlRegs {
    int theta;
    float rho;
    int policy_iters;
    uint32_t top1;
    int stall;
    bool warmup_done;
    float entry_d, last_d, cur_d;
    uint32_t scan;  // merge path: beam positions before this hold expanded entries
};

// src/adaptive_search.cuh:167-190 with update_head_stall_counter,
// update_expander_progress, apply_stage2_state and update_adaptive_state
// (src/adaptive_search_utils.cuh:32-119).
__device__ __forceinline__ void controller_update(CtlRegs& c, uint32_t beam0, int iter, float phase2_rho) {
    const uint32_t top1 = beam0 & 0x7fffffffu;
    const int stall = (c.policy_iters > 0 && top1 == c.top1) ? c.stall + 1 : 0;
    const bool changed = c.warmup_done || stall >= TOP1_WARMUP_STALL_ITERS;
    const float e = c.entry_d;
    const float last = finite_lt_max(c.last_d) ? c.last_d : e;
    const float cur = finite_lt_max(c.cur_d) ? c.cur_d : last;
    c.top1 = top1;
    c.stall = stall;
    c.last_d = last;
    c.cur_d = cur;
    if (changed) {
        c.warmup_done = true;
        c.theta = PHASE2_THETA;
        c.rho = phase2_rho;
        c.policy_iters += 1;
    } else if (iter == 0 || (iter % CHECK_INTERVAL) == 0) {
        // expander progress (src/adaptive_search_utils.cuh:51-72), computed only where it is used
        float rate = 0.0f;
        const float denom = fabsf(e);
        if (isfinite(last) && isfinite(cur) && isfinite(e) && !(denom <= 1.0e-20f)) {
            const float prog = __fdiv_rn(__fsub_rn(last, cur), denom);
            if (isfinite(prog) && prog > 0.0f) rate = prog < 1.0f ? prog : 1.0f;
        }
        const float span = phase2_rho > PHASE1_RHO ? __fsub_rn(phase2_rho, PHASE1_RHO) : __fsub_rn(RHO_MAX, RHO_MIN);
        const float base = c.policy_iters == 0 ? PHASE1_RHO : c.rho;
        const float cap = phase2_rho > PHASE1_RHO ? phase2_rho : RHO_MAX;
        c.warmup_done = false;
        c.theta = PHASE1_THETA;
        c.rho = clamp_f(__fmaf_rn(span, rate, base), RHO_MIN, cap);
        c.policy_iters += 1;
    }
}

}  // namespace
}  // namespace fg
