/*
 * fg_oracle.c -- CPU restatement of FlashGANN's adaptive quantised beam search.
 *
 * TEST INFRASTRUCTURE ONLY (see fg_oracle.h).  Not part of the product: the
 * CUDA library never links it, and only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / reference legs load it.
 *
 * The restatement follows the reference kernel step by step.  Citations are
 * file:line inside the reference project (SophiaSun18/FlashGANN).  Where the
 * reference's own GPU execution is racy (concurrent hash inserts from
 * different warps in the speculative path), this file fixes one order: every
 * visited-set lookup of a round happens before that round's inserts, and a
 * child that appears more than once in a round is accepted for its first
 * occurrence in (task, lane) order.
 *
 * Floating point: compiled with -ffp-contract=off; the multiply-adds that
 * nvcc contracts in the reference build are written here as fmaf() and are
 * pinned by tests/golden (oracle/ref_harness.cu runs the reference's own
 * device functions on a B200).
 */
#include "fg_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define OG_WARP 32
#define OG_MAX_INDEX 0xFFFFFFFFu
#define OG_MSB 0x80000000u
#define OG_MAX_BEAM 1024

/* include/utils.cuh:68-78 */
static uint32_t rp2(uint32_t x) {
    if (x <= 1) return 1;
    --x;
    x |= x >> 1; x |= x >> 2; x |= x >> 4; x |= x >> 8; x |= x >> 16;
    return x + 1;
}

/* include/utils.cuh:88-102 */
static int clamp_i(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }
static float clamp_f(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

void og_default_knobs(og_knobs* k) {
    k->block_size = 256;
    k->search_width = 8;
    k->theta_min = 1;
    k->theta_max = 8;
    k->rho_min = 0.0f;
    k->rho_max = 0.99f;
    k->min_phase2_keep = 4;
    k->check_interval = 1;
    k->buffer_bound = 32;
    k->phase1_theta = 1;
    k->phase1_rho = 0.25f;
    k->phase2_theta = 8;
    k->stall_iters = 4;
    k->max_iterations = 1 << 10;
    k->reset_interval = 16;
    k->hash_base_bitlen = 11;
}

/* include/qg.hpp:66-73 */
void og_compute_layout(uint64_t dim, int degree, og_layout* L) {
    uint64_t D = 1;
    while (D < dim) D <<= 1;
    L->dim = dim;
    L->padded_dim = D;
    L->degree = degree;
    L->code_off = dim;
    L->factor_off = dim + (D / 64) * 2 * (uint64_t)degree;
    L->nbr_off = L->factor_off + 3 * (uint64_t)degree;
    L->row = L->nbr_off + (uint64_t)degree;
}

/* include/utils.cuh:119-127 */
uint32_t og_effective_sort_beam(uint32_t beam) {
    if (beam == 0) return 0;
    uint32_t r = rp2(beam);
    if (r <= 128) return r < OG_WARP ? OG_WARP : r;
    return beam;
}

/* src/adaptive_search_utils.cuh:231-236 + round_up_power2 at gpu_search_adaptive.cu:17 */
uint32_t og_candidate_buffer_size(int degree, const og_knobs* kn) {
    uint32_t maxcap = (uint32_t)kn->theta_max * (uint32_t)degree;
    uint32_t cap = (uint32_t)kn->buffer_bound;
    if (cap > maxcap) cap = maxcap;
    return rp2(cap);
}

/* include/utils.cuh:137-151 */
uint32_t og_hash_bitlen(uint32_t padded_beam, uint32_t cand_buf, uint32_t reset_interval,
                        uint32_t base_bitlen) {
    uint64_t req64 = (uint64_t)padded_beam + (uint64_t)cand_buf * reset_interval;
    uint32_t req = req64 > 0xffffffffull ? 0xffffffffu : (uint32_t)req64;
    uint32_t target = (req * 4u + 2u) / 3u;
    uint32_t cap = 1u << base_bitlen;
    while (cap < target) cap <<= 1;
    uint32_t b = 0;
    while ((1u << b) < cap) ++b;
    return b;
}

/* ---------------- visited hash: include/utils.cuh:683-750 ---------------- */
static void hash_init(uint32_t* t, unsigned bitlen) { memset(t, 0xff, sizeof(uint32_t) << bitlen); }

static uint32_t hash_insert(uint32_t* t, unsigned bitlen, uint32_t key) {
    const uint32_t size = 1u << bitlen, mask = size - 1;
    uint32_t i = (key ^ (key >> bitlen)) & mask;
    for (uint32_t n = 0; n < size; ++n) {
        uint32_t old = t[i];
        if (old == OG_MAX_INDEX) { t[i] = key; return 1; }
        if (old == key) return 0;
        i = (i + 1) & mask;
    }
    return 0;
}

static uint32_t hash_contains(const uint32_t* t, unsigned bitlen, uint32_t key) {
    const uint32_t size = 1u << bitlen, mask = size - 1;
    uint32_t i = (key ^ (key >> bitlen)) & mask;
    for (uint32_t n = 0; n < size; ++n) {
        uint32_t old = t[i];
        if (old == key) return 1;
        if (old == OG_MAX_INDEX) return 0;
        i = (i + 1) & mask;
    }
    return 0;
}

/* ------------- warp bitonic network: include/utils.cuh:307-414 -------------
 * A warp of 32 lanes holding N (key, value) registers each is simulated as an
 * array k[lane * N + i].  Compare-exchange never swaps equal keys
 * (utils.cuh:312,320); a shuffle step reads every lane's value before any lane
 * updates. */
static void sim_swap_shfl(float* k, uint32_t* v, int N, int i, unsigned c, const unsigned char* p) {
    float nk[OG_WARP];
    uint32_t nv[OG_WARP];
    for (int l = 0; l < OG_WARP; ++l) {
        float k0 = k[l * N + i], k1 = k[(l ^ (int)c) * N + i];
        uint32_t v0 = v[l * N + i], v1 = v[(l ^ (int)c) * N + i];
        if ((k0 != k1) && ((k0 < k1) != (p[l] != 0))) { nk[l] = k1; nv[l] = v1; }
        else { nk[l] = k0; nv[l] = v0; }
    }
    for (int l = 0; l < OG_WARP; ++l) { k[l * N + i] = nk[l]; v[l * N + i] = nv[l]; }
}

static void sim_swap_reg(float* k, uint32_t* v, int a, int b, int asc) {
    if ((k[a] != k[b]) && ((k[a] < k[b]) != (asc != 0))) {
        float tk = k[a]; k[a] = k[b]; k[b] = tk;
        uint32_t tv = v[a]; v[a] = v[b]; v[b] = tv;
    }
}

static void sim_warp_merge(float* k, uint32_t* v, int N, unsigned range) {
    unsigned char p[OG_WARP];
    if (N == 1) {
        if (range == 1) return;
        for (unsigned c = range / 2; c >= 1; c >>= 1) {
            for (int l = 0; l < OG_WARP; ++l) p[l] = (((unsigned)l & range) != 0) == (((unsigned)l & c) != 0);
            sim_swap_shfl(k, v, 1, 0, c, p);
        }
    } else if (N == 2) {
        if (range == 1) {
            for (int l = 0; l < OG_WARP; ++l) sim_swap_reg(k, v, l * 2, l * 2 + 1, (l & 1) == 0);
            return;
        }
        for (unsigned c = range / 2; c >= 1; c >>= 1) {
            for (int l = 0; l < OG_WARP; ++l) p[l] = (((unsigned)l & range) != 0) == (((unsigned)l & c) != 0);
            for (int i = 0; i < 2; ++i) sim_swap_shfl(k, v, 2, i, c, p);
        }
        for (int l = 0; l < OG_WARP; ++l) sim_swap_reg(k, v, l * 2, l * 2 + 1, ((unsigned)l & range) == 0);
    } else {
        if (range == 1) {
            for (int l = 0; l < OG_WARP; ++l)
                for (unsigned b = 2; b <= (unsigned)N; b <<= 1)
                    for (unsigned c = b / 2; c >= 1; c >>= 1)
                        for (int i = 0; i < N; ++i) {
                            int j = i ^ (int)c;
                            if (i >= j) continue;
                            unsigned line = (unsigned)i + (unsigned)N * (unsigned)l;
                            int asc = ((line & b) != 0) == ((line & c) != 0);
                            sim_swap_reg(k, v, l * N + i, l * N + j, asc);
                        }
            return;
        }
        for (unsigned c = range / 2; c >= 1; c >>= 1) {
            for (int l = 0; l < OG_WARP; ++l) p[l] = (((unsigned)l & range) != 0) == (((unsigned)l & c) != 0);
            for (int i = 0; i < N; ++i) sim_swap_shfl(k, v, N, i, c, p);
        }
        for (int l = 0; l < OG_WARP; ++l) {
            int asc = ((unsigned)l & range) == 0;
            for (unsigned c = (unsigned)N / 2; c >= 1; c >>= 1)
                for (int i = 0; i < N; ++i) {
                    int j = i ^ (int)c;
                    if (i >= j) continue;
                    sim_swap_reg(k, v, l * N + i, l * N + j, asc);
                }
        }
    }
}

static void sim_warp_sort(float* k, uint32_t* v, int N) {
    for (unsigned range = 1; range <= OG_WARP; range <<= 1) sim_warp_merge(k, v, N, range);
}

/* include/utils.cuh:417-457 with N_1 = 1 (every candidate buffer is <= 32). */
void og_candidate_sort(uint32_t* idx, float* dist, uint32_t cbs) {
    float k[OG_WARP];
    uint32_t v[OG_WARP];
    for (uint32_t l = 0; l < OG_WARP; ++l) {
        k[l] = l < cbs ? dist[l] : FLT_MAX;
        v[l] = l < cbs ? idx[l] : OG_MAX_INDEX;
    }
    sim_warp_sort(k, v, 1);
    for (uint32_t l = 0; l < OG_WARP && l < cbs; ++l) { dist[l] = k[l]; idx[l] = v[l]; }
}

/* include/utils.cuh:490-586 (topk_small_by_bitonic_sort<1, N2>). */
static void bitonic_topk(uint32_t* idx, float* dist, uint32_t cbs, uint32_t itopk, int first, int N2) {
    uint32_t* cidx = idx + itopk;
    float* cdist = dist + itopk;
    float k1[OG_WARP];
    uint32_t v1[OG_WARP];
    for (uint32_t l = 0; l < OG_WARP; ++l) {
        k1[l] = l < cbs ? cdist[l] : FLT_MAX;
        v1[l] = l < cbs ? cidx[l] : OG_MAX_INDEX;
    }
    sim_warp_sort(k1, v1, 1);
    for (uint32_t l = 0; l < OG_WARP; ++l)
        if (l < cbs && l < itopk) { cdist[l] = k1[l]; cidx[l] = v1[l]; }

    float k2[OG_WARP * 4];
    uint32_t v2[OG_WARP * 4];
    for (int l = 0; l < OG_WARP; ++l)
        for (int i = 0; i < N2; ++i) {
            uint32_t j = first ? (uint32_t)(l + 32 * i) : (uint32_t)(N2 * l + i);
            k2[l * N2 + i] = j < itopk ? dist[j] : FLT_MAX;
            v2[l * N2 + i] = j < itopk ? idx[j] : OG_MAX_INDEX;
        }
    if (first) sim_warp_sort(k2, v2, N2);
    for (int l = 0; l < OG_WARP; ++l)
        for (int i = 0; i < N2; ++i) {
            uint32_t j = (uint32_t)(N2 * l + i);
            uint32_t kk = itopk - 1u - j;
            if (kk >= itopk || kk >= cbs) continue;
            if (k2[l * N2 + i] > cdist[kk]) { k2[l * N2 + i] = cdist[kk]; v2[l * N2 + i] = cidx[kk]; }
        }
    sim_warp_merge(k2, v2, N2, 32);
    for (int l = 0; l < OG_WARP; ++l)
        for (int i = 0; i < N2; ++i) {
            uint32_t j = (uint32_t)(N2 * l + i);
            if (j < itopk) { dist[j] = k2[l * N2 + i]; idx[j] = v2[l * N2 + i]; }
        }
}

/* include/utils.cuh:588-616 */
static int mp_partition(const float* a, int an, const float* b, int bn, int diag) {
    int lo = diag - bn > 0 ? diag - bn : 0;
    int hi = diag < an ? diag : an;
    while (lo <= hi) {
        int ai = (lo + hi) >> 1, bi = diag - ai;
        float al = ai > 0 ? a[ai - 1] : -FLT_MAX;
        float ar = ai < an ? a[ai] : FLT_MAX;
        float bl = bi > 0 ? b[bi - 1] : -FLT_MAX;
        float br = bi < bn ? b[bi] : FLT_MAX;
        if (al > br) hi = ai - 1;
        else if (bl > ar) lo = ai + 1;
        else return ai;
    }
    return lo;
}

/* include/utils.cuh:618-680 (merge-path with per-thread output segments). */
static void mergepath_topk(uint32_t* idx, float* dist, uint32_t cbs, uint32_t itopk, int block_size) {
    uint32_t* cidx = idx + itopk;
    float* cdist = dist + itopk;
    og_candidate_sort(cidx, cdist, cbs);
    int active = (int)((itopk + 3) / 4);
    active = ((active + 31) / 32) * 32;
    if (active > block_size) active = block_size;
    uint32_t* sidx = (uint32_t*)malloc(sizeof(uint32_t) * itopk);
    float* sdist = (float*)malloc(sizeof(float) * itopk);
    for (int t = 0; t < active; ++t) {
        int ob = (int)(((uint32_t)t * itopk) / (uint32_t)active);
        int oe = (int)(((uint32_t)(t + 1) * itopk) / (uint32_t)active);
        if (ob > (int)itopk) ob = (int)itopk;
        if (oe > (int)itopk) oe = (int)itopk;
        int tb = mp_partition(dist, (int)itopk, cdist, (int)cbs, ob);
        int te = mp_partition(dist, (int)itopk, cdist, (int)cbs, oe);
        int ti = tb, ci = ob - tb, ce = oe - te;
        for (int o = ob; o < oe; ++o) {
            int take = (ci >= ce) || (ti < te && dist[ti] <= cdist[ci]);
            if (take) { sdist[o] = dist[ti]; sidx[o] = idx[ti]; ++ti; }
            else { sdist[o] = cdist[ci]; sidx[o] = cidx[ci]; ++ci; }
        }
    }
    memcpy(idx, sidx, sizeof(uint32_t) * itopk);
    memcpy(dist, sdist, sizeof(float) * itopk);
    free(sidx);
    free(sdist);
}

/* include/utils.cuh:1369-1399 with the width dispatch of :1134-1367. */
int og_beam_merge(uint32_t* idx, float* dist, uint32_t cbs, uint32_t itopk, int first, int block_size) {
    if (cbs == 0 || cbs > OG_WARP || itopk == 0) return OG_ERR_ARG;
    uint32_t n2 = (itopk + OG_WARP - 1) / OG_WARP;
    if (n2 > 32) n2 = 4; /* the dispatch's default case (utils.cuh:1360-1365) */
    if (itopk % OG_WARP == 0 && (n2 == 1 || n2 == 2 || n2 == 4))
        bitonic_topk(idx, dist, cbs, itopk, first, (int)n2);
    else
        mergepath_topk(idx, dist, cbs, itopk, block_size);
    return OG_OK;
}

/* min/max with -0 < +0 (the GPU's min.f32 / max.f32 on signed zeros) */
static float gpu_fminf(float a, float b) {
    if (a == b) return signbit(a) ? a : b;
    return fminf(a, b);
}
static float gpu_fmaxf(float a, float b) {
    if (a == b) return signbit(a) ? b : a;
    return fmaxf(a, b);
}

/* ----------------------- query preparation -----------------------
 * include/utils.cuh:790-821 (sign flip + unnormalised FWHT, stages len=1..D/2)
 * and :840-939 (6-bit quantisation, 16-entry nibble LUT, sum). */
void og_query_prepare(const float* q, const float* signs, int dim, int D, float* r, uint8_t* quant,
                      uint8_t* lut, og_qfactors* qf) {
    for (int i = 0; i < dim; ++i) r[i] = q[i] * signs[i];
    for (int i = dim; i < D; ++i) r[i] = 0.0f;
    for (int len = 1; len < D; len <<= 1) {
        int pairs = D >> 1;
        for (int pi = 0; pi < pairs; ++pi) {
            int blk = pi / len, j = pi % len, base = blk * (len << 1);
            int i1 = base + j, i2 = i1 + len;
            float u = r[i1], v = r[i2];
            r[i1] = u + v;
            r[i2] = u - v;
        }
    }
    /* The reference's min/max tree runs on the GPU, whose min.f32 / max.f32
     * order -0 below +0; with that rule the result does not depend on the
     * reduction order, so a sequential scan gives the same bits. */
    float lo = FLT_MAX, hi = -FLT_MAX;
    for (int i = 0; i < D; ++i) { lo = gpu_fminf(lo, r[i]); hi = gpu_fmaxf(hi, r[i]); }
    const float kinv = 1.0f / 63.0f; /* (1 << QG_BQUERY) - 1, include/common.hpp:17 */
    qf->low = lo;
    qf->high = hi;
    qf->width = (hi - lo) * kinv;
    const float inv_w = 1.0f / qf->width;
    int32_t sum = 0;
    for (int cb = 0; cb < (D >> 2); ++cb) {
        uint8_t qq[4];
        for (int j = 0; j < 4; ++j) {
            int id = (cb << 2) + j;
            float scaled = fmaf(r[id] - lo, inv_w, 0.5f);
            qq[j] = (uint8_t)lroundf(scaled);
            quant[id] = qq[j];
            sum += qq[j];
        }
        uint8_t* c = lut + (cb << 4);
        c[0] = 0;
        for (int m = 1; m < 16; ++m) {
            int lb = m & -m;
            int pos = (lb == 8) ? 0 : ((lb == 4) ? 1 : ((lb == 2) ? 2 : 3));
            c[m] = (uint8_t)(c[m - lb] + qq[pos]);
        }
    }
    qf->sum_q = sum;
}

/* include/utils.cuh:941-1027: one neighbour's estimate; the integer LUT sum is
 * identical for the 8-lane and the 1-lane variants. */
float og_estimate(const uint8_t* lut, const og_qfactors* qf, const uint8_t* codes, int ni, int D,
                  float tx, float fdq, float fvq, float pdist, int zero_on_invalid) {
    if (tx == FLT_MAX) return zero_on_invalid ? 0.0f : FLT_MAX;
    const uint8_t* c = codes + (size_t)ni * (size_t)(D >> 3);
    uint32_t raw = 0;
    for (int cb = 0; cb < (D >> 2); ++cb) {
        uint8_t packed = c[cb >> 1];
        uint8_t code = (cb & 1) ? (uint8_t)(packed >> 4) : (uint8_t)(packed & 0x0f);
        raw += lut[(cb << 4) + code];
    }
    float rf = (float)((int32_t)(raw << 1) - qf->sum_q);
    float est = tx + pdist;
    est = fmaf(fdq * qf->width, rf, est);
    est = fmaf(fvq, qf->low, est);
    return est;
}

/* include/utils.cuh:270-305: lane-strided fused accumulation, then a
 * shfl_down tree (16, 8, 4, 2, 1) read at lane 0. */
float og_warp_distance(int dim, const float* a, const float* b, int use_ip) {
    float s[OG_WARP];
    for (int l = 0; l < OG_WARP; ++l) {
        float val = 0.0f;
        for (int i = l; i < dim; i += OG_WARP) {
            if (use_ip) val = fmaf(a[i], b[i], val);
            else { float d = a[i] - b[i]; val = fmaf(d, d, val); }
        }
        s[l] = val;
    }
    for (int off = 16; off >= 1; off >>= 1)
        for (int l = 0; l < off; ++l) s[l] = s[l] + s[l + off];
    return use_ip ? -s[0] : s[0];
}

/* ------------------- adaptive controller -------------------
 * src/adaptive_search_utils.cuh:8-135 */
typedef struct ctrl_state {
    int theta;
    float rho;
    int policy_iters;
    uint32_t top1;
    int stall;
    int warmup_done;
    float entry_d, last_d, cur_d;
} ctrl_state;

static float max_rho_bound(int degree, const og_knobs* kn) {
    if ((uint32_t)degree <= (uint32_t)kn->min_phase2_keep) return kn->rho_min;
    return 1.0f - (float)kn->min_phase2_keep / (float)degree;
}

static int finite_lt_max(float x) { return isfinite(x) && x < FLT_MAX; }

static float expander_progress(const ctrl_state* s, float* last, float* cur) {
    float e = s->entry_d;
    *last = finite_lt_max(s->last_d) ? s->last_d : e;
    *cur = finite_lt_max(s->cur_d) ? s->cur_d : *last;
    float denom = fabsf(e);
    if (!isfinite(*last) || !isfinite(*cur) || !isfinite(e) || denom <= 1.0e-20f) return 0.0f;
    float prog = (*last - *cur) / denom;
    if (!isfinite(prog) || prog <= 0.0f) return 0.0f;
    return prog < 1.0f ? prog : 1.0f;
}

/* include/utils.cuh:104-117 */
static uint32_t keep_per_parent(uint32_t maxdeg, float rho) {
    float kf = 1.0f - rho;
    if (kf < 0.0f) kf = 0.0f;
    if (kf > 1.0f) kf = 1.0f;
    uint32_t kc = (uint32_t)ceilf((float)maxdeg * kf);
    if (kc < 1) kc = 1;
    if (kc > maxdeg) kc = maxdeg;
    return kc;
}

/* src/adaptive_search_utils.cuh:121-135 */
static int keep_for_expander(uint32_t active, const ctrl_state* s, const og_knobs* kn, int cut_valid,
                             uint32_t near) {
    int ac = (int)active;
    int rho_keep = (int)keep_per_parent(active, s->rho);
    uint32_t bound = (uint32_t)kn->buffer_bound / (uint32_t)s->theta;
    int budget = clamp_i((int)bound, 1, ac);
    int mk = rho_keep < budget ? rho_keep : budget;
    if (cut_valid) mk = clamp_i((int)near, 1, mk);
    return clamp_i(mk, 1, ac);
}

/* update_adaptive_state's rho and keep_count_for_expander for one case
 * (src/adaptive_search_utils.cuh:177-221), exposed for the golden tests. */
void og_rho_update(float rho_prev, int policy_iters, float rate, float phase2_rho, uint32_t active, int cut_valid,
                   uint32_t near, const og_knobs* kn, float* rho_out, int* keep_out) {
    ctrl_state s;
    memset(&s, 0, sizeof(s));
    s.rho = rho_prev;
    s.policy_iters = policy_iters;
    float span = phase2_rho > kn->phase1_rho ? phase2_rho - kn->phase1_rho : kn->rho_max - kn->rho_min;
    float base = policy_iters == 0 ? kn->phase1_rho : rho_prev;
    float cap = phase2_rho > kn->phase1_rho ? phase2_rho : kn->rho_max;
    s.rho = clamp_f(fmaf(span, rate, base), kn->rho_min, cap);
    s.theta = kn->phase1_theta;
    *rho_out = s.rho;
    *keep_out = keep_for_expander(active, &s, kn, cut_valid, near);
}

/* src/adaptive_search.cuh:167-190 with :32-39, :51-119 of the utils header. */
static void controller_step(ctrl_state* s, const uint32_t* beam_idx, int iter, float phase2_rho,
                            const og_knobs* kn) {
    uint32_t top1 = beam_idx[0] & 0x7fffffffu;
    int stall = (s->policy_iters > 0 && top1 == s->top1) ? s->stall + 1 : 0;
    int changed = s->warmup_done || stall >= kn->stall_iters;
    float last, cur;
    float rate = expander_progress(s, &last, &cur);
    if (changed) {
        s->top1 = top1;
        s->stall = stall;
        s->warmup_done = 1;
        s->last_d = last;
        s->cur_d = cur;
        s->theta = kn->phase2_theta;
        s->rho = phase2_rho;
        s->policy_iters += 1;
    } else if (iter == 0 || (iter % kn->check_interval) == 0) {
        float span = phase2_rho > kn->phase1_rho ? phase2_rho - kn->phase1_rho : kn->rho_max - kn->rho_min;
        float base = s->policy_iters == 0 ? kn->phase1_rho : s->rho;
        float cap = phase2_rho > kn->phase1_rho ? phase2_rho : kn->rho_max;
        float next = clamp_f(fmaf(span, rate, base), kn->rho_min, cap);
        s->top1 = top1;
        s->stall = stall;
        s->warmup_done = 0;
        s->last_d = last;
        s->cur_d = cur;
        s->theta = kn->phase1_theta;
        s->rho = next;
        s->policy_iters += 1;
    } else {
        s->top1 = top1;
        s->stall = stall;
        s->last_d = last;
        s->cur_d = cur;
    }
}

/* include/utils.cuh:752-787 */
static uint32_t pick_expanders(int N, uint32_t* out, int M, uint32_t* beam) {
    uint32_t num = 0;
    uint32_t mx = (uint32_t)M;
    if (mx % 32) mx += 32 - (mx % 32);
    for (uint32_t j0 = 0; j0 < mx; j0 += 32) {
        uint32_t ballot = 0;
        for (uint32_t l = 0; l < 32; ++l) {
            uint32_t j = j0 + l;
            if (j < (uint32_t)M && (beam[j] & OG_MSB) == 0) ballot |= 1u << l;
        }
        for (uint32_t l = 0; l < 32; ++l) {
            if (!(ballot & (1u << l))) continue;
            uint32_t i = (uint32_t)__builtin_popcount(ballot & ((1u << l) - 1u)) + num;
            if (i < (uint32_t)N) { out[i] = j0 + l; beam[j0 + l] |= OG_MSB; }
        }
        num += (uint32_t)__builtin_popcount(ballot);
        if (num > (uint32_t)N) num = (uint32_t)N;
        if (num >= (uint32_t)N) break;
    }
    return num;
}

static const float* row_of(const og_index* x, uint32_t node) { return x->data + (size_t)node * x->L.row; }

/* src/adaptive_search.cuh:5-466 */
int og_search_one(const og_index* x, const og_knobs* kn, const float* query, int K, int beam,
                  uint32_t* out_ids, float* out_dists, og_stats* st, og_trace* tr) {
    if (K < 1 || beam < 1 || beam > OG_MAX_BEAM || x->L.degree < 1) return OG_ERR_ARG;
    const int dim = (int)x->L.dim, D = (int)x->L.padded_dim, deg = x->L.degree;
    const int wpb = kn->block_size / OG_WARP;
    const int SW = kn->search_width;
    const uint32_t padded = og_effective_sort_beam((uint32_t)beam);
    const uint32_t cbs = og_candidate_buffer_size(deg, kn);
    uint32_t collect_cap = (uint32_t)kn->buffer_bound;
    if (collect_cap > cbs) collect_cap = cbs;
    const uint32_t bitlen = og_hash_bitlen(padded, cbs, (uint32_t)kn->reset_interval, (uint32_t)kn->hash_base_bitlen);
    const float phase2_rho = max_rho_bound(deg, kn);
    const int max_iter = (beam * 11 + 9) / 10;
    const int use_ip = x->use_ip;

    uint32_t* all_idx = (uint32_t*)malloc(sizeof(uint32_t) * (padded + cbs));
    float* all_dist = (float*)malloc(sizeof(float) * (padded + cbs));
    uint32_t* hash = (uint32_t*)malloc(sizeof(uint32_t) << bitlen);
    uint32_t* ppos = (uint32_t*)malloc(sizeof(uint32_t) * SW);
    uint32_t* pnode = (uint32_t*)malloc(sizeof(uint32_t) * SW);
    float* pdist = (float*)malloc(sizeof(float) * SW);
    float* rot = (float*)malloc(sizeof(float) * D);
    uint8_t* quant = (uint8_t*)malloc((size_t)D);
    uint8_t* lut = (uint8_t*)malloc((size_t)D * 4);
    /* speculative-path scratch: one round of wpb tasks x 32 lanes */
    uint32_t* t_child = (uint32_t*)malloc(sizeof(uint32_t) * wpb * 32);
    unsigned char* t_keep = (unsigned char*)malloc((size_t)wpb * 32);
    uint32_t* beam_idx = all_idx;
    float* beam_dist = all_dist;
    uint32_t* cidx = all_idx + padded;
    float* cdist = all_dist + padded;

    ctrl_state s;
    s.theta = kn->phase1_theta;
    s.rho = kn->phase1_rho;
    s.policy_iters = 0;
    s.top1 = OG_MAX_INDEX;
    s.stall = 0;
    s.warmup_done = 0;
    s.entry_d = FLT_MAX;
    s.last_d = FLT_MAX;
    s.cur_d = FLT_MAX;
    og_stats local;
    memset(&local, 0, sizeof(local));

    hash_init(hash, bitlen);
    for (uint32_t i = 0; i < padded + cbs; ++i) { all_idx[i] = OG_MAX_INDEX; all_dist[i] = FLT_MAX; }
    for (int i = 0; i < SW; ++i) { pnode[i] = OG_MAX_INDEX; pdist[i] = FLT_MAX; }

    /* :110-118 entry point into candidate slot 0 */
    float ed = og_warp_distance(dim, query, row_of(x, x->entry_point), use_ip);
    cidx[0] = x->entry_point;
    cdist[0] = ed;
    s.entry_d = ed;
    hash_insert(hash, bitlen, x->entry_point);
    local.evaluations = 1;

    og_qfactors qf;
    og_query_prepare(query, x->signs, dim, D, rot, quant, lut, &qf);

    int traced = 0;
    for (int iter = 0; iter < kn->max_iterations; ++iter) {
        if ((iter + 1) % kn->reset_interval == 0) {
            hash_init(hash, bitlen);
            for (int i = 0; i < beam; ++i) hash_insert(hash, bitlen, beam_idx[i] & ~OG_MSB);
        }
        if (iter >= max_iter) break;

        og_beam_merge(all_idx, all_dist, cbs, padded, iter == 0, kn->block_size);
        local.iterations++;
        for (uint32_t i = (uint32_t)beam; i < padded; ++i) { beam_idx[i] = OG_MAX_INDEX; beam_dist[i] = FLT_MAX; }
        for (uint32_t i = 0; i < cbs; ++i) { cidx[i] = OG_MAX_INDEX; cdist[i] = FLT_MAX; }
        for (int i = 0; i < SW; ++i) { pnode[i] = OG_MAX_INDEX; pdist[i] = FLT_MAX; }
        uint32_t compact = 0;
        /* :25-30 of the utils header */
        float cutoff;
        if (beam_idx[beam - 1] == OG_MAX_INDEX) cutoff = FLT_MAX;
        else cutoff = beam_dist[(K < beam ? K : beam) - 1];

        int was_phase2 = s.warmup_done;
        controller_step(&s, beam_idx, iter, phase2_rho, kn);
        if (!was_phase2 && s.warmup_done && local.phase2_iter == 0) local.phase2_iter = (uint64_t)iter;

        uint32_t keep_exp = pick_expanders(s.theta, ppos, beam, beam_idx);
        if (!keep_exp) break;
        for (int p = 0; p < SW; ++p)
            if (p < (int)keep_exp) {
                pnode[p] = beam_idx[ppos[p]] & 0x7fffffffu;
                pdist[p] = beam_dist[ppos[p]];
            }
        if (tr && traced < tr->trace_cap) {
            for (int p = 0; p < SW; ++p) tr->trace[(size_t)traced * SW + p] = p < (int)keep_exp ? pnode[p] : OG_MAX_INDEX;
            tr->trace_count[traced] = (int32_t)keep_exp;
            traced++;
        }
        local.expansions += keep_exp;
        /* record_selected_expander_dist (:41-49 of the utils header) */
        {
            float sel = pdist[keep_exp - 1];
            s.last_d = finite_lt_max(s.cur_d) ? s.cur_d : s.entry_d;
            s.cur_d = sel;
        }
        const float cut_ok = isfinite(cutoff) && cutoff < FLT_MAX;

        if (!(s.theta > 1)) {
            /* :221-343 single expander */
            const uint32_t work = (uint32_t)deg < cbs ? (uint32_t)deg : cbs;
            const uint32_t pn = pnode[0];
            const int pvalid = pn != OG_MAX_INDEX;
            const float* prow = pvalid ? row_of(x, pn) : NULL;
            const uint32_t* nb = pvalid ? (const uint32_t*)(prow + x->L.nbr_off) : NULL;
            for (uint32_t i = 0; i < cbs; ++i) {
                uint32_t ch = OG_MAX_INDEX;
                if (i < work && pvalid) {
                    ch = nb[i];
                    if (ch >= x->n || hash_contains(hash, bitlen, ch)) ch = OG_MAX_INDEX;
                }
                cidx[i] = ch;
                cdist[i] = ch == OG_MAX_INDEX ? FLT_MAX : 0.0f;
            }
            int keep = keep_for_expander(work, &s, kn, 0, 0);
            uint32_t vcount = 0;
            for (uint32_t i = 0; i < work; ++i) vcount += (cidx[i] != OG_MAX_INDEX && cdist[i] < FLT_MAX);
            int keep_all = keep >= (int)vcount;
            int eff = keep;
            if (!keep_all) {
                const float* fac = prow + x->L.factor_off;
                const uint8_t* codes = (const uint8_t*)(prow + x->L.code_off);
                for (uint32_t i = 0; i < work; ++i) {
                    if (cidx[i] == OG_MAX_INDEX) continue;
                    float est = og_estimate(lut, &qf, codes, (int)i, D, fac[i], fac[deg + i], fac[2 * deg + i], pdist[0], 1);
                    local.estimates++;
                    int ok = isfinite(est);
                    cdist[i] = ok ? est : FLT_MAX;
                    if (!ok) cidx[i] = OG_MAX_INDEX;
                }
                uint32_t near = 0;
                if (cut_ok)
                    for (uint32_t i = 0; i < work; ++i)
                        if (cidx[i] != OG_MAX_INDEX && isfinite(cdist[i]) && cdist[i] <= cutoff) near++;
                eff = keep_for_expander(work, &s, kn, cut_ok, near);
                og_candidate_sort(cidx, cdist, cbs);
                for (uint32_t i = 0; i < cbs; ++i)
                    if ((int)i >= eff) { cidx[i] = OG_MAX_INDEX; cdist[i] = FLT_MAX; }
            }
            const int admit = keep_all ? (int)work : eff;
            for (int i = 0; i < admit; ++i) {
                uint32_t ch = cidx[i];
                uint32_t ins = 0;
                if (ch != OG_MAX_INDEX && cdist[i] < FLT_MAX) ins = hash_insert(hash, bitlen, ch);
                if (!ins) { cidx[i] = OG_MAX_INDEX; cdist[i] = FLT_MAX; }
                else { cdist[i] = og_warp_distance(dim, query, row_of(x, ch), use_ip); local.evaluations++; }
            }
        } else {
            /* :344-444 speculative multi-expander */
            const int tiles = (deg + OG_WARP - 1) / OG_WARP;
            const int tasks = (int)keep_exp * tiles;
            for (int rb = 0; rb < tasks; rb += wpb) {
                int nt = tasks - rb < wpb ? tasks - rb : wpb;
                /* every lookup of the round precedes the round's inserts */
                for (int w = 0; w < nt; ++w) {
                    int task = rb + w;
                    int pi = task / tiles, tile = task - pi * tiles;
                    const float* prow = row_of(x, pnode[pi]);
                    const uint32_t* nb = (const uint32_t*)(prow + x->L.nbr_off);
                    const float* fac = prow + x->L.factor_off;
                    const uint8_t* codes = (const uint8_t*)(prow + x->L.code_off);
                    uint32_t child[32];
                    int valid[32];
                    float tx[32], fdq[32], fvq[32], est[32];
                    for (int l = 0; l < 32; ++l) {
                        uint32_t ni = (uint32_t)(tile * 32 + l);
                        child[l] = OG_MAX_INDEX;
                        valid[l] = 0;
                        tx[l] = FLT_MAX; fdq[l] = 0.0f; fvq[l] = 0.0f;
                        if (ni < (uint32_t)deg) {
                            child[l] = nb[ni];
                            valid[l] = child[l] != OG_MAX_INDEX && child[l] < x->n && !hash_contains(hash, bitlen, child[l]);
                            if (valid[l]) { tx[l] = fac[ni]; fdq[l] = fac[deg + ni]; fvq[l] = fac[2 * deg + ni]; }
                        }
                    }
                    uint32_t active = (uint32_t)(deg - tile * 32);
                    if (active > 32) active = 32;
                    int keep = keep_for_expander(active, &s, kn, 0, 0);
                    int raw_valid = 0;
                    for (int l = 0; l < 32; ++l) raw_valid += valid[l];
                    int keep_all = keep >= raw_valid;
                    for (int l = 0; l < 32; ++l) {
                        est[l] = FLT_MAX;
                        if (!keep_all && valid[l]) {
                            est[l] = og_estimate(lut, &qf, codes, tile * 32 + l, D, tx[l], fdq[l], fvq[l], pdist[pi], 0);
                            local.estimates++;
                            valid[l] = isfinite(est[l]);
                        }
                    }
                    int eff = keep;
                    if (!keep_all) {
                        uint32_t near = 0;
                        for (int l = 0; l < 32; ++l) near += (valid[l] && cut_ok && est[l] <= cutoff);
                        eff = keep_for_expander(active, &s, kn, cut_ok, near);
                    }
                    for (int l = 0; l < 32; ++l) {
                        int kl;
                        if (keep_all) kl = valid[l];
                        else {
                            /* include/utils.cuh:251-267 */
                            float mine = valid[l] ? est[l] : FLT_MAX;
                            int rank = 0;
                            for (int src = 0; src < 32; ++src) {
                                float other = valid[src] ? est[src] : FLT_MAX;
                                if (valid[src] && (other < mine || (other == mine && src < l))) rank++;
                            }
                            kl = valid[l] && eff > 0 && rank < eff;
                        }
                        t_child[w * 32 + l] = child[l];
                        t_keep[w * 32 + l] = (unsigned char)kl;
                    }
                }
                /* inserts and compaction in (task, lane) order */
                for (int w = 0; w < nt; ++w)
                    for (int l = 0; l < 32; ++l) {
                        if (!t_keep[w * 32 + l]) continue;
                        if (!hash_insert(hash, bitlen, t_child[w * 32 + l])) continue;
                        if (compact < collect_cap) { cidx[compact] = t_child[w * 32 + l]; cdist[compact] = FLT_MAX; }
                        compact++;
                    }
            }
            if (compact > collect_cap) compact = collect_cap;
            for (uint32_t i = 0; i < compact; ++i) {
                cdist[i] = og_warp_distance(dim, query, row_of(x, cidx[i]), use_ip);
                local.evaluations++;
            }
        }
    }
    og_beam_merge(all_idx, all_dist, cbs, padded, 0, kn->block_size);

    /* :455-464 */
    uint32_t last = 0;
    float last_d = FLT_MAX;
    for (int i = 0; i < K; ++i) {
        uint32_t r = i < beam ? (beam_idx[i] & 0x7fffffffu) : OG_MAX_INDEX;
        float rd = i < beam ? beam_dist[i] : last_d;
        if (r != OG_MAX_INDEX) { last = r; last_d = rd; }
        out_ids[i] = r == OG_MAX_INDEX ? last : r;
        if (out_dists) out_dists[i] = r == OG_MAX_INDEX ? last_d : rd;
    }
    if (tr) tr->n_iters = traced;
    if (st) *st = local;

    free(all_idx); free(all_dist); free(hash); free(ppos); free(pnode); free(pdist);
    free(rot); free(quant); free(lut); free(t_child); free(t_keep);
    return OG_OK;
}

int og_search_batch(const og_index* x, const og_knobs* kn, int nq, const float* queries, int K, int beam,
                    uint32_t* out_ids, int threads, og_stats* total) {
    if (nq < 0 || K < 1 || beam < 1 || beam > OG_MAX_BEAM) return OG_ERR_ARG;
    uint64_t it = 0, ex = 0, ev = 0, es = 0;
    int err = 0;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for num_threads(threads) schedule(dynamic, 4) reduction(+ : it, ex, ev, es) reduction(| : err)
#endif
    for (int q = 0; q < nq; ++q) {
        og_stats s;
        err |= og_search_one(x, kn, queries + (size_t)q * x->L.dim, K, beam, out_ids + (size_t)q * K, NULL, &s, NULL);
        it += s.iterations; ex += s.expansions; ev += s.evaluations; es += s.estimates;
    }
    (void)threads;
    if (total) {
        total->iterations = it; total->expansions = ex; total->evaluations = ev; total->estimates = es;
        total->phase2_iter = 0;
    }
    return err ? OG_ERR_ARG : OG_OK;
}

/* include/common.hpp:26-47 (host build: plain multiply then add, scalar
 * distance from include/distance.hpp:14-29). */
uint32_t og_entry_point_centroid(const float* data, uint64_t n, uint64_t dim, uint64_t row, int use_ip) {
    float* c = (float*)calloc(dim, sizeof(float));
    const float inv = 1.0f / (float)n;
    for (uint64_t i = 0; i < n; ++i) {
        const float* r = data + i * row;
        for (uint64_t d = 0; d < dim; ++d) {
            float t = r[d] * inv;
            c[d] = c[d] + t;
        }
    }
    uint32_t best = 0;
    float bd = FLT_MAX;
    for (uint64_t i = 0; i < n; ++i) {
        const float* r = data + i * row;
        float s = 0.0f;
        for (uint64_t d = 0; d < dim; ++d) {
            float t;
            if (use_ip) t = r[d] * c[d];
            else { float df = r[d] - c[d]; t = df * df; }
            s = s + t;
        }
        if (use_ip) s = -s;
        if (s < bd) { bd = s; best = (uint32_t)i; }
    }
    free(c);
    return best;
}

/* include/common.hpp:49-66 */
float og_compute_recall(const uint32_t* pred, const int32_t* gt, uint64_t nq, int topk, int gt_k) {
    uint64_t correct = 0;
    int ek = topk < gt_k ? topk : gt_k;
    for (uint64_t i = 0; i < nq; ++i)
        for (int j = 0; j < topk; ++j) {
            int p = (int)pred[i * topk + j];
            for (int k = 0; k < ek; ++k)
                if (p == gt[i * gt_k + k]) { correct++; break; }
        }
    return (float)correct / (float)(nq * (uint64_t)topk);
}
