// ref_harness.cu -- a harness of our own around the reference's sm_100a build.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles it together with the
// reference's unmodified gpu_search_adaptive.cu (read from the reference
// tree, never copied) into oracle/_ref/libfgref.so.  It exposes:
//   * the reference's public class API QuantizationGraph / gpu_search_adaptive
//     (include/qg.hpp:17,62-63, gpu_search_adaptive.cu:12-114) behind C entry
//     points, for golden result ids and for bench.py's reference leg;
//   * small kernels that call the reference's own device functions on
//     caller-supplied inputs, so the CPU oracle's arithmetic (contraction,
//     rounding, tie order) can be pinned against the reference build:
//       query_prepare_lut_gpu   (include/utils.cuh:840-939)
//       scan_one_neighbor_lanes_gpu<8> / scan_one_neighbor_lane_seq_lut_gpu
//                               (include/utils.cuh:941-1027)
//       warp_distance           (include/utils.cuh:270-305)
//       dispatch_topk_candidate_sort_and_merge (include/utils.cuh:1369-1399)
//       update_adaptive_state / keep_count_for_expander
//                               (src/adaptive_search_utils.cuh:121-205)
// Nothing here runs in the product.
#include <cstdint>
#include <cstring>
#include <string>

#include "include/qg.hpp"
#include "src/adaptive_search.cuh"

namespace {
int check(cudaError_t e) { return e == cudaSuccess ? 0 : static_cast<int>(e); }
}

extern "C" {

// ---------------------------------------------------------------- class API
void* ref_qg_create(const char* path, size_t n, size_t dim, int degree, int use_ip) {
    auto* qg = new QuantizationGraph(n, dim, degree, std::string(path));
    qg->set_metric(use_ip ? METRIC_IP : METRIC_L2);
    return qg;
}

int ref_qg_search(void* h, int nq, const float* queries, int K, uint32_t* out, int beam, double* elapsed) {
    double e = 0.0;
    static_cast<QuantizationGraph*>(h)->gpu_search_adaptive(nq, queries, K, out, beam, e);
    *elapsed = e;
    return 0;
}

void ref_qg_free(void* h) { delete static_cast<QuantizationGraph*>(h); }

int ref_internal_topk() { return INTERNAL_TOPK; }
}

// ------------------------------------------------------------ query prepare
__global__ void harness_query_prep(const float* queries, int dim, int D, const float* signs, float* rot_out,
                                   uint8_t* lut_out, float* fac_out, int32_t* sumq_out) {
    extern __shared__ unsigned char smem[];
    float* qbuf = reinterpret_cast<float*>(smem);
    float* rot = qbuf + dim;
    uint8_t* lut = reinterpret_cast<uint8_t*>(rot + D);
    __shared__ QueryFactors qf;
    const float* q = queries + static_cast<size_t>(blockIdx.x) * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) qbuf[i] = q[i];
    if (threadIdx.x == 0) {
        qf.rotated_query = rot;
        qf.quantized_query = nullptr;
        qf.lut = lut;
        qf.low_val = FLT_MAX;
        qf.high_val = -FLT_MAX;
        qf.width = 0.0f;
        qf.sum_q = 0;
    }
    __syncthreads();
    query_prepare_lut_gpu(qbuf, qf, signs, dim, D);
    __syncthreads();
    for (int i = threadIdx.x; i < D; i += blockDim.x) rot_out[static_cast<size_t>(blockIdx.x) * D + i] = rot[i];
    for (int i = threadIdx.x; i < 4 * D; i += blockDim.x) lut_out[static_cast<size_t>(blockIdx.x) * 4 * D + i] = lut[i];
    if (threadIdx.x == 0) {
        fac_out[blockIdx.x * 3 + 0] = qf.low_val;
        fac_out[blockIdx.x * 3 + 1] = qf.high_val;
        fac_out[blockIdx.x * 3 + 2] = qf.width;
        sumq_out[blockIdx.x] = qf.sum_q;
    }
}

// ------------------------------------------------------ RaBitQ estimates
// One block per (query, parent row).  lanes8_out gets the theta=1 8-lane
// estimate of every neighbour, seq_out the speculative 1-lane estimate.
__global__ void harness_scan(const float* rows, size_t row_floats, size_t code_off, size_t factor_off, int degree,
                             int D, const uint32_t* parent_ids, const float* parent_dists, const uint8_t* luts,
                             const float* qfacs, const int32_t* sumqs, float* lanes8_out, float* seq_out) {
    extern __shared__ unsigned char smem[];
    uint8_t* lut = smem;
    __shared__ QueryFactors qf;
    const int b = blockIdx.x;
    for (int i = threadIdx.x; i < 4 * D; i += blockDim.x) lut[i] = luts[static_cast<size_t>(b) * 4 * D + i];
    if (threadIdx.x == 0) {
        qf.rotated_query = nullptr;
        qf.quantized_query = nullptr;
        qf.lut = lut;
        qf.low_val = qfacs[b * 3 + 0];
        qf.high_val = qfacs[b * 3 + 1];
        qf.width = qfacs[b * 3 + 2];
        qf.sum_q = sumqs[b];
    }
    __syncthreads();
    const float* prow = rows + static_cast<size_t>(parent_ids[b]) * row_floats;
    const float* fac = prow + factor_off;
    const uint8_t* codes = reinterpret_cast<const uint8_t*>(prow + code_off);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int group = lane >> 3, glane = lane & 7;
    for (int base = warp * 4; base < degree; base += (blockDim.x >> 5) * 4) {
        const int i = base + group;
        float est = 0.0f;
        if (i < degree) {
            est = scan_one_neighbor_lanes_gpu<8>(qf, codes, i, fac + i, fac + degree + i, fac + 2 * degree + i,
                                                 parent_dists[b], D, D >> 3);
            if (glane == 0) lanes8_out[static_cast<size_t>(b) * degree + i] = est;
        }
    }
    for (int i = threadIdx.x; i < degree; i += blockDim.x) {
        seq_out[static_cast<size_t>(b) * degree + i] = scan_one_neighbor_lane_seq_lut_gpu(
            qf, codes, i, fac[i], fac[degree + i], fac[2 * degree + i], parent_dists[b], D, D >> 3);
    }
}

// ---------------------------------------------------------- exact distance
// One warp per (query, node) pair.
__global__ void harness_l2(const float* queries, int dim, const float* rows, size_t row_floats, const uint32_t* qidx,
                           const uint32_t* nodes, int npairs, int use_ip, float* out) {
    extern __shared__ float qs[];
    const int warp = threadIdx.x >> 5;
    const int pair = blockIdx.x * (blockDim.x >> 5) + warp;
    if (pair >= npairs) return;
    float* q = qs + warp * dim;
    const float* src = queries + static_cast<size_t>(qidx[pair]) * dim;
    for (int i = threadIdx.x & 31; i < dim; i += 32) q[i] = src[i];
    __syncwarp();
    float d = warp_distance(dim, q, rows + static_cast<size_t>(nodes[pair]) * row_floats, use_ip != 0);
    if ((threadIdx.x & 31) == 0) out[pair] = d;
}

// ------------------------------------------------------------- beam merge
// One block per case: beam (itopk entries) + candidates (cbs) -> merged beam.
__global__ void harness_merge(uint32_t* idx, float* dist, int itopk, int cbs, int first) {
    extern __shared__ unsigned char smem[];
    const int total = itopk + cbs;
    uint32_t* sidx = reinterpret_cast<uint32_t*>(smem);
    float* sdist = reinterpret_cast<float*>(sidx + total);
    uint32_t* midx = reinterpret_cast<uint32_t*>(sdist + total);
    float* mdist = reinterpret_cast<float*>(midx + itopk);
    const size_t off = static_cast<size_t>(blockIdx.x) * total;
    for (int i = threadIdx.x; i < total; i += blockDim.x) { sidx[i] = idx[off + i]; sdist[i] = dist[off + i]; }
    __syncthreads();
    dispatch_topk_candidate_sort_and_merge(sidx, sdist, midx, mdist, cbs, itopk, first != 0);
    __syncthreads();
    for (int i = threadIdx.x; i < total; i += blockDim.x) { idx[off + i] = sidx[i]; dist[off + i] = sdist[i]; }
}

// ------------------------------------------------------------- controller
// For each case: run update_adaptive_state and keep_count_for_expander.
__global__ void harness_ctrl(int n, const float* rho_prev, const int* policy_iters, const float* rate,
                             const float* phase2_rho, const uint32_t* active, const int* cut_valid,
                             const uint32_t* near, float* rho_out, int* keep_out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    GPUAdaptiveSearchState s;
    s.adaptive_spec_degree = 1;
    s.adaptive_rho = rho_prev[i];
    s.policy_iters = policy_iters[i];
    s.top1_node = 0;
    s.top1_stall_iters = 0;
    s.warmup_done = false;
    s.entry_distance = 1.0f;
    s.last_expander_distance = FLT_MAX;
    s.current_expander_distance = FLT_MAX;
    GPUAdaptiveSearchState t = update_adaptive_state(0u, 0, FLT_MAX, FLT_MAX, rate[i], s, phase2_rho[i]);
    rho_out[i] = t.adaptive_rho;
    keep_out[i] = keep_count_for_expander(active[i], t, cut_valid[i] != 0, near[i]);
}

extern "C" {

int ref_query_prep(const float* d_queries, int nq, int dim, int D, const float* d_signs, float* d_rot,
                   uint8_t* d_lut, float* d_fac, int32_t* d_sumq) {
    size_t sm = static_cast<size_t>(dim + D) * sizeof(float) + 4 * D;
    harness_query_prep<<<nq, BLOCK_SIZE, sm>>>(d_queries, dim, D, d_signs, d_rot, d_lut, d_fac, d_sumq);
    int rc = check(cudaGetLastError());
    return rc ? rc : check(cudaDeviceSynchronize());
}

int ref_scan(const float* d_rows, size_t row_floats, size_t code_off, size_t factor_off, int degree, int D, int nb,
             const uint32_t* d_parents, const float* d_pdists, const uint8_t* d_luts, const float* d_qfacs,
             const int32_t* d_sumqs, float* d_lanes8, float* d_seq) {
    harness_scan<<<nb, BLOCK_SIZE, 4 * D>>>(d_rows, row_floats, code_off, factor_off, degree, D, d_parents, d_pdists,
                                            d_luts, d_qfacs, d_sumqs, d_lanes8, d_seq);
    int rc = check(cudaGetLastError());
    return rc ? rc : check(cudaDeviceSynchronize());
}

int ref_l2(const float* d_queries, int dim, const float* d_rows, size_t row_floats, const uint32_t* d_qidx,
           const uint32_t* d_nodes, int npairs, int use_ip, float* d_out) {
    const int wpb = 8;
    harness_l2<<<(npairs + wpb - 1) / wpb, wpb * 32, wpb * dim * sizeof(float)>>>(
        d_queries, dim, d_rows, row_floats, d_qidx, d_nodes, npairs, use_ip, d_out);
    int rc = check(cudaGetLastError());
    return rc ? rc : check(cudaDeviceSynchronize());
}

int ref_merge(uint32_t* d_idx, float* d_dist, int ncase, int itopk, int cbs, int first) {
    size_t sm = static_cast<size_t>(itopk + cbs) * 8 + static_cast<size_t>(itopk) * 8;
    if (sm > 48 * 1024) {
        int rc = check(cudaFuncSetAttribute(harness_merge, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(sm)));
        if (rc) return rc;
    }
    harness_merge<<<ncase, BLOCK_SIZE, sm>>>(d_idx, d_dist, itopk, cbs, first);
    int rc = check(cudaGetLastError());
    return rc ? rc : check(cudaDeviceSynchronize());
}

int ref_ctrl(int n, const float* d_rho_prev, const int* d_policy, const float* d_rate, const float* d_p2rho,
             const uint32_t* d_active, const int* d_cut, const uint32_t* d_near, float* d_rho_out, int* d_keep_out) {
    harness_ctrl<<<(n + 127) / 128, 128>>>(n, d_rho_prev, d_policy, d_rate, d_p2rho, d_active, d_cut, d_near,
                                            d_rho_out, d_keep_out);
    int rc = check(cudaGetLastError());
    return rc ? rc : check(cudaDeviceSynchronize());
}
}
