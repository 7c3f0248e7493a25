// fg_shard_merge.cu -- the per-query merge of a sharded index's top-K lists.
//
// With the base split into S shards, each with its own graph, every query is
// searched on every shard and each shard returns its own ascending top-k
// (local ids, distances).  After the lists are all-gathered (NCCL over
// NVLink), this kernel forms the global top-K of every query: the lists'
// stable merge ordered by (distance, shard, position in the shard's list).
// There is nothing like it in the reference, whose index is one graph on one
// device (gpu_search_adaptive.cu:65-72).
//
// One warp per query.  The S lists' distances are staged in the warp's
// shared memory (coalesced loads); each of the first min(k, K) entries of
// every list computes its own output position as its position in its list
// plus, for every other list, the number of entries that precede it there:
// those with a smaller distance, and those with an equal one in a list of a
// lower shard (binary searches in shared memory).  Entries at position >= K
// are dropped, so every output slot is written exactly once and no sorting
// network or inter-warp step is needed.  Traffic is S*k*8 bytes read and K*8
// written per query, tiny beside the searches it follows.
#include <cstdint>

#include <cuda_runtime.h>

#include "fg_internal.h"

namespace fg {
namespace {

constexpr int kMaxShards = 64;

struct ShardOffsets {
    uint32_t v[kMaxShards];
};

// first index in a[0..n) with a[i] >= x (strict = false) or a[i] > x (strict = true)
__device__ __forceinline__ int bound(const float* a, int n, float x, bool strict) {
    int lo = 0, hi = n;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        const float y = a[mid];
        if (strict ? (y <= x) : (y < x)) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

__global__ void shard_merge_kernel(const uint32_t* __restrict__ ids, const float* __restrict__ dists,
                                   const ShardOffsets off, int S, int nq, int k, int K, uint32_t* __restrict__ out_ids,
                                   float* __restrict__ out_dists) {
    extern __shared__ float sdist[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int q = blockIdx.x * (blockDim.x >> 5) + warp;
    if (q >= nq) return;  // warps are independent: no block barrier below
    float* d = sdist + static_cast<size_t>(warp) * S * k;
    for (int s = 0; s < S; ++s) {
        const float* src = dists + (static_cast<size_t>(s) * nq + q) * k;
        for (int p = lane; p < k; p += 32) d[s * k + p] = src[p];
    }
    __syncwarp();
    const int lim = k < K ? k : K;
    for (int i = lane; i < S * lim; i += 32) {
        const int s = i / lim, p = i - s * lim;
        const float v = d[s * k + p];
        int rank = p;
        for (int t = 0; t < S && rank < K; ++t)
            if (t != s) rank += bound(d + t * k, k, v, t < s);
        if (rank < K) {
            const size_t o = static_cast<size_t>(q) * K + rank;
            out_ids[o] = ids[(static_cast<size_t>(s) * nq + q) * k + p] + off.v[s];
            if (out_dists) out_dists[o] = v;
        }
    }
}

}  // namespace

int shard_merge_max_shards() { return kMaxShards; }

cudaError_t launch_shard_merge(const uint32_t* ids, const float* dists, const uint32_t* offsets, int shards, int nq,
                               int k, int K, uint32_t* out_ids, float* out_dists, cudaStream_t stream) {
    ShardOffsets off{};
    for (int s = 0; s < shards; ++s) off.v[s] = offsets ? offsets[s] : 0u;
    const size_t per_warp = static_cast<size_t>(shards) * k * sizeof(float);
    // up to 4 queries per CTA while their lists fit 48 KB of shared memory
    int wpc = 4;
    while (wpc > 1 && per_warp * wpc > 48 * 1024) wpc >>= 1;
    const size_t smem = per_warp * wpc;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(shard_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    const int grid = (nq + wpc - 1) / wpc;
    shard_merge_kernel<<<grid, 32 * wpc, smem, stream>>>(ids, dists, off, shards, nq, k, K, out_ids, out_dists);
    return cudaGetLastError();
}

}  // namespace fg
