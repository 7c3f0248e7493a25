// fg_api.cu -- the C ABI (include/flashgann.h): index residency, search
// launches, and the host helpers of the reference CLI.
#include <algorithm>
#include <cfloat>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include <cuda_runtime.h>

#include "fg_config.h"
#include "fg_internal.h"

struct fg_index {
    int device = 0;
    uint64_t n = 0, dim = 0, D = 0, code_off = 0, factor_off = 0, nbr_off = 0, row = 0;
    int degree = 0;
    uint32_t entry = 0;
    int metric = FG_METRIC_L2;
    int goal = FG_GOAL_LATENCY;
    float* d_rows = nullptr;
    float* d_signs = nullptr;
    // buffers of the host-buffer search path, grown on demand
    float* d_queries = nullptr;
    size_t cap_queries = 0;
    uint32_t* d_results = nullptr;
    size_t cap_results = 0;
    float* d_dists = nullptr;  // fg_search_multi with distances
    size_t cap_dists = 0;
    uint32_t* d_counter = nullptr;  // persistent-CTA work counter
    cudaStream_t stream = nullptr;
    // fg_search_async: per-slot device buffers and work counter, grown on demand
    struct AsyncSlot {
        float* d_queries = nullptr;
        size_t cap_queries = 0;
        uint32_t* d_results = nullptr;
        size_t cap_results = 0;
        uint32_t* d_counter = nullptr;
    } slots[FG_ASYNC_SLOTS];
    // work counters of fg_search_device, one per stream, so that searches on
    // different streams may overlap on the device
    std::vector<std::pair<cudaStream_t, uint32_t*>> stream_counters;
};

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(FG_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Makes `dev` current for the scope and restores the caller's device.
struct DeviceGuard {
    int prev = -1;
    cudaError_t err = cudaSuccess;
    explicit DeviceGuard(int dev) {
        err = cudaGetDevice(&prev);
        if (err == cudaSuccess && prev != dev) err = cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

uint64_t padded_dim_of(uint64_t dim) {
    uint64_t D = 1;
    while (D < dim) D <<= 1;
    return D;
}

void fill_layout(fg_index* x, uint64_t n, uint64_t dim, int degree) {
    x->n = n;
    x->dim = dim;
    x->D = padded_dim_of(dim);
    x->degree = degree;
    x->code_off = dim;
    x->factor_off = dim + (x->D / 64) * 2 * static_cast<uint64_t>(degree);
    x->nbr_off = x->factor_off + 3 * static_cast<uint64_t>(degree);
    x->row = x->nbr_off + static_cast<uint64_t>(degree);
}

int check_shape(uint64_t n, uint64_t dim, int degree, int metric) {
    if (n < 1 || n > 0x7FFFFFFFull) return fail(FG_ERR_ARG, "num_nodes %llu outside [1, 2^31-1]", (unsigned long long)n);
    if (dim < 32 || dim > FG_MAX_DIM)
        return fail(FG_ERR_UNSUPPORTED, "dim %llu outside the supported range [32, %d]", (unsigned long long)dim, FG_MAX_DIM);
    if (degree < 1 || degree > FG_MAX_DEGREE)
        return fail(FG_ERR_UNSUPPORTED, "degree %d outside the supported range [1, %d]", degree, FG_MAX_DEGREE);
    if (metric != FG_METRIC_L2 && metric != FG_METRIC_IP) return fail(FG_ERR_ARG, "unknown metric %d", metric);
    return FG_OK;
}

// include/common.hpp:26-47: node nearest the centroid of the raw vectors,
// centroid accumulated as c[d] += row[d] * (1/n) in node order.
uint32_t centroid_entry(const float* rows, uint64_t n, uint64_t dim, uint64_t row, int metric) {
    std::vector<float> c(dim, 0.0f);
    const float inv = 1.0f / static_cast<float>(n);
    for (uint64_t i = 0; i < n; ++i) {
        const float* r = rows + i * row;
        for (uint64_t d = 0; d < dim; ++d) {
            volatile float t = r[d] * inv;
            c[d] = c[d] + t;
        }
    }
    uint32_t best = 0;
    float bd = FLT_MAX;
    for (uint64_t i = 0; i < n; ++i) {
        const float* r = rows + i * row;
        float s = 0.0f;
        for (uint64_t d = 0; d < dim; ++d) {
            volatile float t;
            if (metric == FG_METRIC_IP) t = r[d] * c[d];
            else {
                const float df = r[d] - c[d];
                t = df * df;
            }
            s = s + t;
        }
        if (metric == FG_METRIC_IP) s = -s;
        if (s < bd) {
            bd = s;
            best = static_cast<uint32_t>(i);
        }
    }
    return best;
}

int alloc_device(fg_index* x, uint64_t n) {
    size_t free_b = 0, total_b = 0;
    cudaError_t e = cudaMemGetInfo(&free_b, &total_b);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemGetInfo");
    const size_t need = static_cast<size_t>(n) * x->row * sizeof(float) + x->D * sizeof(float);
    if (need > free_b)
        return fail(FG_ERR_OOM, "codebook needs %.2f GiB, %.2f GiB free on device %d", need / 1073741824.0,
                    free_b / 1073741824.0, x->device);
    e = cudaMalloc(&x->d_rows, static_cast<size_t>(n) * x->row * sizeof(float));
    if (e != cudaSuccess) return fail(FG_ERR_OOM, "cudaMalloc(codebook): %s", cudaGetErrorString(e));
    e = cudaMalloc(&x->d_signs, x->D * sizeof(float));
    if (e != cudaSuccess) return fail(FG_ERR_OOM, "cudaMalloc(signs): %s", cudaGetErrorString(e));
    e = cudaMalloc(&x->d_counter, 256);
    if (e != cudaSuccess) return fail(FG_ERR_OOM, "cudaMalloc(counter): %s", cudaGetErrorString(e));
    e = cudaStreamCreateWithFlags(&x->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamCreate");
    return FG_OK;
}

void destroy(fg_index* x) {
    if (!x) return;
    DeviceGuard g(x->device);
    if (x->d_rows) cudaFree(x->d_rows);
    if (x->d_signs) cudaFree(x->d_signs);
    if (x->d_queries) cudaFree(x->d_queries);
    if (x->d_results) cudaFree(x->d_results);
    if (x->d_dists) cudaFree(x->d_dists);
    if (x->d_counter) cudaFree(x->d_counter);
    for (auto& sl : x->slots) {
        if (sl.d_queries) cudaFree(sl.d_queries);
        if (sl.d_results) cudaFree(sl.d_results);
        if (sl.d_counter) cudaFree(sl.d_counter);
    }
    for (auto& sc : x->stream_counters) cudaFree(sc.second);
    if (x->stream) cudaStreamDestroy(x->stream);
    delete x;
}

// Checks the device ordinal; FG_DEVICE_CURRENT becomes the calling thread's
// current device (the device the reference's search uses).
int check_device(int* device) {
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count < 1) return fail(FG_ERR_NO_DEVICE, "no CUDA device available (%s)", cudaGetErrorString(e));
    if (*device == FG_DEVICE_CURRENT && (e = cudaGetDevice(device)) != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (*device < 0 || *device >= count) return fail(FG_ERR_ARG, "device %d outside [0, %d)", *device, count);
    return FG_OK;
}

// Grows a device buffer of the host-buffer search paths to hold n elements.
template <typename T>
int grow(T** buf, size_t* cap, size_t n, const char* what) {
    if (n <= *cap) return FG_OK;
    if (*buf) cudaFree(*buf);
    *buf = nullptr;
    *cap = 0;
    cudaError_t e = cudaMalloc(buf, n * sizeof(T));
    if (e != cudaSuccess) return fail(FG_ERR_OOM, "cudaMalloc(%s): %s", what, cudaGetErrorString(e));
    *cap = n;
    return FG_OK;
}

// The work counter fg_search_device uses on `stream` (allocated on the
// stream's first search): launches on one stream run in order and share it,
// launches on different streams get their own.
constexpr size_t kMaxStreamCounters = 64;
int stream_counter(fg_index* x, cudaStream_t stream, uint32_t** out) {
    for (auto& sc : x->stream_counters)
        if (sc.first == stream) {
            *out = sc.second;
            return FG_OK;
        }
    if (x->stream_counters.size() >= kMaxStreamCounters)
        return fail(FG_ERR_UNSUPPORTED, "more than %zu streams searched one index", kMaxStreamCounters);
    uint32_t* c = nullptr;
    const cudaError_t e = cudaMalloc(&c, 256);
    if (e != cudaSuccess) return fail(FG_ERR_OOM, "cudaMalloc(counter): %s", cudaGetErrorString(e));
    x->stream_counters.emplace_back(stream, c);
    *out = c;
    return FG_OK;
}

fg::SearchArgs base_args(const fg_index* x) {
    fg::SearchArgs a;
    a.rows = x->d_rows;
    a.signs = x->d_signs;
    a.n = x->n;
    a.row = x->row;
    a.code_off = x->code_off;
    a.factor_off = x->factor_off;
    a.nbr_off = x->nbr_off;
    a.dim = static_cast<int>(x->dim);
    a.padded_dim = static_cast<int>(x->D);
    a.degree = x->degree;
    a.entry = x->entry;
    a.use_ip = x->metric == FG_METRIC_IP;
    a.goal = x->goal;
    a.work_counter = x->d_counter;
    return a;
}

}  // namespace

extern "C" {

const char* fg_status_string(int s) {
    switch (s) {
        case FG_OK: return "ok";
        case FG_ERR_IO: return "i/o error";
        case FG_ERR_FORMAT: return "bad file format";
        case FG_ERR_ARG: return "invalid argument";
        case FG_ERR_CUDA: return "CUDA error";
        case FG_ERR_OOM: return "out of device memory";
        case FG_ERR_UNSUPPORTED: return "unsupported configuration";
        case FG_ERR_NO_DEVICE: return "no CUDA device";
        default: return "unknown status";
    }
}

const char* fg_last_error(void) { return g_err.c_str(); }

int fg_index_load(const char* path, uint64_t n, uint64_t dim, int32_t degree, int32_t metric, int32_t device,
                  fg_index** out) {
    g_err.clear();
    if (!out || !path) return fail(FG_ERR_ARG, "null argument");
    *out = nullptr;
    int rc = check_shape(n, dim, degree, metric);
    if (rc) return rc;
    FILE* f = fopen(path, "rb");
    if (!f) return fail(FG_ERR_IO, "cannot open codebook file: %s", path);
    auto* x = new fg_index();
    x->device = device;
    x->metric = metric;
    fill_layout(x, n, dim, degree);
    const uint64_t row_bytes = x->row * sizeof(float);
    const uint64_t need = 4 + n * row_bytes + x->D * sizeof(float);
    fseeko(f, 0, SEEK_END);
    const uint64_t size = static_cast<uint64_t>(ftello(f));
    fseeko(f, 0, SEEK_SET);
    if (size < need) {
        fclose(f);
        destroy(x);
        return fail(FG_ERR_FORMAT, "codebook %s has %llu bytes, layout (n=%llu dim=%llu degree=%d) needs %llu", path,
                    (unsigned long long)size, (unsigned long long)n, (unsigned long long)dim, degree,
                    (unsigned long long)need);
    }
    if ((rc = check_device(&device))) {
        fclose(f);
        destroy(x);
        return rc;
    }
    x->device = device;
    DeviceGuard g(device);
    if (g.err != cudaSuccess) {
        fclose(f);
        destroy(x);
        return cuda_fail(g.err, "cudaSetDevice");
    }
    if ((rc = alloc_device(x, n))) {
        fclose(f);
        destroy(x);
        return rc;
    }
    uint32_t entry = 0;
    if (fread(&entry, 4, 1, f) != 1) {
        fclose(f);
        destroy(x);
        return fail(FG_ERR_IO, "short read of %s", path);
    }
    // stream the rows through a pinned staging buffer
    const uint64_t chunk_rows = std::max<uint64_t>(1, (64ull << 20) / row_bytes);
    float* stage = nullptr;
    cudaError_t e = cudaMallocHost(&stage, chunk_rows * row_bytes);
    if (e != cudaSuccess) {
        fclose(f);
        destroy(x);
        return cuda_fail(e, "cudaMallocHost");
    }
    for (uint64_t r0 = 0; r0 < n && !rc; r0 += chunk_rows) {
        const uint64_t m = std::min(chunk_rows, n - r0);
        if (fread(stage, row_bytes, m, f) != m) rc = fail(FG_ERR_IO, "short read of %s", path);
        else if ((e = cudaMemcpy(x->d_rows + r0 * x->row, stage, m * row_bytes, cudaMemcpyHostToDevice)) != cudaSuccess)
            rc = cuda_fail(e, "cudaMemcpy(codebook)");
    }
    std::vector<float> signs(x->D);
    if (!rc && fread(signs.data(), sizeof(float), x->D, f) != x->D) rc = fail(FG_ERR_IO, "short read of signs in %s", path);
    if (!rc && (e = cudaMemcpy(x->d_signs, signs.data(), x->D * sizeof(float), cudaMemcpyHostToDevice)) != cudaSuccess)
        rc = cuda_fail(e, "cudaMemcpy(signs)");
    if (!rc && entry == 0xFFFFFFFFu) {
        // centroid fallback over the raw vectors (re-read, as the reference keeps them in host memory)
        std::vector<float> raw(n * x->row);
        fseeko(f, 4, SEEK_SET);
        if (fread(raw.data(), row_bytes, n, f) != n) rc = fail(FG_ERR_IO, "short read of %s", path);
        else entry = centroid_entry(raw.data(), n, dim, x->row, metric);
    }
    cudaFreeHost(stage);
    fclose(f);
    if (!rc && entry >= n) rc = fail(FG_ERR_FORMAT, "entry point %u outside [0, %llu)", entry, (unsigned long long)n);
    if (rc) {
        destroy(x);
        return rc;
    }
    x->entry = entry;
    *out = x;
    return FG_OK;
}

int fg_index_create(const float* rows, const float* signs, uint32_t entry, uint64_t n, uint64_t dim, int32_t degree,
                    int32_t metric, int32_t device, fg_index** out) {
    g_err.clear();
    if (!out || !rows || !signs) return fail(FG_ERR_ARG, "null argument");
    *out = nullptr;
    int rc = check_shape(n, dim, degree, metric);
    if (rc) return rc;
    if ((rc = check_device(&device))) return rc;
    auto* x = new fg_index();
    x->device = device;
    x->metric = metric;
    fill_layout(x, n, dim, degree);
    DeviceGuard g(device);
    if (g.err != cudaSuccess) {
        destroy(x);
        return cuda_fail(g.err, "cudaSetDevice");
    }
    if ((rc = alloc_device(x, n))) {
        destroy(x);
        return rc;
    }
    cudaError_t e = cudaMemcpy(x->d_rows, rows, n * x->row * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(x->d_signs, signs, x->D * sizeof(float), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        destroy(x);
        return cuda_fail(e, "cudaMemcpy(codebook)");
    }
    if (entry == 0xFFFFFFFFu) entry = centroid_entry(rows, n, dim, x->row, metric);
    if (entry >= n) {
        destroy(x);
        return fail(FG_ERR_FORMAT, "entry point %u outside [0, %llu)", entry, (unsigned long long)n);
    }
    x->entry = entry;
    *out = x;
    return FG_OK;
}

int fg_index_create_device(const float* d_rows, const float* d_signs, uint32_t entry, uint64_t n, uint64_t dim,
                           int32_t degree, int32_t metric, int32_t device, fg_index** out) {
    g_err.clear();
    if (!out || !d_rows || !d_signs) return fail(FG_ERR_ARG, "null argument");
    *out = nullptr;
    int rc = check_shape(n, dim, degree, metric);
    if (rc) return rc;
    if (entry >= n) return fail(FG_ERR_ARG, "entry point %u outside [0, %llu)", entry, (unsigned long long)n);
    if ((rc = check_device(&device))) return rc;
    auto* x = new fg_index();
    x->device = device;
    x->metric = metric;
    fill_layout(x, n, dim, degree);
    DeviceGuard g(device);
    if (g.err != cudaSuccess) {
        destroy(x);
        return cuda_fail(g.err, "cudaSetDevice");
    }
    if ((rc = alloc_device(x, n))) {
        destroy(x);
        return rc;
    }
    cudaError_t e = cudaMemcpy(x->d_rows, d_rows, n * x->row * sizeof(float), cudaMemcpyDeviceToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(x->d_signs, d_signs, x->D * sizeof(float), cudaMemcpyDeviceToDevice);
    if (e != cudaSuccess) {
        destroy(x);
        return cuda_fail(e, "cudaMemcpy(codebook, device to device)");
    }
    x->entry = entry;
    *out = x;
    return FG_OK;
}

int fg_index_free(fg_index* x) {
    destroy(x);
    return FG_OK;
}

int fg_index_layout(const fg_index* x, fg_layout* o) {
    if (!x || !o) return fail(FG_ERR_ARG, "null argument");
    o->num_nodes = x->n;
    o->dim = x->dim;
    o->padded_dim = x->D;
    o->code_offset = x->code_off;
    o->factor_offset = x->factor_off;
    o->neighbor_offset = x->nbr_off;
    o->row_offset = x->row;
    o->degree = x->degree;
    o->entry_point = x->entry;
    o->metric = x->metric;
    o->device = x->device;
    return FG_OK;
}

int fg_index_set_metric(fg_index* x, int32_t metric) {
    if (!x) return fail(FG_ERR_ARG, "null index");
    if (metric != FG_METRIC_L2 && metric != FG_METRIC_IP) return fail(FG_ERR_ARG, "unknown metric %d", metric);
    x->metric = metric;
    return FG_OK;
}

int fg_index_set_plan_goal(fg_index* x, int32_t goal) {
    if (!x) return fail(FG_ERR_ARG, "null index");
    if (goal != FG_GOAL_LATENCY && goal != FG_GOAL_THROUGHPUT) return fail(FG_ERR_ARG, "unknown plan goal %d", goal);
    x->goal = goal;
    return FG_OK;
}

int fg_search_plan(fg_index* x, int32_t nq, int32_t K, int32_t beam, int32_t* kernel, int32_t* resident_queries) {
    g_err.clear();
    if (!x) return fail(FG_ERR_ARG, "null index");
    if (nq < 0) return fail(FG_ERR_ARG, "nq must be >= 0 (got %d)", nq);
    DeviceGuard g(x->device);
    if (g.err != cudaSuccess) return cuda_fail(g.err, "cudaSetDevice");
    fg::SearchArgs a = base_args(x);
    a.nq = nq;
    a.K = K;
    a.beam = beam;
    fg::SearchPlan plan;
    char err[256];
    const int rc = fg::plan_search(a, &plan, x->device, err, sizeof(err));
    if (rc) return fail(rc, "%s", err);
    int k = FG_PLAN_CTA, resident = 0;
    if (plan.kernel == 1) {
        k = plan.warp_mode == 1 ? FG_PLAN_STAGED : plan.warp_mode == 2 ? FG_PLAN_PAIR : FG_PLAN_WARP;
        resident = plan.resident_queries;
    } else {
        int sms = 0;
        cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, x->device);
        if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
        resident = plan.blocks_per_sm * sms;  // one query per CTA
    }
    if (kernel) *kernel = k;
    if (resident_queries) *resident_queries = resident;
    return FG_OK;
}

int fg_search_device_ex(fg_index* x, int32_t nq, const float* d_queries, int32_t K, uint32_t* d_out, float* d_dist,
                        int32_t beam, void* stream, fg_query_stats* d_stats, uint32_t* d_trace,
                        int32_t* d_trace_count, int32_t trace_cap) {
    g_err.clear();
    if (!x) return fail(FG_ERR_ARG, "null index");
    if (nq < 0) return fail(FG_ERR_ARG, "nq must be >= 0 (got %d)", nq);
    if (nq > 0 && (!d_queries || !d_out)) return fail(FG_ERR_ARG, "null query or result buffer");
    if ((d_trace == nullptr) != (d_trace_count == nullptr) || (d_trace && trace_cap < 1))
        return fail(FG_ERR_ARG, "trace buffers need both pointers and trace_cap >= 1");
    DeviceGuard g(x->device);
    if (g.err != cudaSuccess) return cuda_fail(g.err, "cudaSetDevice");
    fg::SearchArgs a = base_args(x);
    a.queries = d_queries;
    a.out_ids = d_out;
    a.out_dists = d_dist;
    a.stats = d_stats;
    a.trace = d_trace;
    a.trace_count = d_trace_count;
    a.trace_cap = trace_cap;
    a.nq = nq;
    a.K = K;
    a.beam = beam;
    fg::SearchPlan plan;
    char err[256];
    int rc = fg::plan_search(a, &plan, x->device, err, sizeof(err));
    if (rc) return fail(rc, "%s", err);
    if (nq == 0) return FG_OK;
    if ((rc = stream_counter(x, static_cast<cudaStream_t>(stream), &a.work_counter)) != FG_OK) return rc;
    cudaError_t e = fg::launch_search(a, plan, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "search launch");
    return FG_OK;
}

int fg_search_device(fg_index* x, int32_t nq, const float* d_queries, int32_t K, uint32_t* d_out, float* d_dist,
                     int32_t beam, void* stream) {
    return fg_search_device_ex(x, nq, d_queries, K, d_out, d_dist, beam, stream, nullptr, nullptr, nullptr, 0);
}

int fg_search(fg_index* x, int32_t nq, const float* queries, int32_t K, uint32_t* result_idx, int32_t beam,
              double* elapsed_s) {
    g_err.clear();
    if (!x) return fail(FG_ERR_ARG, "null index");
    if (nq < 0) return fail(FG_ERR_ARG, "nq must be >= 0 (got %d)", nq);
    if (nq > 0 && (!queries || !result_idx)) return fail(FG_ERR_ARG, "null query or result buffer");
    if (elapsed_s) *elapsed_s = 0.0;
    DeviceGuard g(x->device);
    if (g.err != cudaSuccess) return cuda_fail(g.err, "cudaSetDevice");
    fg::SearchArgs a = base_args(x);
    a.nq = nq;
    a.K = K;
    a.beam = beam;
    fg::SearchPlan plan;
    char err[256];
    int rc = fg::plan_search(a, &plan, x->device, err, sizeof(err));
    if (rc) return fail(rc, "%s", err);
    if (nq == 0) return FG_OK;
    const size_t qn = static_cast<size_t>(nq) * x->dim, rn = static_cast<size_t>(nq) * K;
    cudaError_t e;
    if (qn > x->cap_queries) {
        if (x->d_queries) cudaFree(x->d_queries);
        x->d_queries = nullptr;
        x->cap_queries = 0;
        if ((e = cudaMalloc(&x->d_queries, qn * sizeof(float))) != cudaSuccess) return fail(FG_ERR_OOM, "cudaMalloc(queries): %s", cudaGetErrorString(e));
        x->cap_queries = qn;
    }
    if (rn > x->cap_results) {
        if (x->d_results) cudaFree(x->d_results);
        x->d_results = nullptr;
        x->cap_results = 0;
        if ((e = cudaMalloc(&x->d_results, rn * sizeof(uint32_t))) != cudaSuccess) return fail(FG_ERR_OOM, "cudaMalloc(results): %s", cudaGetErrorString(e));
        x->cap_results = rn;
    }
    a.queries = x->d_queries;
    a.out_ids = x->d_results;
    if ((e = cudaMemcpyAsync(x->d_queries, queries, qn * sizeof(float), cudaMemcpyHostToDevice, x->stream)) != cudaSuccess)
        return cuda_fail(e, "cudaMemcpyAsync(queries)");
    if ((e = cudaStreamSynchronize(x->stream)) != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
    // timed like gpu_search_adaptive.cu:98-107: launch and synchronisation
    const auto t0 = std::chrono::high_resolution_clock::now();
    if ((e = fg::launch_search(a, plan, x->stream)) != cudaSuccess) return cuda_fail(e, "search launch");
    if ((e = cudaStreamSynchronize(x->stream)) != cudaSuccess) return cuda_fail(e, "search");
    const auto t1 = std::chrono::high_resolution_clock::now();
    if (elapsed_s) *elapsed_s = std::chrono::duration<double>(t1 - t0).count();
    if ((e = cudaMemcpyAsync(result_idx, x->d_results, rn * sizeof(uint32_t), cudaMemcpyDeviceToHost, x->stream)) != cudaSuccess)
        return cuda_fail(e, "cudaMemcpyAsync(results)");
    if ((e = cudaStreamSynchronize(x->stream)) != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
    return FG_OK;
}

int fg_search_async(fg_index* x, int32_t slot, int32_t nq, const float* queries, int32_t K, uint32_t* result_idx,
                    int32_t beam, void* stream) {
    g_err.clear();
    if (!x) return fail(FG_ERR_ARG, "null index");
    if (slot < 0 || slot >= FG_ASYNC_SLOTS) return fail(FG_ERR_ARG, "slot %d outside [0, %d)", slot, FG_ASYNC_SLOTS);
    if (nq < 0) return fail(FG_ERR_ARG, "nq must be >= 0 (got %d)", nq);
    if (nq > 0 && (!queries || !result_idx)) return fail(FG_ERR_ARG, "null query or result buffer");
    DeviceGuard g(x->device);
    if (g.err != cudaSuccess) return cuda_fail(g.err, "cudaSetDevice");
    fg::SearchArgs a = base_args(x);
    a.nq = nq;
    a.K = K;
    a.beam = beam;
    fg::SearchPlan plan;
    char err[256];
    int rc = fg::plan_search(a, &plan, x->device, err, sizeof(err));
    if (rc) return fail(rc, "%s", err);
    if (nq == 0) return FG_OK;
    fg_index::AsyncSlot& sl = x->slots[slot];
    const size_t qn = static_cast<size_t>(nq) * x->dim, rn = static_cast<size_t>(nq) * K;
    if ((rc = grow(&sl.d_queries, &sl.cap_queries, qn, "queries")) != FG_OK) return rc;
    if ((rc = grow(&sl.d_results, &sl.cap_results, rn, "results")) != FG_OK) return rc;
    cudaError_t e;
    if (!sl.d_counter && (e = cudaMalloc(&sl.d_counter, 256)) != cudaSuccess)
        return fail(FG_ERR_OOM, "cudaMalloc(counter): %s", cudaGetErrorString(e));
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    a.queries = sl.d_queries;
    a.out_ids = sl.d_results;
    a.work_counter = sl.d_counter;
    if ((e = cudaMemcpyAsync(sl.d_queries, queries, qn * sizeof(float), cudaMemcpyHostToDevice, st)) != cudaSuccess)
        return cuda_fail(e, "cudaMemcpyAsync(queries)");
    if ((e = fg::launch_search(a, plan, st)) != cudaSuccess) return cuda_fail(e, "search launch");
    if ((e = cudaMemcpyAsync(result_idx, sl.d_results, rn * sizeof(uint32_t), cudaMemcpyDeviceToHost, st)) != cudaSuccess)
        return cuda_fail(e, "cudaMemcpyAsync(results)");
    return FG_OK;
}

int fg_search_multi(fg_index* const* indexes, int32_t count, int32_t nq, const float* queries, int32_t K,
                    uint32_t* result_idx, float* result_dist, int32_t beam, double* elapsed_s) {
    g_err.clear();
    if (!indexes || count < 1) return fail(FG_ERR_ARG, "need at least one index");
    if (nq < 0) return fail(FG_ERR_ARG, "nq must be >= 0 (got %d)", nq);
    if (nq > 0 && (!queries || !result_idx)) return fail(FG_ERR_ARG, "null query or result buffer");
    if (elapsed_s) *elapsed_s = 0.0;
    const fg_index* x0 = indexes[0];
    for (int i = 0; i < count; ++i) {
        const fg_index* x = indexes[i];
        if (!x) return fail(FG_ERR_ARG, "null index %d", i);
        if (x->n != x0->n || x->dim != x0->dim || x->degree != x0->degree || x->metric != x0->metric ||
            x->entry != x0->entry)
            return fail(FG_ERR_ARG, "index %d does not hold the same graph as index 0", i);
    }
    std::vector<fg::SearchArgs> args(count);
    std::vector<fg::SearchPlan> plans(count);
    std::vector<int> lo(count), hi(count);
    const int per = nq / count, extra = nq % count;
    for (int i = 0; i < count; ++i) {
        lo[i] = i * per + (i < extra ? i : extra);
        hi[i] = lo[i] + per + (i < extra ? 1 : 0);
    }
    cudaError_t e;
    int rc;
    // copies and launches of every device first, so that the devices run concurrently
    for (int i = 0; i < count; ++i) {
        fg_index* x = indexes[i];
        const int m = hi[i] - lo[i];
        DeviceGuard g(x->device);
        if (g.err != cudaSuccess) return cuda_fail(g.err, "cudaSetDevice");
        fg::SearchArgs& a = args[i];
        a = base_args(x);
        a.nq = m;
        a.K = K;
        a.beam = beam;
        char err[256];
        if ((rc = fg::plan_search(a, &plans[i], x->device, err, sizeof(err))) != FG_OK) return fail(rc, "%s", err);
        if (m == 0) continue;
        const size_t qn = static_cast<size_t>(m) * x->dim, rn = static_cast<size_t>(m) * K;
        if ((rc = grow(&x->d_queries, &x->cap_queries, qn, "queries")) != FG_OK) return rc;
        if ((rc = grow(&x->d_results, &x->cap_results, rn, "results")) != FG_OK) return rc;
        if (result_dist && (rc = grow(&x->d_dists, &x->cap_dists, rn, "distances")) != FG_OK) return rc;
        a.queries = x->d_queries;
        a.out_ids = x->d_results;
        a.out_dists = result_dist ? x->d_dists : nullptr;
        if ((e = cudaMemcpyAsync(x->d_queries, queries + static_cast<size_t>(lo[i]) * x->dim, qn * sizeof(float),
                                 cudaMemcpyHostToDevice, x->stream)) != cudaSuccess)
            return cuda_fail(e, "cudaMemcpyAsync(queries)");
    }
    const auto t0 = std::chrono::high_resolution_clock::now();
    for (int i = 0; i < count; ++i) {
        if (hi[i] == lo[i]) continue;
        DeviceGuard g(indexes[i]->device);
        if ((e = fg::launch_search(args[i], plans[i], indexes[i]->stream)) != cudaSuccess)
            return cuda_fail(e, "search launch");
    }
    for (int i = 0; i < count; ++i) {
        if (hi[i] == lo[i]) continue;
        DeviceGuard g(indexes[i]->device);
        if ((e = cudaStreamSynchronize(indexes[i]->stream)) != cudaSuccess) return cuda_fail(e, "search");
    }
    const auto t1 = std::chrono::high_resolution_clock::now();
    if (elapsed_s) *elapsed_s = std::chrono::duration<double>(t1 - t0).count();
    for (int i = 0; i < count; ++i) {
        fg_index* x = indexes[i];
        const size_t rn = static_cast<size_t>(hi[i] - lo[i]) * K;
        if (rn == 0) continue;
        DeviceGuard g(x->device);
        if ((e = cudaMemcpy(result_idx + static_cast<size_t>(lo[i]) * K, x->d_results, rn * sizeof(uint32_t),
                            cudaMemcpyDeviceToHost)) != cudaSuccess)
            return cuda_fail(e, "cudaMemcpy(results)");
        if (result_dist && (e = cudaMemcpy(result_dist + static_cast<size_t>(lo[i]) * K, x->d_dists,
                                           rn * sizeof(float), cudaMemcpyDeviceToHost)) != cudaSuccess)
            return cuda_fail(e, "cudaMemcpy(distances)");
    }
    return FG_OK;
}

}  // extern "C"

namespace {

// Scratch of fg_search_noalloc: the work counter, the staged queries and the
// staged result ids of one call, all in this fixed array instead of buffers
// from cudaMalloc.  Every call on a device uses the same array, so it holds
// the previous call's data until the next call overwrites it.
static __device__ __align__(256) unsigned char g_noalloc_scratch[FG_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxScratchDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxScratchDevices] = {};

// Address of g_noalloc_scratch on `device` (which must be current), looked
// up once per device by the first fg_search_noalloc call there.
int noalloc_scratch(int device, unsigned char** out) {
    if (device < 0 || device >= kMaxScratchDevices)
        return fail(FG_ERR_UNSUPPORTED, "fg_search_noalloc supports devices 0..%d (got %d)", kMaxScratchDevices - 1, device);
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_ptr[device]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-allocation scratch)");
        g_scratch_ptr[device] = p;
    }
    *out = static_cast<unsigned char*>(g_scratch_ptr[device]);
    return FG_OK;
}

}  // namespace

extern "C" {

int fg_search_noalloc(fg_index* x, int32_t nq, const float* queries, int32_t K, uint32_t* result_idx, int32_t beam,
                      double* elapsed_s) {
    g_err.clear();
    if (!x) return fail(FG_ERR_ARG, "null index");
    if (nq < 0) return fail(FG_ERR_ARG, "nq must be >= 0 (got %d)", nq);
    if (nq > 0 && (!queries || !result_idx)) return fail(FG_ERR_ARG, "null query or result buffer");
    if (elapsed_s) *elapsed_s = 0.0;
    DeviceGuard g(x->device);
    if (g.err != cudaSuccess) return cuda_fail(g.err, "cudaSetDevice");
    fg::SearchArgs a = base_args(x);
    a.nq = nq;
    a.K = K;
    a.beam = beam;
    fg::SearchPlan plan;
    char err[256];
    int rc = fg::plan_search(a, &plan, x->device, err, sizeof(err));
    if (rc) return fail(rc, "%s", err);
    // scratch layout: [work counter | queries nq*dim | result ids nq*K], 256-byte aligned parts
    const size_t qbytes = static_cast<size_t>(nq) * x->dim * sizeof(float);
    const size_t rbytes = static_cast<size_t>(nq) * K * sizeof(uint32_t);
    const size_t q_off = 256, r_off = q_off + ((qbytes + 255) & ~size_t(255));
    if (r_off + rbytes > FG_NOALLOC_SCRATCH_BYTES)
        return fail(FG_ERR_ARG,
                    "fg_search_noalloc: %d queries of dim %llu with K=%d need %zu bytes of scratch, above its fixed "
                    "%d bytes; split the batch or call fg_search",
                    nq, static_cast<unsigned long long>(x->dim), K, r_off + rbytes, FG_NOALLOC_SCRATCH_BYTES);
    unsigned char* s = nullptr;
    if ((rc = noalloc_scratch(x->device, &s)) != FG_OK) return rc;
    if (nq == 0) return FG_OK;
    a.work_counter = reinterpret_cast<uint32_t*>(s);
    a.queries = reinterpret_cast<const float*>(s + q_off);
    a.out_ids = reinterpret_cast<uint32_t*>(s + r_off);
    cudaError_t e;
    if ((e = cudaMemcpyAsync(s + q_off, queries, qbytes, cudaMemcpyHostToDevice, x->stream)) != cudaSuccess)
        return cuda_fail(e, "cudaMemcpyAsync(queries)");
    if ((e = cudaStreamSynchronize(x->stream)) != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
    const auto t0 = std::chrono::high_resolution_clock::now();
    // launch_search zeroes the work counter on the stream before the kernel
    if ((e = fg::launch_search(a, plan, x->stream)) != cudaSuccess) return cuda_fail(e, "search launch");
    if ((e = cudaStreamSynchronize(x->stream)) != cudaSuccess) return cuda_fail(e, "search");
    const auto t1 = std::chrono::high_resolution_clock::now();
    if (elapsed_s) *elapsed_s = std::chrono::duration<double>(t1 - t0).count();
    if ((e = cudaMemcpyAsync(result_idx, s + r_off, rbytes, cudaMemcpyDeviceToHost, x->stream)) != cudaSuccess)
        return cuda_fail(e, "cudaMemcpyAsync(results)");
    if ((e = cudaStreamSynchronize(x->stream)) != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
    return FG_OK;
}

int fg_query_prepare_device(const float* d_queries, int32_t nq, int32_t dim, const float* d_signs, float* d_rotated,
                            uint8_t* d_quant, uint8_t* d_lut, float* d_factors, int32_t* d_sum_q, void* stream) {
    g_err.clear();
    if (nq < 0 || dim < 32 || dim > FG_MAX_DIM) return fail(FG_ERR_ARG, "bad nq %d / dim %d", nq, dim);
    if (nq > 0 && (!d_queries || !d_signs || !d_factors)) return fail(FG_ERR_ARG, "null argument");
    cudaError_t e = fg::launch_query_prepare(d_queries, nq, dim, d_signs, d_rotated, d_quant, d_lut, d_factors, d_sum_q,
                                             static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? FG_OK : cuda_fail(e, "query prepare launch");
}

int fg_beam_merge_device(uint32_t* d_idx, float* d_dist, int32_t ncase, int32_t itopk, int32_t cbs, int32_t first,
                         void* stream) {
    g_err.clear();
    if (ncase < 0 || itopk < 1 || itopk > FG_MAX_BEAM || cbs < 1 || cbs > 32) return fail(FG_ERR_ARG, "bad merge shape");
    if (fg::effective_sort_beam(static_cast<uint32_t>(itopk)) != static_cast<uint32_t>(itopk))
        return fail(FG_ERR_ARG, "itopk %d is not an effective sort beam size", itopk);
    cudaError_t e = fg::launch_beam_merge(d_idx, d_dist, ncase, itopk, cbs, first, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? FG_OK : cuda_fail(e, "merge launch");
}

int fg_shard_merge_device(const uint32_t* d_ids, const float* d_dists, const uint32_t* shard_offsets, int32_t shards,
                          int32_t nq, int32_t k, int32_t K, uint32_t* d_out_ids, float* d_out_dists, void* stream) {
    g_err.clear();
    if (shards < 1 || shards > fg::shard_merge_max_shards())
        return fail(FG_ERR_ARG, "shards %d outside [1, %d]", shards, fg::shard_merge_max_shards());
    if (nq < 0 || k < 1 || K < 1) return fail(FG_ERR_ARG, "bad merge shape nq=%d k=%d K=%d", nq, k, K);
    if (static_cast<int64_t>(shards) * k < K)
        return fail(FG_ERR_ARG, "%d lists of %d entries cannot fill the top-%d", shards, k, K);
    if (static_cast<size_t>(shards) * k * sizeof(float) > 227u * 1024u)
        return fail(FG_ERR_UNSUPPORTED, "%d lists of %d distances exceed one CTA's shared memory", shards, k);
    if (nq == 0) return FG_OK;
    if (!d_ids || !d_dists || !d_out_ids) return fail(FG_ERR_ARG, "null buffer");
    cudaError_t e = fg::launch_shard_merge(d_ids, d_dists, shard_offsets, shards, nq, k, K, d_out_ids, d_out_dists,
                                           static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? FG_OK : cuda_fail(e, "shard merge launch");
}

uint32_t fg_effective_sort_beam_size(uint32_t beam) { return fg::effective_sort_beam(beam); }

uint32_t fg_entry_point_centroid(const float* rows, uint64_t n, uint64_t dim, uint64_t row, int32_t metric) {
    if (!rows || n == 0 || dim == 0 || row < dim) return 0xFFFFFFFFu;
    return centroid_entry(rows, n, dim, row, metric);
}

float fg_compute_recall(const uint32_t* pred, const int32_t* gt, uint64_t nq, int32_t topk, int32_t gt_k) {
    uint64_t correct = 0;
    const int ek = std::min(topk, gt_k);
    for (uint64_t i = 0; i < nq; ++i)
        for (int j = 0; j < topk; ++j) {
            const int p = static_cast<int>(pred[i * topk + j]);
            for (int k = 0; k < ek; ++k)
                if (p == gt[i * gt_k + k]) {
                    ++correct;
                    break;
                }
        }
    return static_cast<float>(correct) / static_cast<float>(nq * static_cast<uint64_t>(topk));
}

int fg_append_run_stats_csv(const char* path, int32_t k, int32_t beam, double runtime, double latency,
                            double throughput, double recall) {
    if (!path) return fail(FG_ERR_ARG, "null path");
    const bool exists = std::filesystem::exists(path);
    std::ofstream out(path, std::ios::app);
    if (!out.is_open()) return fail(FG_ERR_IO, "cannot open CSV file %s", path);
    if (!exists) out << "TopK," << "Beam_size," << "Runtime," << "Latency," << "Throughput," << "Recall\n";
    out << k << "," << beam << "," << runtime << "," << latency << "," << throughput << "," << recall << "\n";
    return out.good() ? FG_OK : fail(FG_ERR_IO, "write to %s failed", path);
}

int32_t fg_infer_metric_from_path(const char* path) {
    if (!path) return FG_METRIC_L2;
    std::string s(path);
    std::transform(s.begin(), s.end(), s.begin(), [](unsigned char c) { return static_cast<char>(std::tolower(c)); });
    return s.find("text2image1m") != std::string::npos ? FG_METRIC_IP : FG_METRIC_L2;
}

int fg_vecs_info(const char* path, uint64_t* count, int32_t* dim) {
    if (!path || !count || !dim) return fail(FG_ERR_ARG, "null argument");
    FILE* f = fopen(path, "rb");
    if (!f) return fail(FG_ERR_IO, "cannot open %s", path);
    int32_t d = 0;
    const size_t got = fread(&d, 4, 1, f);
    fseeko(f, 0, SEEK_END);
    const uint64_t size = static_cast<uint64_t>(ftello(f));
    fclose(f);
    if (got != 1 || d <= 0) {
        *count = 0;
        *dim = got == 1 ? d : 0;
        if (size == 0) return FG_OK;
        return fail(FG_ERR_FORMAT, "%s: bad leading dimension %d", path, d);
    }
    *dim = d;
    *count = size / (4 + 4 * static_cast<uint64_t>(d));
    return FG_OK;
}

int fg_vecs_read(const char* path, void* dst, uint64_t count, int32_t dim) {
    if (!path || (!dst && count)) return fail(FG_ERR_ARG, "null argument");
    FILE* f = fopen(path, "rb");
    if (!f) return fail(FG_ERR_IO, "cannot open %s", path);
    char* out = static_cast<char*>(dst);
    for (uint64_t i = 0; i < count; ++i) {
        int32_t d = 0;
        if (fread(&d, 4, 1, f) != 1 || fread(out + i * 4ull * dim, 4, static_cast<size_t>(dim), f) != static_cast<size_t>(dim)) {
            fclose(f);
            return fail(FG_ERR_IO, "%s: short read at row %llu", path, (unsigned long long)i);
        }
        if (d != dim) {
            fclose(f);
            return fail(FG_ERR_FORMAT, "%s: row %llu has dim %d, expected %d", path, (unsigned long long)i, d, dim);
        }
    }
    fclose(f);
    return FG_OK;
}

}  // extern "C"
