// qg_compat.hpp -- the reference's C++ class API over libflashgann.so.
//
// Drop-in for SophiaSun18/FlashGANN's include/qg.hpp (class
// QuantizationGraph, include/qg.hpp:14-89) together with its implementation
// in gpu_search_adaptive.cu:12-114: put this file in place of include/qg.hpp
// (or include it from there), drop gpu_search_adaptive.cu from the build and
// link libflashgann.so.  The reference's main.cu then builds unchanged.
//
// Same names, argument meaning and error behaviour as the reference class:
//   * the constructor reads the qg_codebook file and throws
//     std::runtime_error("Cannot open codebook file: <path>") when it cannot
//     be opened (include/qg.hpp:22-23);
//   * gpu_search_adaptive(nq, queries, K, result_idx, beam_sz, elapsed) takes
//     host buffers, is synchronous, runs on the current device and sets
//     `elapsed` to the seconds of the search launch and its synchronisation
//     (gpu_search_adaptive.cu:98-107);
//   * a CUDA error prints to stderr and exits with EXIT_FAILURE, as the
//     reference's CUDA_SAFE_CALL does (include/utils.cuh:42-50); too little
//     free device memory throws std::runtime_error("QG upload exceeds
//     currently available GPU memory") (gpu_search_adaptive.cu:61-63).
// Differences: the codebook is uploaded once, in the constructor, and stays
// resident until destruction (the reference uploads and frees it on every
// search), so the memory error comes from the constructor; a configuration
// outside this build's envelope (dim < 32 or > 4096, degree > 32, beam >
// 1024) and a malformed file throw std::runtime_error where the reference
// would read out of bounds; the object is not copyable (the reference's
// implicit copy frees its buffers twice).  get_data_ptr() / get_signs_ptr()
// return host copies read from the file on first use.
//
// When the reference's common.hpp and metric.hpp are on the include path (as
// they are next to include/qg.hpp) they provide vidType and MetricType, as
// they do for the reference's qg.hpp; otherwise this header defines both with
// the reference's values.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#if __has_include("common.hpp") && __has_include("metric.hpp")
#include "common.hpp"
#include "metric.hpp"
#else
typedef uint32_t vidType;                   // include/common.hpp:15
enum MetricType { METRIC_L2, METRIC_IP };  // include/metric.hpp:9
#endif

#include "flashgann.h"

class QuantizationGraph {
public:
    QuantizationGraph(size_t num_node, size_t dim, int degree, const std::string& codebook_path)
        : path_(codebook_path) {
        const int rc = fg_index_load(codebook_path.c_str(), num_node, dim, degree, FG_METRIC_L2, FG_DEVICE_CURRENT,
                                     &index_);
        if (rc != FG_OK) fail(rc, "fg_index_load");
        if (fg_index_layout(index_, &layout_) != FG_OK) fail(FG_ERR_ARG, "fg_index_layout");
        printf("Loaded codebook: %zu nodes, dim=%zu, degree=%d, padded_dim=%zu, row_offset=%zu floats (entry_point=%u)\n",
               static_cast<size_t>(layout_.num_nodes), static_cast<size_t>(layout_.dim), layout_.degree,
               static_cast<size_t>(layout_.padded_dim), static_cast<size_t>(layout_.row_offset), layout_.entry_point);
    }

    ~QuantizationGraph() { fg_index_free(index_); }

    QuantizationGraph(const QuantizationGraph&) = delete;
    QuantizationGraph& operator=(const QuantizationGraph&) = delete;

    const float* get_data_ptr() const {
        load_host_copy();
        return host_rows_.data();
    }
    const float* get_signs_ptr() const {
        load_host_copy();
        return host_signs_.data();
    }
    size_t get_data_bytes() const { return static_cast<size_t>(layout_.num_nodes * layout_.row_offset * sizeof(float)); }
    size_t get_signs_bytes() const { return static_cast<size_t>(layout_.padded_dim * sizeof(float)); }
    MetricType get_metric() const { return metric_; }
    void set_metric(MetricType metric) {
        const int rc = fg_index_set_metric(index_, metric == METRIC_IP ? FG_METRIC_IP : FG_METRIC_L2);
        if (rc != FG_OK) fail(rc, "fg_index_set_metric");
        metric_ = metric;
    }

    size_t get_code_offset() const { return static_cast<size_t>(layout_.code_offset); }
    size_t get_factor_offset() const { return static_cast<size_t>(layout_.factor_offset); }
    size_t get_neighbor_offset() const { return static_cast<size_t>(layout_.neighbor_offset); }
    size_t get_row_offset() const { return static_cast<size_t>(layout_.row_offset); }
    vidType get_entry_point() const { return static_cast<vidType>(layout_.entry_point); }

    void gpu_search_adaptive(int nq, const float* queries, int K, vidType* result_idx, int beam_sz, double& elapsed) {
        static_assert(sizeof(vidType) == sizeof(uint32_t), "vidType is a 32-bit node id");
        const int rc = fg_search(index_, nq, queries, K, reinterpret_cast<uint32_t*>(result_idx), beam_sz, &elapsed);
        if (rc != FG_OK) fail(rc, "gpu_search_adaptive");
    }

private:
    [[noreturn]] void fail(int rc, const char* what) const {
        const std::string msg = std::string(what) + ": " + fg_last_error();
        if (rc == FG_ERR_CUDA || rc == FG_ERR_NO_DEVICE) {
            fprintf(stderr, "CUDA error in %s\n", msg.c_str());
            exit(EXIT_FAILURE);
        }
        if (rc == FG_ERR_IO && index_ == nullptr && strncmp(fg_last_error(), "cannot open", 11) == 0)
            throw std::runtime_error("Cannot open codebook file: " + path_);
        if (rc == FG_ERR_OOM) throw std::runtime_error("QG upload exceeds currently available GPU memory (" + msg + ")");
        throw std::runtime_error(msg);
    }

    // qg_codebook: u32 entry point, num_nodes rows of row_offset floats, padded_dim signs
    void load_host_copy() const {
        if (!host_rows_.empty() || layout_.num_nodes == 0) return;
        FILE* f = fopen(path_.c_str(), "rb");
        if (!f) throw std::runtime_error("Cannot open codebook file: " + path_);
        std::vector<float> rows(static_cast<size_t>(layout_.num_nodes * layout_.row_offset));
        std::vector<float> signs(static_cast<size_t>(layout_.padded_dim));
        uint32_t entry = 0;
        const bool ok = fread(&entry, 4, 1, f) == 1 && fread(rows.data(), sizeof(float), rows.size(), f) == rows.size() &&
                        fread(signs.data(), sizeof(float), signs.size(), f) == signs.size();
        fclose(f);
        if (!ok) throw std::runtime_error("short codebook file: " + path_);
        host_rows_.swap(rows);
        host_signs_.swap(signs);
    }

    std::string path_;
    fg_index* index_ = nullptr;
    fg_layout layout_{};
    MetricType metric_ = METRIC_L2;
    mutable std::vector<float> host_rows_;
    mutable std::vector<float> host_signs_;
};
