// fg_cli.cpp -- the gpu_flashgann command line, drop-in for the reference's
// main.cu:11-109 (same positional arguments, optional -csv, stdout lines and
// CSV row), running the search through libflashgann's C ABI.
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "../../include/flashgann.h"
#include "fg_config.h"

namespace {

int die(int rc, const char* what) {
    fprintf(stderr, "Error: %s: %s (%s)\n", what, fg_status_string(rc), fg_last_error());
    return 1;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 5) {
        fprintf(stderr,
                "Usage: %s <data.fvecs> <query.fvecs> <gt.ivecs> <qg_codebook> [K=100] [beam_size=128] [degree=32] "
                "[-csv output.csv] [-device N] [-gpus G]\n",
                argv[0]);
        return 1;
    }
    const char* data_file = argv[1];
    const char* query_file = argv[2];
    const char* gt_file = argv[3];
    const char* codebook = argv[4];
    int K = 100, beam = 128, degree = 32, device = 0, gpus = 1;
    std::string csv;
    int ai = 5;
    if (ai < argc && argv[ai][0] != '-') K = atoi(argv[ai++]);
    if (ai < argc && argv[ai][0] != '-') beam = atoi(argv[ai++]);
    if (ai < argc && argv[ai][0] != '-') degree = atoi(argv[ai++]);
    while (ai < argc) {
        std::string a = argv[ai];
        if (a == "-csv" && ai + 1 < argc) {
            csv = argv[++ai];
        } else if (a == "-device" && ai + 1 < argc) {
            device = atoi(argv[++ai]);
        } else if (a == "-gpus" && ai + 1 < argc) {
            gpus = atoi(argv[++ai]);
            if (gpus < 1) {
                fprintf(stderr, "-gpus needs a count >= 1\n");
                return 1;
            }
        } else {
            fprintf(stderr, "Unknown argument: %s\n", a.c_str());
            return 1;
        }
        ++ai;
    }
    printf("========================================\n");
    printf("FlashGANN-B200 loading from:\n");
    printf("========================================\n");
    printf("Data file: %s\n", data_file);
    printf("Query file: %s\n", query_file);
    printf("Ground truth: %s\n", gt_file);
    printf("QG codebook: %s\n", codebook);
    printf("K: %d\n", K);
    printf("Beam size: %d\n", beam);
    printf("Degree: %d\n", degree);
    if (!csv.empty()) printf("CSV output: %s\n", csv.c_str());
    const int metric = fg_infer_metric_from_path(data_file);
    printf("Metric: %s\n", metric == FG_METRIC_IP ? "ip" : "l2");
    printf("Internal top-k (build knob): %d\n", INTERNAL_TOPK);
    printf("========================================\n\n");

    uint64_t n = 0, nq = 0, gt_nq = 0;
    int dim = 0, qdim = 0, gt_k = 0;
    int rc;
    if ((rc = fg_vecs_info(data_file, &n, &dim))) return die(rc, "data");
    if ((rc = fg_vecs_info(query_file, &nq, &qdim))) return die(rc, "queries");
    if ((rc = fg_vecs_info(gt_file, &gt_nq, &gt_k))) return die(rc, "ground truth");
    printf("Loading data: n=%llu, dim=%d\n", (unsigned long long)n, dim);
    printf("Loading queries: n=%llu, dim=%d\n", (unsigned long long)nq, qdim);
    printf("Loading ground truth: n=%llu, dim=%d\n", (unsigned long long)gt_nq, gt_k);
    if (qdim != dim) {
        fprintf(stderr, "Query dimension %d does not match data dimension %d\n", qdim, dim);
        return 1;
    }
    if (gt_nq != nq) {
        fprintf(stderr, "Ground-truth query count %llu does not match query count %llu\n", (unsigned long long)gt_nq,
                (unsigned long long)nq);
        return 1;
    }
    std::vector<float> queries(nq * static_cast<uint64_t>(dim));
    std::vector<int32_t> gt(gt_nq * static_cast<uint64_t>(gt_k));
    if ((rc = fg_vecs_read(query_file, queries.data(), nq, qdim))) return die(rc, "queries");
    if ((rc = fg_vecs_read(gt_file, gt.data(), gt_nq, gt_k))) return die(rc, "ground truth");

    // -gpus G: the codebook on devices device .. device+G-1, the batch split across them
    std::vector<fg_index*> indexes(gpus, nullptr);
    auto free_all = [&]() {
        for (fg_index* x : indexes) fg_index_free(x);
    };
    for (int g = 0; g < gpus; ++g) {
        if ((rc = fg_index_load(codebook, n, static_cast<uint64_t>(dim), degree, metric, device + g, &indexes[g]))) {
            free_all();
            return die(rc, "codebook");
        }
    }
    fg_index* index = indexes[0];
    fg_layout L;
    fg_index_layout(index, &L);
    printf("Loaded codebook: %llu nodes, dim=%llu, degree=%d, padded_dim=%llu, row_offset=%llu floats (entry_point=%u)\n",
           (unsigned long long)L.num_nodes, (unsigned long long)L.dim, L.degree, (unsigned long long)L.padded_dim,
           (unsigned long long)L.row_offset, L.entry_point);

    std::vector<uint32_t> results(nq * static_cast<uint64_t>(K));
    double elapsed = 0.0;
    rc = gpus == 1 ? fg_search(index, static_cast<int32_t>(nq), queries.data(), K, results.data(), beam, &elapsed)
                   : fg_search_multi(indexes.data(), gpus, static_cast<int32_t>(nq), queries.data(), K, results.data(),
                                     nullptr, beam, &elapsed);
    free_all();
    if (rc) return die(rc, "search");

    const float recall = fg_compute_recall(results.data(), gt.data(), nq, K, gt_k) * 100.0f;
    const double latency_ms = nq > 0 ? elapsed * 1000.0 / static_cast<double>(nq) : 0.0;
    const double qps = elapsed > 0.0 ? static_cast<double>(nq) / elapsed : 0.0;
    printf("\n========================================\n");
    printf("Results\n");
    printf("========================================\n");
    printf("Total time: %.6f ms\n", elapsed * 1000.0);
    printf("Throughput: %.6f queries/sec\n", qps);
    printf("Avg latency: %.6f ms/query\n", latency_ms);
    printf("Recall@%d: %.6f\n", K, recall);
    printf("========================================\n");
    if (!csv.empty()) {
        if ((rc = fg_append_run_stats_csv(csv.c_str(), K, beam, elapsed, latency_ms, qps, recall)))
            return die(rc, "csv");
        printf("Saved GPU stats CSV row to: %s\n", csv.c_str());
    }
    return 0;
}
