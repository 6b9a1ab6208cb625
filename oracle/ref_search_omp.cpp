// Test / baseline infrastructure only (never part of the product path).
//
// Multi-threaded driver around the reference's own CPU search classes:
//   CPUBaseSearch::search    (reference include/cpu_search_base.hpp:22-82)
//   CPURabitqSearch::search  (reference include/cpu_search_rabitq.hpp:28-150)
// Both are const and re-entrant, so one instance is shared by all OpenMP
// threads, each thread running whole queries.  This is the "reference CPU,
// all host cores" arm of the benchmark and a second parity oracle.
//
// Usage:
//   ref_search_omp --graph g.bin --base b.fvecs --query q.fvecs
//                  [--codebook cb.bin] [--mode base|rabitq] [--K 10]
//                  [--topk 64] [--max-iter 1024] [--threads N]
//                  [--nq N] [--out ids.u32]
// Prints one JSON line: {"mode":..,"nq":..,"threads":..,"seconds":..,"qps":..,"entry":..}

#include <omp.h>

#include <chrono>
#include <cfloat>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "cpu_graph.hpp"
#include "data_loader.hpp"
#include "rabitq.hpp"
#include "cpu_search_base.hpp"
#include "cpu_search_rabitq.hpp"

// Same float arithmetic as the reference CLIs' entry-point rule
// (reference src/cpu_cli.cpp:35-62): float centroid accumulated as
// row[d] * (1/n), then the first row with the smallest squared distance.
static vid_t centroid_nearest(const CPUGraph& g) {
    const size_t n = g.num_nodes;
    const int dim = g.dim;
    std::vector<float> c(static_cast<size_t>(dim), 0.0f);
    const float inv = 1.0f / static_cast<float>(n);
    for (size_t i = 0; i < n; ++i) {
        const float* row = g.vectors.data() + i * dim;
        for (int d = 0; d < dim; ++d) c[d] += row[d] * inv;
    }
    vid_t best = 0;
    float best_d = FLT_MAX;
    for (size_t i = 0; i < n; ++i) {
        const float* row = g.vectors.data() + i * dim;
        float s = 0.0f;
        for (int d = 0; d < dim; ++d) {
            const float diff = row[d] - c[d];
            s += diff * diff;
        }
        if (s < best_d) { best_d = s; best = static_cast<vid_t>(i); }
    }
    return best;
}

int main(int argc, char** argv) {
    std::string graph, base, query, codebook, mode = "base", out;
    int K = 10, max_iter = 1024, threads = 0;
    unsigned topk = 64;
    long long nq_limit = -1;
    long long entry_override = -1;
    for (int i = 1; i < argc; ++i) {
        std::string a = argv[i];
        auto val = [&]() -> std::string {
            if (i + 1 >= argc) { std::fprintf(stderr, "missing value for %s\n", a.c_str()); std::exit(2); }
            return argv[++i];
        };
        if (a == "--graph") graph = val();
        else if (a == "--base") base = val();
        else if (a == "--query") query = val();
        else if (a == "--codebook") codebook = val();
        else if (a == "--mode") mode = val();
        else if (a == "--K") K = std::stoi(val());
        else if (a == "--topk") topk = static_cast<unsigned>(std::stoul(val()));
        else if (a == "--max-iter") max_iter = std::stoi(val());
        else if (a == "--threads") threads = std::stoi(val());
        else if (a == "--nq") nq_limit = std::stoll(val());
        else if (a == "--entry") entry_override = std::stoll(val());
        else if (a == "--out") out = val();
        else { std::fprintf(stderr, "unknown argument %s\n", a.c_str()); return 2; }
    }
    if (graph.empty() || base.empty() || query.empty()) {
        std::fprintf(stderr, "need --graph --base --query\n");
        return 2;
    }
    if (threads > 0) omp_set_num_threads(threads);

    CPUGraph g;
    g.load(graph, base);
    size_t nq = 0, qd = 0;
    float* q = read_fvecs(query.c_str(), nq, qd);
    if (nq_limit >= 0 && static_cast<size_t>(nq_limit) < nq) nq = static_cast<size_t>(nq_limit);

    vid_t entry = entry_override >= 0 ? static_cast<vid_t>(entry_override) : centroid_nearest(g);
    std::vector<vid_t> res(nq * static_cast<size_t>(K), UINT32_MAX);
    int used_threads = 1;
    double secs = 0.0;

    if (mode == "rabitq") {
        if (codebook.empty()) { std::fprintf(stderr, "rabitq needs --codebook\n"); return 2; }
        CPURabitqData rq = load_rabitq_codebook(codebook, g.num_nodes, g.dim, g.degree);
        if (entry_override < 0 && rq.entry_point != UINT32_MAX) entry = rq.entry_point;
        CPURabitqSearchCfg cfg{topk, entry, max_iter};
        CPURabitqSearch s(g, rq, cfg);
        auto t0 = std::chrono::steady_clock::now();
        #pragma omp parallel
        {
            #pragma omp single
            used_threads = omp_get_num_threads();
            #pragma omp for schedule(dynamic, 4)
            for (long long i = 0; i < static_cast<long long>(nq); ++i)
                s.search(q + static_cast<size_t>(i) * g.dim, res.data() + static_cast<size_t>(i) * K, K);
        }
        secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    } else if (mode == "base") {
        CPUBaseSearchCfg cfg{topk, entry, max_iter};
        CPUBaseSearch s(g, cfg);
        auto t0 = std::chrono::steady_clock::now();
        #pragma omp parallel
        {
            #pragma omp single
            used_threads = omp_get_num_threads();
            #pragma omp for schedule(dynamic, 4)
            for (long long i = 0; i < static_cast<long long>(nq); ++i)
                s.search(q + static_cast<size_t>(i) * g.dim, res.data() + static_cast<size_t>(i) * K, K);
        }
        secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    } else {
        std::fprintf(stderr, "Unknown mode: %s\n", mode.c_str());
        return 1;
    }

    if (!out.empty()) {
        FILE* f = std::fopen(out.c_str(), "wb");
        if (!f) { std::fprintf(stderr, "cannot write %s\n", out.c_str()); return 1; }
        std::fwrite(res.data(), sizeof(vid_t), res.size(), f);
        std::fclose(f);
    }
    std::printf("{\"mode\": \"%s\", \"nq\": %zu, \"threads\": %d, \"seconds\": %.6f, \"qps\": %.3f, \"entry\": %u}\n",
                mode.c_str(), nq, used_threads, secs, secs > 0 ? nq / secs : 0.0, entry);
    delete[] q;
    return 0;
}
