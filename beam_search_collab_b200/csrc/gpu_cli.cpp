// gpu_cli.cpp -- drop-in replacement for the reference gpu_cli
// (src/gpu_cli.cu:353-492): one JSON object on stdin, the same keys,
// defaults, error messages and stdout lines, with the search running through
// the C ABI of libbsearch_b200.so (include/bsearch.h).
//
//   {"data":   {"graph", "base", "query", "gt", "codebook"?},
//    "search": {"mode", "K", "topk_size", "filter_capacity",
//               "max_iterations", "reset_interval"}}
//
// stdout: "Loaded graph/vectors" lines, "data: ...", "search: mode=... K=...",
// ["Loaded rabitq codebook: ..."], "  time: X ms  qps: Y" (mean of 5 launches,
// wall clock, queries already on the device), ["  duplicates: ..."],
// "recall@K: R".  An optional "print_stats": true in "search" adds one
// "  stats: ..." line with the search counters; an optional "results" path in
// "data" receives the result ids as raw uint32 [nq][K] (BS_NO_NODE past the
// end of the beam).  Neither key exists in the reference; both are ignored
// by it.
#include <chrono>
#include <cstdio>
#include <cstdint>
#include <iostream>
#include <iterator>
#include <sstream>
#include <string>
#include <unordered_set>
#include <vector>

#include "bsearch.h"
#include "bs_io.hpp"
#include "json_lite.hpp"

namespace {

// src/gpu_cli.cu:28-51 -- skips -1, counts duplicates, divides by nq*min(K, gt_k)
float compute_recall(const uint32_t* predicted, const int32_t* gt, size_t nq, int topk, int gt_k) {
    size_t correct = 0, dups = 0;
    for (size_t i = 0; i < nq; i++) {
        std::unordered_set<int> gt_set(gt + i * gt_k, gt + (i + 1) * gt_k);
        std::unordered_set<int> seen;
        for (int j = 0; j < topk; j++) {
            const int pred = static_cast<int>(predicted[i * topk + j]);
            if (pred == -1) continue;
            if (!seen.insert(pred).second) { dups++; continue; }
            if (gt_set.count(pred) != 0) correct++;
        }
    }
    if (dups > 0)
        std::cout << "  duplicates: " << dups << " total (" << static_cast<double>(dups) / nq << " avg/query)"
                  << std::endl;
    return static_cast<float>(correct) / (nq * std::min(topk, gt_k));
}

int die(const std::string& msg) {
    std::cerr << msg << std::endl;
    return 1;
}

bool check(bs_status s, const char* what) {
    if (s == BS_OK) return true;
    std::cerr << what << " failed: " << bs_last_error() << std::endl;
    return false;
}

}  // namespace

int main() {
    using bsb::json::Value;
    Value j;
    try {
        const std::string text((std::istreambuf_iterator<char>(std::cin)), std::istreambuf_iterator<char>());
        j = bsb::json::parse(text);
    } catch (const std::exception& e) {
        std::cerr << "JSON parse error: " << e.what() << std::endl;
        return 1;
    }

    try {
        {
            const Value* s = j.find("search");
            const std::string mode = s ? s->value("mode", std::string()) : std::string();
            if (mode.rfind("sophia_", 0) == 0)
                return die("Unknown mode: " + mode + " (the legacy sophia_* modes are not part of this build)");
        }
        if (!j.contains("data")) return die("Missing \"data\" key");
        const Value& jd = *j.find("data");
        auto need = [&](const char* k) -> std::string {
            const Value* v = jd.find(k);
            if (!v || v->kind != Value::String)
                throw std::runtime_error(std::string("[json.exception.out_of_range.403] key '") + k + "' not found");
            return v->str;
        };
        const std::string graph_file = need("graph");
        const std::string base_file = need("base");
        const std::string query_file = need("query");
        const std::string gt_file = need("gt");
        const std::string codebook_file = jd.value("codebook", std::string());
        const std::string results_file = jd.value("results", std::string());

        // graph + base (CPUGraph::load + GPUGraph, include/cpu_graph.hpp:125-173):
        // the files stream straight to the device (bs_index_load)
        bs_index* index = nullptr;
        if (bs_index_load(graph_file.c_str(), base_file.c_str(), 0, &index) != BS_OK) return die(bs_last_error());
        uint64_t n = 0, nq = 0, ngt = 0;
        int32_t degree = 0, dim = 0, qdim = 0, gt_k = 0;
        bs_index_info(index, &n, &dim, &degree);
        std::cout << "Loaded graph: " << n << " nodes, degree " << degree << " from " << graph_file << "\n";
        std::cout << "Loaded vectors: " << n << " x " << dim << " from " << base_file << "\n";
        std::vector<float> queries;
        std::vector<int32_t> gt;
        std::string err;
        if (!bsb::io::read_vecs<float>(query_file, nq, qdim, queries, err)) return die(err);
        if (nq > 0 && qdim != dim) return die("query dimension does not match the base vectors");
        if (!bsb::io::read_vecs<int32_t>(gt_file, ngt, gt_k, gt, err)) return die(err);
        if (ngt < nq) return die("ground truth has fewer rows than queries");
        uint32_t entry = 0;
        if (!check(bs_index_entry_point(index, &entry), "bs_index_entry_point")) return 1;

        void* d_queries = nullptr;
        const size_t qbytes = static_cast<size_t>(nq) * dim * sizeof(float);
        if (!check(bs_device_alloc(index, qbytes, &d_queries), "query upload")) return 1;
        if (!check(bs_copy_to_device(index, d_queries, queries.data(), qbytes), "query upload")) return 1;

        std::cout << "data: " << n << " points, dim=" << dim << ", degree=" << degree << ", queries=" << nq
                  << ", entry=" << entry << std::endl;

        if (!j.contains("search")) return die("Missing \"search\" key");
        const Value& js = *j.find("search");
        bs_search_params prm;
        bs_search_params_default(&prm);
        const std::string mode = js.value("mode", std::string("base"));
        prm.mode = mode.c_str();
        prm.K = static_cast<int32_t>(js.value("K", static_cast<int64_t>(100)));
        if (prm.K <= 0) return die("K must be positive");
        const int K = prm.K;

        void* d_results = nullptr;
        const size_t rbytes = static_cast<size_t>(nq) * K * sizeof(uint32_t);
        if (!check(bs_device_alloc(index, rbytes, &d_results), "result buffer")) return 1;
        if (!check(bs_device_fill(index, d_results, 0xFF, rbytes), "result buffer")) return 1;
        std::vector<uint32_t> h_results(static_cast<size_t>(nq) * K);

        std::cout << "search: mode=" << mode << " K=" << K << std::endl;

        prm.topk_size = static_cast<uint32_t>(js.value("topk_size", static_cast<int64_t>(256)));
        prm.filter_capacity = static_cast<uint32_t>(js.value("filter_capacity", static_cast<int64_t>(1024)));
        prm.max_iterations = static_cast<int32_t>(js.value("max_iterations", static_cast<int64_t>(1024)));
        if (mode == "rabitq") {
            if (codebook_file.empty()) return die("rabitq mode requires \"codebook\" in data config");
            if (!check(bs_index_load_codebook(index, codebook_file.c_str()), "load_rabitq_codebook")) return 1;
            uint32_t rq_entry = BS_NO_NODE;
            bs_index_rabitq_entry(index, &rq_entry);
            int32_t pdim = 1;
            while (pdim < dim) pdim <<= 1;
            std::cout << "Loaded rabitq codebook: " << n << " nodes, dim=" << dim << ", degree=" << degree
                      << ", padded_dim=" << pdim << " (entry=" << rq_entry << ")\n";
            prm.entry_point = rq_entry != BS_NO_NODE ? rq_entry : entry;
        } else {
            prm.reset_interval = static_cast<int32_t>(js.value("reset_interval", static_cast<int64_t>(16)));
            prm.entry_point = entry;
            if (prm.topk_size < static_cast<uint32_t>(K))
                return die("topk_size (" + std::to_string(prm.topk_size) + ") must be >= K (" + std::to_string(K) + ")");
            const bool known = mode == "base" || mode == "warp1" || mode == "warp2" || mode == "warp4" ||
                               mode == "warp8" || mode == "bwarp1" || mode == "bwarp2" || mode == "bwarp4" ||
                               mode == "bwarp8";
            if (!known) return die("Unknown mode: " + mode);
        }

        // src/gpu_cli.cu:153-165: 5 back-to-back launches, one synchronize,
        // wall-clock mean per launch
        bs_stats st{};
        if (!check(bs_search(index, &prm, static_cast<const float*>(d_queries), static_cast<uint32_t>(nq),
                             static_cast<uint32_t*>(d_results), nullptr, &st, nullptr),
                   "search"))
            return 1;
        constexpr int kRuns = 5;
        const auto t0 = std::chrono::high_resolution_clock::now();
        for (int r = 0; r < kRuns; ++r)
            if (!check(bs_search(index, &prm, static_cast<const float*>(d_queries), static_cast<uint32_t>(nq),
                                 static_cast<uint32_t*>(d_results), nullptr, nullptr, nullptr),
                       "search"))
                return 1;
        if (!check(bs_synchronize(index, nullptr), "search")) return 1;
        const auto t1 = std::chrono::high_resolution_clock::now();
        const double elapsed = std::chrono::duration<double>(t1 - t0).count() / kRuns;
        std::cout << "  time: " << elapsed * 1000.0 << " ms"
                  << "  qps: " << nq / elapsed << std::endl;
        if (js.value("print_stats", static_cast<int64_t>(0)) != 0)
            std::cout << "  stats: expansions/q=" << static_cast<double>(st.expansions) / (nq ? nq : 1)
                      << " distances/q=" << static_cast<double>(st.distances) / (nq ? nq : 1)
                      << " estimates/q=" << static_cast<double>(st.estimates) / (nq ? nq : 1)
                      << " integer_exact=" << st.integer_exact << std::endl;

        if (!check(bs_copy_to_host(index, h_results.data(), d_results, rbytes), "result download")) return 1;
        const float recall = compute_recall(h_results.data(), gt.data(), nq, K, gt_k);
        std::cout << "recall@" << K << ": " << recall << std::endl;
        if (!results_file.empty()) {
            std::FILE* f = std::fopen(results_file.c_str(), "wb");
            const bool ok = f && std::fwrite(h_results.data(), sizeof(uint32_t), h_results.size(), f) == h_results.size();
            if (f) std::fclose(f);
            if (!ok) return die("Cannot write results: " + results_file);
        }

        bs_device_free(index, d_queries);
        bs_device_free(index, d_results);
        bs_index_destroy(index);
    } catch (const std::exception& e) {
        std::cerr << e.what() << std::endl;
        return 1;
    }
    return 0;
}
