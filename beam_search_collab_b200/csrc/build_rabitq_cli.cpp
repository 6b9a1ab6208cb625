// build_rabitq_cli.cpp -- drop-in replacement for the reference codebook
// builder's command line (src/build_rabitq.cpp:104-131):
//
//   build_rabitq -base <base.fvecs> -graph <graph.bin> -out <codebook> [-seed <uint32>]
//
// (plus -device <n>).  The build runs on the GPU through the C ABI
// (bs_index_load + bs_index_build_codebook); the file it writes is
// byte-identical to the reference tool's for the same inputs and seed.
// stdout carries the reference's progress lines and one "  time:" line.
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <iostream>
#include <string>

#include "bsearch.h"

int main(int argc, char** argv) {
    std::string base_file, graph_file, out_file;
    uint32_t seed = 12345;
    int device = 0;
    for (int i = 1; i < argc; ++i) {
        const std::string arg = argv[i];
        if (arg == "-base" && i + 1 < argc) base_file = argv[++i];
        else if (arg == "-graph" && i + 1 < argc) graph_file = argv[++i];
        else if (arg == "-out" && i + 1 < argc) out_file = argv[++i];
        else if (arg == "-seed" && i + 1 < argc) seed = static_cast<uint32_t>(std::stoul(argv[++i]));
        else if (arg == "-device" && i + 1 < argc) device = std::stoi(argv[++i]);
    }
    if (base_file.empty() || graph_file.empty() || out_file.empty()) {
        std::cerr << "Usage: " << argv[0] << " -base <base.fvecs> -graph <graph.bin> -out <codebook>"
                  << " [-seed <uint32>]\n";
        return 1;
    }
    // the builder never searches: no neighbourhood blocks (rows repeated per
    // node for the search kernel, 25 GB for a 1M-node degree-64 graph)
    setenv("BSEARCH_LAYOUT", "gather", 0);
    bs_index* index = nullptr;
    if (bs_index_load(graph_file.c_str(), base_file.c_str(), device, &index) != BS_OK) {
        std::cerr << "Error: " << bs_last_error() << "\n";
        return 1;
    }
    uint64_t n = 0;
    int32_t dim = 0, degree = 0;
    bs_index_info(index, &n, &dim, &degree);
    int padded_dim = 1;
    while (padded_dim < dim) padded_dim <<= 1;
    const int wpp = padded_dim / 32;
    std::cout << "dim=" << dim << " padded_dim=" << padded_dim << " degree=" << degree << " n=" << n
              << " words_per_plane=" << wpp << "\n";
    const uint64_t code_off = static_cast<uint64_t>(dim);
    const uint64_t factor_off = code_off + static_cast<uint64_t>(wpp) * degree;
    const uint64_t nbr_off = factor_off + 3ull * degree;
    const uint64_t row_floats = nbr_off + static_cast<uint64_t>(degree);
    std::cout << "Row layout: raw_vec=" << code_off << " codes=" << (factor_off - code_off)
              << " factors=" << (nbr_off - factor_off) << " nbrs=" << degree << " total=" << row_floats
              << " floats\n";
    std::cout << "Quantizing edges...\n";
    const auto t0 = std::chrono::steady_clock::now();
    uint32_t entry = 0;
    if (bs_index_build_codebook(index, seed, out_file.c_str(), &entry) != BS_OK) {
        std::cerr << "Error: " << bs_last_error() << "\n";
        bs_index_destroy(index);
        return 1;
    }
    const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    std::cout << "Entry point (medoid): " << entry << "\n";
    std::cout << "Wrote codebook to " << out_file << "\n";
    std::cout << "Done. Codebook: " << out_file << " ("
              << (sizeof(uint32_t) + n * row_floats * sizeof(float) + padded_dim * sizeof(float)) << " bytes)\n";
    std::cout << "  time: " << ms << " ms (build and file write)\n";
    bs_index_destroy(index);
    return 0;
}
