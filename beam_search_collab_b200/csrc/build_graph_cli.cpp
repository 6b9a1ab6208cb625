// build_graph_cli.cpp -- drop-in replacement for the reference graph builder
// build_graph (src/build_graph.cpp): the same arguments and output file,
// with the build running on the GPU through bs_index_build_graph.
//
//   build_graph --base base.fvecs --graph graph.bin [--degree 32]
//               [--beam-width 128] [--alpha 2.0] [--metric l2] [--seed 1234]
//               [--device 0]
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <iostream>
#include <stdexcept>
#include <string>
#include <vector>

#include "bsearch.h"
#include "bs_io.hpp"

int main(int argc, char** argv) {
    try {
        const auto t0 = std::chrono::steady_clock::now();
        std::string base_path, graph_path, metric = "l2";
        int degree = 32, beam_width = 128, device = 0;
        double alpha = 2.0;
        uint32_t seed = 1234;
        for (int i = 1; i < argc; ++i) {
            const std::string arg = argv[i];
            auto value = [&]() -> std::string {
                if (i + 1 >= argc) throw std::runtime_error("Missing value for argument: " + arg);
                return argv[++i];
            };
            if (arg == "--base") base_path = value();
            else if (arg == "--graph") graph_path = value();
            else if (arg == "--degree") degree = std::stoi(value());
            else if (arg == "--beam-width") beam_width = std::stoi(value());
            else if (arg == "--alpha") alpha = std::stod(value());
            else if (arg == "--metric") metric = value();
            else if (arg == "--seed") seed = static_cast<uint32_t>(std::stoul(value()));
            else if (arg == "--device") device = std::stoi(value());
            else if (arg == "--help") {
                std::cout << "Usage: build_graph --base base.fvecs --graph graph.bin [options]\n"
                          << "  --degree <int>       fixed out-degree (default: 32)\n"
                          << "  --beam-width <int>   build beam width L (default: 128)\n"
                          << "  --alpha <float>      Vamana pruning alpha (default: 2.0)\n"
                          << "  --metric <l2>        build distance metric (default: l2)\n"
                          << "  --seed <int>         shuffle seed (default: 1234)\n";
                return 0;
            } else {
                throw std::runtime_error("Unknown argument: " + arg);
            }
        }
        if (base_path.empty()) throw std::runtime_error("Missing required argument: --base");
        if (graph_path.empty()) throw std::runtime_error("Missing required argument: --graph");
        if (degree <= 0) throw std::runtime_error("--degree must be positive");
        if (beam_width <= 0) throw std::runtime_error("--beam-width must be positive");
        if (alpha < 1.0) throw std::runtime_error("--alpha must be at least 1.0");
        if (metric == "ip") throw std::runtime_error("metric ip is not supported by this build");
        if (metric != "l2") throw std::runtime_error("Unsupported metric: " + metric);

        uint64_t n = 0;
        int32_t dim = 0;
        std::vector<float> vecs;
        std::string err;
        if (!bsb::io::read_vecs<float>(base_path, n, dim, vecs, err)) throw std::runtime_error(err);
        if (n == 0) throw std::runtime_error("Base dataset is empty");
        std::cout << "Building Vamana graph: n=" << n << " dim=" << dim << " degree=" << degree
                  << " beam_width=" << beam_width << " alpha=" << alpha << " metric=l2\n";
        bs_index* ix = nullptr;
        bs_graph_desc desc{n, dim, degree, vecs.data(), nullptr};
        if (bs_index_create(&desc, device, &ix) != BS_OK) throw std::runtime_error(bs_last_error());
        std::vector<uint32_t> edges(n * static_cast<uint64_t>(degree));
        bs_graph_build_params prm{beam_width, static_cast<float>(alpha), seed};
        if (bs_index_build_graph(ix, &prm, edges.data()) != BS_OK) {
            const std::string m = bs_last_error();
            bs_index_destroy(ix);
            throw std::runtime_error(m);
        }
        bs_index_destroy(ix);
        // graph.bin: int32 n, int32 degree, uint32[n*degree] (src/build_graph.cpp:131-140)
        std::FILE* f = std::fopen(graph_path.c_str(), "wb");
        if (!f) throw std::runtime_error("Cannot open output graph file: " + graph_path);
        const int32_t n32 = static_cast<int32_t>(n), d32 = degree;
        bool ok = std::fwrite(&n32, 4, 1, f) == 1 && std::fwrite(&d32, 4, 1, f) == 1 &&
                  std::fwrite(edges.data(), 4, edges.size(), f) == edges.size();
        ok = (std::fclose(f) == 0) && ok;
        if (!ok) throw std::runtime_error("Failed writing graph file: " + graph_path);
        const double secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        std::cout << "Wrote graph to " << graph_path << "\n";
        std::cout << "Total build time: " << secs << "s\n";
        return 0;
    } catch (const std::exception& e) {
        std::cerr << "build_graph error: " << e.what() << "\n";
        return 1;
    }
}
