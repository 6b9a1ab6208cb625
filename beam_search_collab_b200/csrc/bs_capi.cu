// bs_capi.cu -- implementation of the C ABI declared in include/bsearch.h.
//
// Index residency in HBM:
//   vectors   [n][row_stride] f32, row_stride = dim rounded up to 4 (zero pad),
//             so every row starts on a 16-byte boundary for vector / cp.async loads
//   adjacency [n][degree] u32, the graph.bin payload unchanged
//   codes     [n][degree][wpp] u32, factors [n][3][degree] f32, signs [pdim] f32
//             (RaBitQ, the codebook row layout of include/rabitq.hpp:61-64 with
//             the raw-vector and neighbour-id slots dropped)
// Per call: a stream-ordered scratch block (counters, and staging for host
// buffers) from cudaMallocAsync, released on the same stream.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <initializer_list>
#include <mutex>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include "bsearch.h"
#include "bs_internal.h"
#include "bs_io.hpp"

using bsb::DevCounters;
using bsb::LaunchShape;
using bsb::SearchParams;

struct bs_index {
    int device = 0;
    int num_sms = 0;
    size_t smem_optin = 0;
    uint64_t n = 0;
    int32_t dim = 0;
    int32_t degree = 0;
    uint32_t row_stride = 0;
    float* d_vecs = nullptr;     // f32 rows, or null when stored as bytes
    bool u8 = false;             // rows stored as an exact u8 copy
    uint32_t row_bytes = 0;
    uint8_t* d_vecs8 = nullptr;
    uint32_t* d_adj = nullptr;
    // neighbourhood blocks (adjacency row + neighbour rows per node), built
    // when they fit comfortably in device memory
    unsigned char* d_nb = nullptr;
    uint32_t nb_stride = 0, nb_adj_bytes = 0, nb_pitch = 0;
    bool nb_tried = false;       // the blocks are built on first need (or never)
    bool gather_only = false;    // BSEARCH_LAYOUT=gather at creation: no blocks of any kind
    bool int_exact = false;      // every base value an integer
    std::vector<uint64_t> neg_zeros;  // byte rows: flat positions of -0.0 values (ascending)
    float min_val = 0.0f;        // range of the base values
    float max_val = 0.0f;
    // RaBitQ
    bool has_rabitq = false;
    uint32_t rq_entry = BS_NO_NODE;
    int32_t pdim = 0;
    uint32_t* d_codes = nullptr;
    float* d_factors = nullptr;
    float* d_signs = nullptr;
    // RaBitQ node blocks [adjacency | codes | factors | own row], one bulk
    // copy per expansion (null: the gather kernel)
    unsigned char* d_rqb = nullptr;
    uint32_t rq_stride = 0, rq_off_codes = 0, rq_off_fac = 0, rq_off_row = 0;
    // RaBitQ visited arena (per resident warp: bitmap + log), kept between
    // calls and all zero between queries; rabitq calls on this index are
    // ordered one after another through rq_event
    std::mutex rq_mu;
    uint32_t* d_vis = nullptr;
    uint64_t vis_warps = 0;
    uint32_t vis_words = 0, vis_log_cap = 0;
    cudaEvent_t rq_event = nullptr;
    // error word every search kernel on this index ORs its error bits into
    // (read and cleared by bs_index_take_errors)
    unsigned int* d_err = nullptr;
    // cached centroid-nearest entry
    std::mutex mu;
    bool entry_valid = false;
    uint32_t entry = 0;
};

namespace {

thread_local std::string g_err;

bs_status fail(bs_status s, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return s;
}

bs_status cuda_fail(cudaError_t e, const char* what) {
    if (e == cudaErrorMemoryAllocation)
        return fail(BS_ERR_OUT_OF_MEMORY, "%s: %s", what, cudaGetErrorString(e));
    return fail(BS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Makes the index's device current for the scope and restores the caller's.
struct DeviceGuard {
    int prev = -1;
    bool ok = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

// Where a buffer lives, seen from `device`.
enum PtrKind { kHostPtr = 0, kThisDevice = 1, kOtherDevice = 2 };

PtrKind pointer_kind(const void* ptr, int device) {
    if (!ptr) return kHostPtr;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess) {
        cudaGetLastError();   // clear the sticky-free error of an unknown pointer
        return kHostPtr;
    }
    if (a.type == cudaMemoryTypeManaged) return kThisDevice;   // reachable from every device
    if (a.type == cudaMemoryTypeDevice) return a.device == device ? kThisDevice : kOtherDevice;
    return kHostPtr;
}

// true: device memory usable by kernels on `device` (its own memory, or
// managed memory).
bool is_device_ptr(const void* ptr, int device) { return pointer_kind(ptr, device) == kThisDevice; }

// Device memory of another GPU given to a search on `device`: kernels would
// read it across the bus (or fault without peer access), so it is refused.
bool any_foreign(int device, std::initializer_list<const void*> ptrs) {
    for (const void* p : ptrs)
        if (p && pointer_kind(p, device) == kOtherDevice) return true;
    return false;
}

// Page-locked host memory that `device`'s context has mapped: the device
// address its kernels read and write it through, else null (pageable memory,
// or pinned by another device's context).
void* mapped_host_ptr(const void* ptr, int device) {
    if (!ptr) return nullptr;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return (a.type == cudaMemoryTypeHost && a.device == device) ? a.devicePointer : nullptr;
}

struct ModeInfo {
    bool rabitq = false;
    bsb::FilterMode fmode = bsb::kHash;
    int warps = 4;
    bool block = false;     // base: one thread block per query (when the blocks fit)
};

bool parse_mode(const char* m, ModeInfo& mi) {
    if (!m) return false;
    const std::string s(m);
    if (s == "base") { mi = {false, bsb::kHash, 4, true}; return true; }
    if (s == "rabitq") { mi = {true, bsb::kHash, 4}; return true; }
    const struct { const char* name; bsb::FilterMode f; int w; } table[] = {
        {"warp1", bsb::kHash, 1},   {"warp2", bsb::kHash, 2},   {"warp4", bsb::kHash, 4},
        {"warp8", bsb::kHash, 8},   {"bwarp1", bsb::kBloom, 1}, {"bwarp2", bsb::kBloom, 2},
        {"bwarp4", bsb::kBloom, 4}, {"bwarp8", bsb::kBloom, 8},
    };
    for (const auto& t : table)
        if (s == t.name) { mi = {false, t.f, t.w}; return true; }
    return false;
}

// Range of the values, whether every value is an integer and whether any is
// -0.0 (multi-threaded scan of the host array at index creation).
void scan_values(const float* v, uint64_t count, bool& all_int, std::vector<uint64_t>& neg_zeros, float& min_val,
                 float& max_val) {
    unsigned nt = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    if (count < (1u << 20)) nt = 1;
    std::vector<char> ints(nt, 1);
    std::vector<std::vector<uint64_t>> nzs(nt);
    std::vector<float> mins(nt, 0.0f), maxes(nt, 0.0f);
    std::vector<std::thread> th;
    const uint64_t per = (count + nt - 1) / nt;
    for (unsigned t = 0; t < nt; ++t) {
        th.emplace_back([&, t] {
            const uint64_t lo = per * t, hi = std::min(count, lo + per);
            bool ok = true;
            float mn = lo < hi ? v[lo] : 0.0f, mx = mn;
            for (uint64_t i = lo; i < hi; ++i) {
                const float x = v[i];
                ok = ok && (x == std::nearbyint(x));   // false for NaN and inf
                if (x == 0.0f && std::signbit(x)) nzs[t].push_back(i);
                mn = x < mn ? x : mn;
                mx = x > mx ? x : mx;
            }
            ints[t] = ok;
            mins[t] = mn;
            maxes[t] = mx;
        });
    }
    for (auto& t : th) t.join();
    all_int = true;
    neg_zeros.clear();
    min_val = mins[0];
    max_val = maxes[0];
    for (unsigned t = 0; t < nt; ++t) {
        if (per * t >= count) continue;
        all_int = all_int && ints[t];
        neg_zeros.insert(neg_zeros.end(), nzs[t].begin(), nzs[t].end());
        min_val = std::min(min_val, mins[t]);
        max_val = std::max(max_val, maxes[t]);
    }
}

// Query value range for the integer-exact path: with B = floor(sqrt(2^24/dim))
// every |q_d - x_d| <= B keeps dim * B^2 <= 2^24, so all partial sums of the
// squared differences are exact integers.  Empty range (lo > hi) = never.
void team_range_for(const bs_index* ix, float& lo, float& hi) {
    lo = 1.0f;
    hi = 0.0f;
    if (!ix->int_exact) return;
    const double B = std::floor(std::sqrt(16777216.0 / ix->dim));
    const double l = static_cast<double>(ix->max_val) - B, h = static_cast<double>(ix->min_val) + B;
    if (l > h) return;
    lo = static_cast<float>(l);
    hi = static_cast<float>(h);
}

bool force_seq() {
    const char* e = std::getenv("BSEARCH_FORCE_SEQ");
    return e && e[0] && e[0] != '0';
}

// BSEARCH_STORAGE=f32 keeps f32 rows even for byte-valued data (lets the
// tests compare both storages).
bool storage_f32_forced() {
    const char* e = std::getenv("BSEARCH_STORAGE");
    return e && std::strcmp(e, "f32") == 0;
}

// rows of dim floats (integers in [0,255]) -> rows of row_bytes bytes, zero pad
void pack_u8_rows(const float* v, uint64_t n, int32_t dim, uint32_t row_bytes, uint8_t* out) {
    unsigned nt = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    if (n < (1u << 16)) nt = 1;
    std::vector<std::thread> th;
    const uint64_t per = (n + nt - 1) / nt;
    for (unsigned t = 0; t < nt; ++t) {
        th.emplace_back([=] {
            const uint64_t lo = per * t, hi = std::min(n, lo + per);
            for (uint64_t i = lo; i < hi; ++i)
                for (int32_t d = 0; d < dim; ++d)
                    out[i * row_bytes + d] = static_cast<uint8_t>(v[i * dim + d]);
        });
    }
    for (auto& t : th) t.join();
}

// Neighbourhood blocks (one contiguous [adjacency | neighbour rows] block
// per node, so that an expansion is one bulk copy).  Built when the blocks
// take at most 40% of the device's free memory; BSEARCH_LAYOUT=gather turns
// them off.  Row pitch: the stored row, grown to an odd number of 16-byte
// units for f32 rows so that lanes reading one row each hit distinct banks
// (u8 rows rotate their chunks instead).
cudaError_t build_blocks(bs_index* ix) {
    ix->nb_tried = true;
    if (ix->gather_only) return cudaSuccess;
    if (ix->degree > 64) return cudaSuccess;                    // the search supports degree <= 64
    uint32_t pitch;
    if (ix->u8) {
        pitch = ix->row_bytes;
    } else {
        pitch = ix->row_stride * 4u;
        if ((pitch / 16u) % 2u == 0u) pitch += 16u;
    }
    const uint32_t adj_bytes = (static_cast<uint32_t>(ix->degree) * 4u + 15u) & ~15u;
    const uint64_t stride = adj_bytes + static_cast<uint64_t>(ix->degree) * pitch;
    if (stride > 64u * 1024u) return cudaSuccess;              // one block must fit a warp's shared memory
    const uint64_t bytes = stride * ix->n;
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) { cudaGetLastError(); return cudaSuccess; }
    if (bytes > free_b / 5u * 2u) return cudaSuccess;
    if (cudaMalloc(&ix->d_nb, bytes) != cudaSuccess) {
        cudaGetLastError();
        ix->d_nb = nullptr;
        return cudaSuccess;
    }
    ix->nb_stride = static_cast<uint32_t>(stride);
    ix->nb_adj_bytes = adj_bytes;
    ix->nb_pitch = pitch;
    SearchParams p{};
    p.vecs = ix->d_vecs;
    p.vecs8 = ix->d_vecs8;
    p.row_bytes = ix->row_bytes;
    p.row_stride = ix->row_stride;
    p.adj = ix->d_adj;
    p.n = ix->n;
    p.degree = static_cast<uint32_t>(ix->degree);
    p.nb_stride = ix->nb_stride;
    p.nb_adj_bytes = adj_bytes;
    p.nb_pitch = pitch;
    cudaError_t e = bsb::build_neighbourhood_blocks(p, ix->d_nb, nullptr);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return e;
}

// The neighbourhood blocks of the exact and Bloom modes, built once, on the
// first search that can use them (a RaBitQ-only index never pays their
// memory).  Called with ix->mu held.
bs_status ensure_blocks(bs_index* ix) {
    if (ix->nb_tried) return BS_OK;
    const cudaError_t e = build_blocks(ix);
    return e == cudaSuccess ? BS_OK : cuda_fail(e, "neighbourhood blocks");
}

// RaBitQ node blocks [adjacency | codes | factors | own row] (16-byte aligned
// parts), built on the GPU from the attached codebook when they take at most
// 40% of the free memory; BSEARCH_LAYOUT=gather keeps the gather kernel.
cudaError_t build_rq_blocks(bs_index* ix) {
    cudaFree(ix->d_rqb);
    ix->d_rqb = nullptr;
    if (ix->gather_only) return cudaSuccess;
    if (ix->degree > 64) return cudaSuccess;
    auto a16 = [](uint64_t x) { return (x + 15u) & ~static_cast<uint64_t>(15u); };
    const uint64_t deg = static_cast<uint64_t>(ix->degree), wpp = static_cast<uint64_t>(ix->pdim) / 32u;
    const uint64_t off_codes = a16(4u * deg);
    const uint64_t off_fac = a16(off_codes + 4u * deg * wpp);
    const uint64_t off_row = a16(off_fac + 12u * deg);
    const uint64_t stride = a16(off_row + (ix->u8 ? ix->row_bytes : ix->row_stride * 4u));
    if (stride > 48u * 1024u) return cudaSuccess;
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) { cudaGetLastError(); return cudaSuccess; }
    const uint64_t bytes = stride * ix->n;
    if (bytes > free_b / 5u * 2u) return cudaSuccess;
    if (cudaMalloc(&ix->d_rqb, bytes) != cudaSuccess) {
        cudaGetLastError();
        ix->d_rqb = nullptr;
        return cudaSuccess;
    }
    ix->rq_stride = static_cast<uint32_t>(stride);
    ix->rq_off_codes = static_cast<uint32_t>(off_codes);
    ix->rq_off_fac = static_cast<uint32_t>(off_fac);
    ix->rq_off_row = static_cast<uint32_t>(off_row);
    SearchParams p{};
    p.vecs = ix->d_vecs;
    p.vecs8 = ix->d_vecs8;
    p.row_bytes = ix->row_bytes;
    p.row_stride = ix->row_stride;
    p.adj = ix->d_adj;
    p.n = ix->n;
    p.degree = static_cast<uint32_t>(ix->degree);
    p.codes = ix->d_codes;
    p.factors = ix->d_factors;
    p.wpp = static_cast<uint32_t>(wpp);
    p.rq_stride = ix->rq_stride;
    p.rq_off_codes = ix->rq_off_codes;
    p.rq_off_fac = ix->rq_off_fac;
    p.rq_off_row = ix->rq_off_row;
    cudaError_t e = bsb::build_rabitq_blocks(p, ix->d_rqb, nullptr);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return e;
}

// The RaBitQ visited arena for `warps` resident warps: one bitmap over the
// node ids and one log per warp, zeroed once.  Shrinks the warps to fit a
// quarter of the free memory.  Called with ix->rq_mu held.
bs_status ensure_visited_arena(bs_index* ix, uint64_t warps, uint32_t warps_per_block) {
    const uint32_t words = static_cast<uint32_t>(((ix->n + 31u) / 32u + 3u) & ~3ull);
    // ids one query may log before its end clears the whole bitmap instead;
    // BSEARCH_RQ_LOG_CAP overrides it (tests reach the whole-bitmap path)
    uint32_t kLogCap = 16384;
    if (const char* c = std::getenv("BSEARCH_RQ_LOG_CAP")) kLogCap = static_cast<uint32_t>(std::strtoul(c, nullptr, 10));
    kLogCap = (kLogCap + 3u) & ~3u;
    if (ix->d_vis && ix->vis_warps >= warps && ix->vis_words == words) return BS_OK;
    cudaError_t e;
    if (!ix->rq_event && (e = cudaEventCreateWithFlags(&ix->rq_event, cudaEventDisableTiming)) != cudaSuccess)
        return cuda_fail(e, "rabitq event");
    if (ix->d_vis) {
        // the previous arena may still be in use by a queued search
        if ((e = cudaEventSynchronize(ix->rq_event)) != cudaSuccess) return cuda_fail(e, "rabitq arena");
        cudaFree(ix->d_vis);
        ix->d_vis = nullptr;
        ix->vis_warps = 0;
    }
    const uint64_t per_warp = (static_cast<uint64_t>(words) + kLogCap) * 4u;
    size_t free_b = 0, total_b = 0;
    if ((e = cudaMemGetInfo(&free_b, &total_b)) != cudaSuccess) return cuda_fail(e, "cudaMemGetInfo");
    uint64_t fit = (free_b / 4u) / per_warp;
    fit -= fit % warps_per_block;
    if (warps > fit) warps = fit;
    if (warps < warps_per_block)
        return fail(BS_ERR_OUT_OF_MEMORY, "RaBitQ visited arena: %llu bytes per warp do not fit",
                    static_cast<unsigned long long>(per_warp));
    if ((e = cudaMalloc(&ix->d_vis, warps * per_warp)) != cudaSuccess) return cuda_fail(e, "rabitq visited arena");
    if ((e = cudaMemset(ix->d_vis, 0, warps * per_warp)) != cudaSuccess) return cuda_fail(e, "rabitq visited arena");
    ix->vis_warps = warps;
    ix->vis_words = words;
    ix->vis_log_cap = kLogCap;
    return BS_OK;
}

// Plans the launch; when a neighbourhood block per warp does not fit the
// requested warps per block in shared memory, plans the gather layout.
cudaError_t plan(const bs_index* ix, SearchParams& p, LaunchShape& shape, char* why, size_t why_len) {
    if (p.rq_nb) {
        SearchParams p1 = p;
        LaunchShape s1 = shape;
        if (bsb::plan_search_rq_nb(p1, s1, ix->smem_optin, why, why_len) == cudaSuccess) {
            p = p1;
            shape = s1;
            return cudaSuccess;
        }
        p.rq_nb = nullptr;   // the gather kernel
    }
    if (shape.block_query) {
        // base: one thread block per query over the neighbourhood blocks;
        // without them (blocks too large or off) the warp kernels below
        SearchParams p1 = p;
        LaunchShape s1 = shape;
        if (p.nb != nullptr && bsb::plan_search_bq(p1, s1, ix->smem_optin, why, why_len) == cudaSuccess) {
            p = p1;
            shape = s1;
            return cudaSuccess;
        }
        shape.block_query = 0;
    }
    SearchParams p0 = p;
    const LaunchShape s0 = shape;
    const cudaError_t e = bsb::plan_search(p, shape, ix->smem_optin, why, why_len);
    if (e == cudaSuccess || p0.nb == nullptr) return e;
    p0.nb = nullptr;
    p0.nb_stride = p0.nb_adj_bytes = p0.nb_pitch = 0;
    p = p0;
    shape = s0;
    return bsb::plan_search(p, shape, ix->smem_optin, why, why_len);
}

cudaError_t entry_kernels(const bs_index* ix, uint32_t* d_out, float* scratch, cudaStream_t stream) {
    return ix->u8 ? bsb::compute_entry_point_u8(ix->d_vecs8, ix->n, ix->dim, ix->row_bytes, d_out, scratch, stream)
                  : bsb::compute_entry_point(ix->d_vecs, ix->n, ix->dim, ix->row_stride, d_out, scratch, stream);
}

// Search parameters shared by bs_search and bs_search_no_alloc (everything
// but the output, query and scratch pointers).
void fill_params(const bs_index* ix, const ModeInfo& mi, const bs_search_params* prm, uint32_t entry,
                 SearchParams& p, LaunchShape& shape) {
    p = SearchParams{};
    p.sm_count = static_cast<uint32_t>(ix->num_sms);
    p.vecs = ix->d_vecs;
    p.vecs8 = ix->d_vecs8;
    p.row_bytes = ix->row_bytes;
    p.adj = ix->d_adj;
    p.n = ix->n;
    p.dim = static_cast<uint32_t>(ix->dim);
    p.row_stride = ix->row_stride;
    p.degree = static_cast<uint32_t>(ix->degree);
    if (!mi.rabitq && ix->d_nb) {
        p.nb = ix->d_nb;
        p.nb_stride = ix->nb_stride;
        p.nb_adj_bytes = ix->nb_adj_bytes;
        p.nb_pitch = ix->nb_pitch;
    }
    if (mi.rabitq) {
        p.codes = ix->d_codes;
        p.factors = ix->d_factors;
        p.signs = ix->d_signs;
        p.pdim = static_cast<uint32_t>(ix->pdim);
        p.wpp = static_cast<uint32_t>(ix->pdim) / 32u;
        if (ix->d_rqb) {
            p.rq_nb = ix->d_rqb;
            p.rq_stride = ix->rq_stride;
            p.rq_off_codes = ix->rq_off_codes;
            p.rq_off_fac = ix->rq_off_fac;
            p.rq_off_row = ix->rq_off_row;
            // BSEARCH_RQ_ESTIMATOR=lut: the nibble-table estimator (same sums)
            const char* est = std::getenv("BSEARCH_RQ_ESTIMATOR");
            p.rq_lut = (est && std::strcmp(est, "lut") == 0) ? 1u : 0u;
        }
    }
    p.topk = prm->topk_size;
    p.K = static_cast<uint32_t>(prm->K);
    p.entry = entry;
    p.max_iterations = prm->max_iterations;
    p.filter_slots = prm->filter_capacity;
    p.reset_interval = prm->reset_interval;
    team_range_for(ix, p.team_qlo, p.team_qhi);
    if (ix->u8) {   // byte kernels need query bytes too
        p.team_qlo = std::max(p.team_qlo, 0.0f);
        p.team_qhi = std::min(p.team_qhi, 255.0f);
    }
    if (force_seq()) { p.team_qlo = 1.0f; p.team_qhi = 0.0f; }
    p.sticky_err = ix->d_err;
    p.wait_polls = bsb::kDefaultWaitPolls;
    if (const char* w = std::getenv("BSEARCH_WAIT_POLLS")) p.wait_polls = static_cast<uint32_t>(std::strtoul(w, nullptr, 10));
    shape = LaunchShape{};
    if (ix->u8) shape.dmode = bsb::kU8;
    else shape.dmode = p.team_qlo <= p.team_qhi ? bsb::kTeam : bsb::kSeq;
    shape.fmode = mi.fmode;
    shape.warps_per_block = mi.warps;
    shape.block_query = mi.block ? 1 : 0;
}

void free_index(bs_index* ix) {
    if (!ix) return;
    DeviceGuard g(ix->device);
    cudaFree(ix->d_vecs);
    cudaFree(ix->d_vecs8);
    cudaFree(ix->d_adj);
    cudaFree(ix->d_nb);
    cudaFree(ix->d_codes);
    cudaFree(ix->d_factors);
    cudaFree(ix->d_signs);
    cudaFree(ix->d_err);
    cudaFree(ix->d_rqb);
    cudaFree(ix->d_vis);
    if (ix->rq_event) cudaEventDestroy(ix->rq_event);
    delete ix;
}

// A file mapped read-only into the address space (the loaders stream it to
// the device in chunks; the kernel pages it in as the chunks are copied).
struct MappedFile {
    int fd = -1;
    const unsigned char* p = nullptr;
    size_t size = 0;
    ~MappedFile() {
        if (p && size) munmap(const_cast<unsigned char*>(p), size);
        if (fd >= 0) close(fd);
    }
    bool open_ro(const char* path) {
        fd = ::open(path, O_RDONLY);
        if (fd < 0) return false;
        struct stat st;
        if (fstat(fd, &st) != 0) return false;
        size = static_cast<size_t>(st.st_size);
        if (size == 0) return true;
        void* m = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
        if (m == MAP_FAILED) { size = 0; return false; }
        madvise(m, size, MADV_SEQUENTIAL);
        p = static_cast<const unsigned char*>(m);
        return true;
    }
};

// Streams `rows` rows of `in_row` bytes from host memory to the device in
// chunks of about 64 MB through two page-locked buffers: while the GPU copies
// and takes apart chunk c, the host reads chunk c + 1 from the mapping.  Each
// chunk lands either at direct + first_row * in_row (a plain copy), or in a
// device staging buffer handed to consume(chunk, first_row, rows, stream).
template <class F>
cudaError_t pipeline_rows(const unsigned char* src, uint64_t rows, uint64_t in_row, unsigned char* direct, F&& consume) {
    if (rows == 0) return cudaSuccess;
    const uint64_t per = std::max<uint64_t>(1, (64ull << 20) / in_row);
    const uint64_t chunk = per * in_row;
    void* pin[2] = {nullptr, nullptr};
    void* dev[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    cudaStream_t st = nullptr;
    cudaError_t e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
    for (int b = 0; b < 2 && e == cudaSuccess; ++b) {
        e = cudaHostAlloc(&pin[b], chunk, cudaHostAllocDefault);
        if (e == cudaSuccess && !direct) e = cudaMalloc(&dev[b], chunk);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ev[b], cudaEventDisableTiming);
    }
    for (uint64_t r0 = 0, c = 0; e == cudaSuccess && r0 < rows; r0 += per, ++c) {
        const int b = static_cast<int>(c & 1u);
        const uint64_t cnt = std::min(per, rows - r0);
        if ((e = cudaEventSynchronize(ev[b])) != cudaSuccess) break;   // buffer b free again
        std::memcpy(pin[b], src + r0 * in_row, cnt * in_row);
        unsigned char* dst = direct ? direct + r0 * in_row : static_cast<unsigned char*>(dev[b]);
        e = cudaMemcpyAsync(dst, pin[b], cnt * in_row, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess && !direct) e = consume(static_cast<const uint32_t*>(dev[b]), r0, cnt, st);
        if (e == cudaSuccess) e = cudaEventRecord(ev[b], st);
    }
    if (st) {
        const cudaError_t s2 = cudaStreamSynchronize(st);
        if (e == cudaSuccess) e = s2;
        cudaStreamDestroy(st);
    }
    for (int b = 0; b < 2; ++b) {
        if (pin[b]) cudaFreeHost(pin[b]);
        if (dev[b]) cudaFree(dev[b]);
        if (ev[b]) cudaEventDestroy(ev[b]);
    }
    return e;
}

float ord_to_float(uint32_t o) {
    const uint32_t u = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// The index object with its device, dimensions, error word and an
// adjacency array (not filled); the rows are the caller's to upload.
bs_status create_index_shell(const bs_graph_desc* desc, int device, bs_index** out) {
    *out = nullptr;
    if (desc->num_nodes == 0 || desc->dim <= 0 || desc->degree <= 0)
        return fail(BS_ERR_INVALID_ARGUMENT, "num_nodes, dim and degree must be positive");
    if (desc->num_nodes >= (1ull << 31))
        return fail(BS_ERR_UNSUPPORTED, "num_nodes must be below 2^31 (node ids are 31-bit)");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return fail(BS_ERR_CUDA, "no CUDA device available");
    }
    if (device < 0 || device >= ndev) return fail(BS_ERR_INVALID_ARGUMENT, "device %d out of range", device);
    DeviceGuard g(device);
    if (!g.ok) return fail(BS_ERR_CUDA, "cannot select device %d", device);
    auto* ix = new (std::nothrow) bs_index();
    if (!ix) return fail(BS_ERR_OUT_OF_MEMORY, "host allocation failed");
    ix->device = device;
    {
        const char* env = std::getenv("BSEARCH_LAYOUT");
        ix->gather_only = env && std::strcmp(env, "gather") == 0;
    }
    ix->n = desc->num_nodes;
    ix->dim = desc->dim;
    ix->degree = desc->degree;
    ix->row_stride = (static_cast<uint32_t>(desc->dim) + 3u) & ~3u;
    ix->row_bytes = (static_cast<uint32_t>(desc->dim) + 15u) & ~15u;
    cudaDeviceProp prop;
    cudaError_t e = cudaGetDeviceProperties(&prop, device);
    if (e != cudaSuccess) { free_index(ix); return cuda_fail(e, "cudaGetDeviceProperties"); }
    ix->num_sms = prop.multiProcessorCount;
    ix->smem_optin = prop.sharedMemPerBlockOptin;
    const size_t ebytes = static_cast<size_t>(ix->n) * ix->degree * sizeof(uint32_t);
    if ((e = cudaMalloc(&ix->d_err, 256)) != cudaSuccess || (e = cudaMemset(ix->d_err, 0, 256)) != cudaSuccess) {
        free_index(ix);
        return cuda_fail(e, "error word");
    }
    if ((e = cudaMalloc(&ix->d_adj, ebytes)) != cudaSuccess) { free_index(ix); return cuda_fail(e, "adjacency"); }
    // Per-call scratch comes from the device's stream-ordered pool: keep freed
    // blocks cached instead of returning them at every synchronisation.
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
        uint64_t keep = UINT64_MAX;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    }
    cudaGetLastError();
    *out = ix;
    return BS_OK;
}

bs_status ensure_entry(bs_index* ix) {
    std::lock_guard<std::mutex> lk(ix->mu);
    if (ix->entry_valid) return BS_OK;
    const size_t bytes = bsb::entry_point_scratch_bytes(ix->n, ix->dim) + 8;
    void* scratch = nullptr;
    cudaError_t e = cudaMalloc(&scratch, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "entry point scratch");
    uint32_t* d_out = reinterpret_cast<uint32_t*>(static_cast<char*>(scratch) + bytes - 8);
    e = entry_kernels(ix, d_out, static_cast<float*>(scratch), nullptr);
    uint32_t h = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&h, d_out, 4, cudaMemcpyDeviceToHost);
    cudaFree(scratch);
    if (e != cudaSuccess) return cuda_fail(e, "entry point kernel");
    ix->entry = h;
    ix->entry_valid = true;
    return BS_OK;
}

}  // namespace

extern "C" {

BS_API void bs_search_params_default(bs_search_params* p) {
    if (!p) return;
    p->mode = "base";
    p->K = 100;
    p->topk_size = 256;
    p->filter_capacity = 1024;
    p->max_iterations = 1024;
    p->reset_interval = 16;
    p->entry_point = BS_NO_NODE;
}

BS_API const char* bs_last_error(void) { return g_err.c_str(); }

BS_API const char* bs_version(void) { return "beam_search_collab_b200 0.1 (sm_100a)"; }

BS_API bs_status bs_index_create(const bs_graph_desc* desc, int device, bs_index** out) {
    if (!out) return fail(BS_ERR_INVALID_ARGUMENT, "out is NULL");
    *out = nullptr;
    if (!desc || !desc->vectors) return fail(BS_ERR_INVALID_ARGUMENT, "graph descriptor or its vectors are NULL");
    bs_index* ix = nullptr;
    bs_status s = create_index_shell(desc, device, &ix);
    if (s != BS_OK) return s;
    DeviceGuard g(device);
    std::vector<uint64_t> neg_zeros;
    const uint64_t nvals = static_cast<uint64_t>(ix->n) * ix->dim;
    scan_values(desc->vectors, nvals, ix->int_exact, neg_zeros, ix->min_val, ix->max_val);
    // Exact byte copy when every value is an integer in [0,255] (SIFT-like
    // data): a quarter of the HBM bytes per gathered row, integer distances.
    // byte rows lose the sign of -0.0 (no distance depends on it, but the
    // rows a written codebook carries must come back bit for bit): their flat
    // positions are kept on the host, as long as they are few
    ix->u8 = ix->int_exact && ix->min_val >= 0.0f && ix->max_val <= 255.0f && !storage_f32_forced() &&
             neg_zeros.size() <= nvals / 64;
    if (ix->u8) ix->neg_zeros.swap(neg_zeros);
    const size_t ebytes = static_cast<size_t>(ix->n) * ix->degree * sizeof(uint32_t);
    cudaError_t e = cudaSuccess;
    if (ix->u8) {
        const size_t vbytes = static_cast<size_t>(ix->n) * ix->row_bytes;
        std::vector<uint8_t> packed;
        try {
            packed.assign(vbytes, 0);
        } catch (...) {
            free_index(ix);
            return fail(BS_ERR_OUT_OF_MEMORY, "host staging for the byte copy");
        }
        pack_u8_rows(desc->vectors, ix->n, ix->dim, ix->row_bytes, packed.data());
        if ((e = cudaMalloc(&ix->d_vecs8, vbytes)) != cudaSuccess) { free_index(ix); return cuda_fail(e, "vectors"); }
        e = cudaMemcpy(ix->d_vecs8, packed.data(), vbytes, cudaMemcpyHostToDevice);
    } else {
        const size_t vbytes = static_cast<size_t>(ix->n) * ix->row_stride * sizeof(float);
        if ((e = cudaMalloc(&ix->d_vecs, vbytes)) != cudaSuccess) { free_index(ix); return cuda_fail(e, "vectors"); }
        if (ix->row_stride == static_cast<uint32_t>(ix->dim)) {
            e = cudaMemcpy(ix->d_vecs, desc->vectors, vbytes, cudaMemcpyHostToDevice);
        } else {
            e = cudaMemset(ix->d_vecs, 0, vbytes);
            if (e == cudaSuccess)
                e = cudaMemcpy2D(ix->d_vecs, ix->row_stride * sizeof(float), desc->vectors,
                                 ix->dim * sizeof(float), ix->dim * sizeof(float), ix->n,
                                 cudaMemcpyHostToDevice);
        }
    }
    // no edges: an empty graph (node 0 in every slot, as build_graph pads)
    // for bs_index_build_graph to fill
    if (e == cudaSuccess)
        e = desc->edges ? cudaMemcpy(ix->d_adj, desc->edges, ebytes, cudaMemcpyHostToDevice) : cudaMemset(ix->d_adj, 0, ebytes);
    if (e != cudaSuccess) { free_index(ix); return cuda_fail(e, "index upload"); }
    *out = ix;
    return BS_OK;
}

BS_API bs_status bs_index_load(const char* graph_bin, const char* base_fvecs, int device, bs_index** out) {
    if (!out) return fail(BS_ERR_INVALID_ARGUMENT, "out is NULL");
    *out = nullptr;
    if (!graph_bin || !base_fvecs) return fail(BS_ERR_INVALID_ARGUMENT, "file path is NULL");
    // both files checked before any device work (include/cpu_graph.hpp:125-173,
    // include/data_loader.hpp:9-26 lay them out)
    MappedFile gf, bf;
    if (!gf.open_ro(graph_bin)) return fail(BS_ERR_IO, "Cannot open graph file: %s", graph_bin);
    if (gf.size < 8) return fail(BS_ERR_IO, "Cannot read graph header: %s", graph_bin);
    int32_t hdr[2];
    std::memcpy(hdr, gf.p, 8);
    if (hdr[0] <= 0 || hdr[1] <= 0) return fail(BS_ERR_IO, "Invalid graph header in: %s", graph_bin);
    const uint64_t n = static_cast<uint64_t>(hdr[0]);
    const int32_t deg = hdr[1];
    if (gf.size < 8 + n * static_cast<uint64_t>(deg) * 4) return fail(BS_ERR_IO, "Truncated graph file: %s", graph_bin);
    if (!bf.open_ro(base_fvecs)) return fail(BS_ERR_IO, "Cannot open %s", base_fvecs);
    if (bf.size < 4) return fail(BS_ERR_IO, "Invalid vecs header in: %s", base_fvecs);
    int32_t dim = 0;
    std::memcpy(&dim, bf.p, 4);
    if (dim <= 0) return fail(BS_ERR_IO, "Invalid vecs header in: %s", base_fvecs);
    const uint64_t in_row = 4ull * (static_cast<uint64_t>(dim) + 1);
    if (bf.size % in_row != 0) return fail(BS_ERR_IO, "Corrupt vecs file (size not a multiple of the row): %s", base_fvecs);
    const uint64_t nv = bf.size / in_row;
    if (nv != n)
        return fail(BS_ERR_IO, "graph has %llu nodes but %s has %llu vectors", static_cast<unsigned long long>(n),
                    base_fvecs, static_cast<unsigned long long>(nv));
    // the index's arrays, allocated empty, then filled from the mapped files
    bs_graph_desc d{n, dim, deg, nullptr, nullptr};
    bs_index* ix = nullptr;
    bs_status s = create_index_shell(&d, device, &ix);
    if (s != BS_OK) return s;
    DeviceGuard g(device);
    const uint64_t nvals = n * static_cast<uint64_t>(dim);
    const size_t fbytes = static_cast<size_t>(n) * ix->row_stride * 4;
    bsb::LoadScan h{};
    h.all_int = 1;
    h.min_ord = 0xffffffffu;
    h.neg_zero_cap = nvals / 64 + 1;
    bsb::LoadScan* d_scan = nullptr;
    cudaError_t e = cudaMalloc(&ix->d_vecs, fbytes);
    if (e == cudaSuccess) e = cudaMalloc(&d_scan, sizeof(bsb::LoadScan) + h.neg_zero_cap * 8);
    if (e == cudaSuccess) {
        h.neg_zero_pos = reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(d_scan) + sizeof(bsb::LoadScan));
        e = cudaMemcpy(d_scan, &h, sizeof(h), cudaMemcpyHostToDevice);
    }
    // graph payload as it is; base rows taken apart and scanned on the GPU
    if (e == cudaSuccess)
        e = pipeline_rows(gf.p + 8, n, static_cast<uint64_t>(deg) * 4, reinterpret_cast<unsigned char*>(ix->d_adj),
                          [](const uint32_t*, uint64_t, uint64_t, cudaStream_t) { return cudaSuccess; });
    const uint32_t row_stride = ix->row_stride;
    float* d_vecs = ix->d_vecs;
    if (e == cudaSuccess)
        e = pipeline_rows(bf.p, n, in_row, nullptr, [&](const uint32_t* raw, uint64_t r0, uint64_t cnt, cudaStream_t st) {
            return bsb::load_fvecs_chunk(raw, cnt, r0, static_cast<uint32_t>(dim), row_stride, d_vecs, d_scan, st);
        });
    if (e == cudaSuccess) e = cudaMemcpy(&h, d_scan, sizeof(h), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) { cudaFree(d_scan); free_index(ix); return cuda_fail(e, "index upload"); }
    if (h.bad_rows) { cudaFree(d_scan); free_index(ix); return fail(BS_ERR_IO, "Inconsistent row dimension in: %s", base_fvecs); }
    ix->int_exact = h.all_int != 0;
    ix->min_val = h.min_ord == 0xffffffffu ? 0.0f : ord_to_float(h.min_ord);
    ix->max_val = h.max_ord == 0u ? 0.0f : ord_to_float(h.max_ord);
    ix->u8 = ix->int_exact && ix->min_val >= 0.0f && ix->max_val <= 255.0f && !storage_f32_forced() &&
             h.neg_zero_count <= nvals / 64;
    if (ix->u8) {
        // the exact byte copy replaces the f32 rows; the -0.0 positions are
        // kept (ascending) for a codebook written from this index
        ix->neg_zeros.resize(h.neg_zero_count);
        if (h.neg_zero_count)
            e = cudaMemcpy(ix->neg_zeros.data(), h.neg_zero_pos, h.neg_zero_count * 8, cudaMemcpyDeviceToHost);
        std::sort(ix->neg_zeros.begin(), ix->neg_zeros.end());
        if (e == cudaSuccess) e = cudaMalloc(&ix->d_vecs8, static_cast<size_t>(n) * ix->row_bytes);
        if (e == cudaSuccess) e = bsb::rows_to_u8(ix->d_vecs, n, dim, ix->row_stride, ix->row_bytes, ix->d_vecs8, nullptr);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        cudaFree(ix->d_vecs);
        ix->d_vecs = nullptr;
    }
    cudaFree(d_scan);
    if (e != cudaSuccess) { free_index(ix); return cuda_fail(e, "index upload"); }
    *out = ix;
    return BS_OK;
}

BS_API bs_status bs_index_attach_rabitq(bs_index* ix, const bs_rabitq_desc* d) {
    if (!ix || !d || !d->codes || !d->factors || !d->signs)
        return fail(BS_ERR_INVALID_ARGUMENT, "index or RaBitQ arrays are NULL");
    const int32_t pdim = bsb::io::padded_dim_of(ix->dim);
    if (d->padded_dim != pdim)
        return fail(BS_ERR_INVALID_ARGUMENT, "padded_dim %d does not match dim %d (expected %d)", d->padded_dim,
                    ix->dim, pdim);
    if (pdim < 32) return fail(BS_ERR_UNSUPPORTED, "RaBitQ needs dim > 16 (padded_dim >= 32)");
    if (d->entry_point != BS_NO_NODE && d->entry_point >= ix->n)
        return fail(BS_ERR_INVALID_ARGUMENT, "codebook entry point %u out of range", d->entry_point);
    DeviceGuard g(ix->device);
    const size_t wpp = static_cast<size_t>(pdim) / 32;
    const size_t cbytes = static_cast<size_t>(ix->n) * ix->degree * wpp * 4;
    const size_t fbytes = static_cast<size_t>(ix->n) * 3 * ix->degree * 4;
    cudaFree(ix->d_codes);
    cudaFree(ix->d_factors);
    cudaFree(ix->d_signs);
    ix->d_codes = nullptr; ix->d_factors = nullptr; ix->d_signs = nullptr;
    ix->has_rabitq = false;
    cudaError_t e;
    if ((e = cudaMalloc(&ix->d_codes, cbytes)) != cudaSuccess) return cuda_fail(e, "codes");
    if ((e = cudaMalloc(&ix->d_factors, fbytes)) != cudaSuccess) return cuda_fail(e, "factors");
    if ((e = cudaMalloc(&ix->d_signs, pdim * 4)) != cudaSuccess) return cuda_fail(e, "signs");
    if ((e = cudaMemcpy(ix->d_codes, d->codes, cbytes, cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemcpy(ix->d_factors, d->factors, fbytes, cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemcpy(ix->d_signs, d->signs, pdim * 4, cudaMemcpyHostToDevice)) != cudaSuccess)
        return cuda_fail(e, "codebook upload");
    ix->pdim = pdim;
    ix->rq_entry = d->entry_point;
    ix->has_rabitq = true;
    if ((e = build_rq_blocks(ix)) != cudaSuccess) return cuda_fail(e, "rabitq node blocks");
    return BS_OK;
}

BS_API bs_status bs_index_load_codebook(bs_index* ix, const char* path) {
    if (!ix || !path) return fail(BS_ERR_INVALID_ARGUMENT, "index or path is NULL");
    // codebook.bin (include/rabitq.hpp:49-97): u32 entry, n rows of
    // [raw vector (dim) | codes (wpp*deg) | factors (3*deg) | neighbour ids
    // (deg)] 4-byte slots, f32 signs[padded_dim]; the rows are streamed to the
    // device and taken apart there
    MappedFile f;
    if (!f.open_ro(path)) return fail(BS_ERR_IO, "Cannot open codebook: %s", path);
    const int32_t pdim = bsb::io::padded_dim_of(ix->dim);
    if (pdim < 32) return fail(BS_ERR_UNSUPPORTED, "RaBitQ needs dim > 16 (padded_dim >= 32)");
    const uint64_t wpp = static_cast<uint64_t>(pdim) / 32, deg = static_cast<uint64_t>(ix->degree);
    const uint64_t row = static_cast<uint64_t>(ix->dim) + wpp * deg + 4 * deg;
    if (f.size < 4 + ix->n * row * 4 + static_cast<uint64_t>(pdim) * 4)
        return fail(BS_ERR_IO, "Truncated codebook (or dim/degree mismatch): %s", path);
    uint32_t entry = 0;
    std::memcpy(&entry, f.p, 4);
    if (entry != BS_NO_NODE && entry >= ix->n)
        return fail(BS_ERR_INVALID_ARGUMENT, "codebook entry point %u out of range", entry);
    DeviceGuard g(ix->device);
    cudaFree(ix->d_codes);
    cudaFree(ix->d_factors);
    cudaFree(ix->d_signs);
    ix->d_codes = nullptr; ix->d_factors = nullptr; ix->d_signs = nullptr;
    ix->has_rabitq = false;
    cudaError_t e;
    if ((e = cudaMalloc(&ix->d_codes, ix->n * deg * wpp * 4)) != cudaSuccess) return cuda_fail(e, "codes");
    if ((e = cudaMalloc(&ix->d_factors, ix->n * 3 * deg * 4)) != cudaSuccess) return cuda_fail(e, "factors");
    if ((e = cudaMalloc(&ix->d_signs, static_cast<size_t>(pdim) * 4)) != cudaSuccess) return cuda_fail(e, "signs");
    uint32_t* codes = ix->d_codes;
    float* factors = ix->d_factors;
    const uint32_t dim = static_cast<uint32_t>(ix->dim), dg = static_cast<uint32_t>(deg), w = static_cast<uint32_t>(wpp);
    e = pipeline_rows(f.p + 4, ix->n, row * 4, nullptr, [&](const uint32_t* raw, uint64_t r0, uint64_t cnt, cudaStream_t st) {
        return bsb::load_codebook_chunk(raw, cnt, r0, dim, dg, w, codes, factors, st);
    });
    if (e == cudaSuccess)
        e = cudaMemcpy(ix->d_signs, f.p + 4 + ix->n * row * 4, static_cast<size_t>(pdim) * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "codebook upload");
    ix->pdim = pdim;
    ix->rq_entry = entry;
    ix->has_rabitq = true;
    if ((e = build_rq_blocks(ix)) != cudaSuccess) return cuda_fail(e, "rabitq node blocks");
    return BS_OK;
}

BS_API bs_status bs_index_build_codebook(bs_index* ix, uint32_t seed, const char* out_path, uint32_t* entry_out) {
    if (!ix) return fail(BS_ERR_INVALID_ARGUMENT, "index is NULL");
    const int32_t pdim = bsb::io::padded_dim_of(ix->dim);
    if (pdim < 32) return fail(BS_ERR_UNSUPPORTED, "RaBitQ needs dim > 16 (padded_dim >= 32)");
    if (ix->n > 0xffffffffull) return fail(BS_ERR_UNSUPPORTED, "more than 2^32 rows");
    // sign table: the reference's generator and distribution
    // (src/build_rabitq.cpp:138-146), from the same standard library
    std::vector<float> signs(static_cast<size_t>(pdim));
    {
        std::mt19937_64 gen(seed);
        std::uniform_int_distribution<int> coin(0, 1);
        const float scale = 1.0f / std::sqrt(static_cast<float>(pdim));
        for (int32_t i = 0; i < pdim; ++i) signs[static_cast<size_t>(i)] = static_cast<float>(2 * coin(gen) - 1) * scale;
    }
    DeviceGuard g(ix->device);
    if (!g.ok) return fail(BS_ERR_CUDA, "cannot select device %d", ix->device);
    const size_t wpp = static_cast<size_t>(pdim) / 32;
    const size_t deg = static_cast<size_t>(ix->degree);
    const size_t cbytes = static_cast<size_t>(ix->n) * deg * wpp * 4;
    const size_t fbytes = static_cast<size_t>(ix->n) * 3 * deg * 4;
    uint32_t* d_codes = nullptr;
    float* d_factors = nullptr;
    float* d_signs = nullptr;
    unsigned char* d_scratch = nullptr;
    uint32_t* d_stage = nullptr;
    std::FILE* f = nullptr;
    auto cleanup = [&]() {
        cudaFree(d_codes);
        cudaFree(d_factors);
        cudaFree(d_signs);
        cudaFree(d_scratch);
        cudaFree(d_stage);
        if (f) std::fclose(f);
    };
    cudaError_t e;
    if ((e = cudaMalloc(&d_codes, cbytes ? cbytes : 4)) != cudaSuccess ||
        (e = cudaMalloc(&d_factors, fbytes ? fbytes : 4)) != cudaSuccess ||
        (e = cudaMalloc(&d_signs, static_cast<size_t>(pdim) * 4)) != cudaSuccess ||
        (e = cudaMalloc(&d_scratch, bsb::medoid_scratch_bytes(static_cast<uint32_t>(ix->dim)) + 16)) != cudaSuccess) {
        cleanup();
        return cuda_fail(e, "codebook buffers");
    }
    if ((e = cudaMemcpy(d_signs, signs.data(), static_cast<size_t>(pdim) * 4, cudaMemcpyHostToDevice)) != cudaSuccess) {
        cleanup();
        return cuda_fail(e, "sign table upload");
    }
    bsb::CodebookArgs a{};
    a.vecs = ix->u8 ? nullptr : ix->d_vecs;
    a.vecs8 = ix->u8 ? ix->d_vecs8 : nullptr;
    a.row_stride = ix->u8 ? ix->row_bytes : ix->row_stride;
    a.adj = ix->d_adj;
    a.n = ix->n;
    a.dim = static_cast<uint32_t>(ix->dim);
    a.degree = static_cast<uint32_t>(ix->degree);
    a.pdim = static_cast<uint32_t>(pdim);
    a.signs = d_signs;
    a.codes = d_codes;
    a.factors = d_factors;
    uint32_t* d_entry = reinterpret_cast<uint32_t*>(d_scratch + bsb::medoid_scratch_bytes(a.dim));
    uint32_t entry = BS_NO_NODE;
    if ((e = bsb::compute_medoid(a, d_entry, d_scratch, 0)) != cudaSuccess ||
        (e = bsb::quantize_edges(a, ix->smem_optin, ix->num_sms, 0)) != cudaSuccess ||
        (e = cudaMemcpy(&entry, d_entry, 4, cudaMemcpyDeviceToHost)) != cudaSuccess) {
        cleanup();
        return cuda_fail(e, "codebook build");
    }
    if (out_path) {
        // codebook.bin (src/build_rabitq.cpp:268-285): u32 entry, n rows, signs
        f = std::fopen(out_path, "wb");
        if (!f) {
            cleanup();
            return fail(BS_ERR_IO, "Cannot open output file: %s", out_path);
        }
        const uint64_t row_slots = static_cast<uint64_t>(ix->dim) + wpp * deg + 4 * deg;
        const uint64_t chunk = std::max<uint64_t>(1, (256ull << 20) / (row_slots * 4));
        const uint64_t rows = std::min<uint64_t>(chunk, ix->n);
        std::vector<uint32_t> host(static_cast<size_t>(rows * row_slots));
        bool ok = std::fwrite(&entry, 4, 1, f) == 1;
        if (ok && rows && (e = cudaMalloc(&d_stage, rows * row_slots * 4)) != cudaSuccess) {
            cleanup();
            return cuda_fail(e, "codebook staging");
        }
        for (uint64_t r0 = 0; ok && r0 < ix->n; r0 += rows) {
            const uint64_t cnt = std::min<uint64_t>(rows, ix->n - r0);
            if ((e = bsb::pack_codebook_rows(a, r0, cnt, d_stage, ix->num_sms, 0)) != cudaSuccess ||
                (e = cudaMemcpy(host.data(), d_stage, cnt * row_slots * 4, cudaMemcpyDeviceToHost)) != cudaSuccess) {
                cleanup();
                return cuda_fail(e, "codebook rows");
            }
            // byte rows: put back the -0.0 values the byte copy dropped
            const uint64_t lo = r0 * static_cast<uint64_t>(ix->dim), hi = lo + cnt * static_cast<uint64_t>(ix->dim);
            for (auto it = std::lower_bound(ix->neg_zeros.begin(), ix->neg_zeros.end(), lo);
                 it != ix->neg_zeros.end() && *it < hi; ++it) {
                const uint64_t row = *it / static_cast<uint64_t>(ix->dim) - r0, d = *it % static_cast<uint64_t>(ix->dim);
                host[static_cast<size_t>(row * row_slots + d)] = 0x80000000u;
            }
            ok = std::fwrite(host.data(), 4, cnt * row_slots, f) == cnt * row_slots;
        }
        ok = ok && std::fwrite(signs.data(), 4, static_cast<size_t>(pdim), f) == static_cast<size_t>(pdim);
        ok = (std::fclose(f) == 0) && ok;
        f = nullptr;
        if (!ok) {
            cleanup();
            return fail(BS_ERR_IO, "Cannot write codebook: %s", out_path);
        }
    }
    cudaFree(d_stage);
    d_stage = nullptr;
    cudaFree(d_scratch);
    d_scratch = nullptr;
    // attach (replacing any previous codebook)
    cudaFree(ix->d_codes);
    cudaFree(ix->d_factors);
    cudaFree(ix->d_signs);
    ix->d_codes = d_codes;
    ix->d_factors = d_factors;
    ix->d_signs = d_signs;
    ix->pdim = pdim;
    ix->rq_entry = entry;
    ix->has_rabitq = true;
    if (entry_out) *entry_out = entry;
    if ((e = build_rq_blocks(ix)) != cudaSuccess) return cuda_fail(e, "rabitq node blocks");
    return BS_OK;
}

BS_API bs_status bs_index_info(const bs_index* ix, uint64_t* n, int32_t* dim, int32_t* degree) {
    if (!ix) return fail(BS_ERR_INVALID_ARGUMENT, "index is NULL");
    if (n) *n = ix->n;
    if (dim) *dim = ix->dim;
    if (degree) *degree = ix->degree;
    return BS_OK;
}

BS_API bs_status bs_index_entry_point(bs_index* ix, uint32_t* entry) {
    if (!ix || !entry) return fail(BS_ERR_INVALID_ARGUMENT, "index or entry is NULL");
    DeviceGuard g(ix->device);
    const bs_status s = ensure_entry(ix);
    if (s != BS_OK) return s;
    *entry = ix->entry;
    return BS_OK;
}

BS_API bs_status bs_index_rabitq_entry(const bs_index* ix, uint32_t* entry) {
    if (!ix || !entry) return fail(BS_ERR_INVALID_ARGUMENT, "index or entry is NULL");
    *entry = ix->has_rabitq ? ix->rq_entry : BS_NO_NODE;
    return BS_OK;
}

BS_API bs_status bs_index_build_graph(bs_index* ix, const bs_graph_build_params* prm, uint32_t* edges_out) {
    if (!ix || !prm) return fail(BS_ERR_INVALID_ARGUMENT, "index or params is NULL");
    if (ix->degree > 64) return fail(BS_ERR_UNSUPPORTED, "the graph builder supports degree <= 64");
    if (prm->beam_width <= 0 || prm->beam_width > 512)
        return fail(BS_ERR_UNSUPPORTED, "beam_width must be in 1..512");
    if (!(prm->alpha >= 1.0f)) return fail(BS_ERR_INVALID_ARGUMENT, "--alpha must be at least 1.0");
    DeviceGuard g(ix->device);
    if (!g.ok) return fail(BS_ERR_CUDA, "cannot select device %d", ix->device);
    const uint64_t n = ix->n;
    const uint32_t deg = static_cast<uint32_t>(ix->degree);
    // insertion order: the reference's generator and shuffle
    // (src/build_graph.cpp:298-301), from the same standard library
    std::vector<uint32_t> order(n);
    for (uint64_t i = 0; i < n; ++i) order[i] = static_cast<uint32_t>(i);
    {
        std::mt19937 gen(prm->seed);
        std::shuffle(order.begin(), order.end(), gen);
    }
    bsb::GraphBuildArgs a{};
    {
        ModeInfo mi{false, bsb::kHash, 4};
        bs_search_params sp0;
        bs_search_params_default(&sp0);
        LaunchShape shape;
        fill_params(ix, mi, &sp0, 0, a.sp, shape);
        a.sp.nb = nullptr;
    }
    a.degree = deg;
    a.L = static_cast<uint32_t>(prm->beam_width);
    a.alpha = prm->alpha;
    if (bsb::plan_graph_build(a, ix->smem_optin) != cudaSuccess)
        return fail(BS_ERR_UNSUPPORTED, "rows of %d dimensions do not fit the graph builder's shared memory", ix->dim);
    const uint64_t bound = std::max<uint64_t>(1, static_cast<uint64_t>(0.02 * static_cast<double>(n)));
    const uint64_t batch_max = std::max<uint64_t>(1, std::min<uint64_t>(bound, n > 1 ? n - 1 : 1));
    constexpr uint32_t kPoolCap = 2048, kLogCap = 8192, kOvfCap = 65536;
    uint32_t cap_warps = bsb::graph_build_search_warps(a, ix->num_sms, ix->smem_optin);
    if (cap_warps == 0) return fail(BS_ERR_UNSUPPORTED, "graph builder launch shape");
    const uint32_t words = static_cast<uint32_t>(((n + 31u) / 32u + 3u) & ~3ull);
    const uint64_t per_warp = (static_cast<uint64_t>(words) + kLogCap) * 4u;
    size_t free_b = 0, total_b = 0;
    cudaError_t e = cudaMemGetInfo(&free_b, &total_b);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemGetInfo");
    uint64_t vis_warps = std::min<uint64_t>({cap_warps, (batch_max + 3) / 4 * 4, (free_b / 4u) / per_warp});
    vis_warps -= vis_warps % 4;
    if (vis_warps < 4) return fail(BS_ERR_OUT_OF_MEMORY, "graph builder visited sets do not fit");
    const uint64_t items = batch_max * deg;
    const size_t sort_bytes = bsb::graph_build_sort_bytes(items);
    void* d_order = nullptr; void* d_dist = nullptr; void* d_cnt = nullptr; void* d_pool = nullptr;
    void* d_pcnt = nullptr; void* d_vis = nullptr; void* d_rev = nullptr; void* d_sort = nullptr;
    void* d_misc = nullptr;
    auto cleanup = [&]() {
        for (void* q : {d_order, d_dist, d_cnt, d_pool, d_pcnt, d_vis, d_rev, d_sort, d_misc}) cudaFree(q);
    };
    if ((e = cudaMalloc(&d_order, n * 4)) != cudaSuccess || (e = cudaMalloc(&d_dist, n * deg * 4)) != cudaSuccess ||
        (e = cudaMalloc(&d_cnt, n * 4)) != cudaSuccess || (e = cudaMalloc(&d_pool, batch_max * kPoolCap * 8)) != cudaSuccess ||
        (e = cudaMalloc(&d_pcnt, batch_max * 4)) != cudaSuccess || (e = cudaMalloc(&d_vis, vis_warps * per_warp)) != cudaSuccess ||
        (e = cudaMalloc(&d_rev, items * 4 * 5)) != cudaSuccess || (e = cudaMalloc(&d_sort, sort_bytes + 16)) != cudaSuccess ||
        (e = cudaMalloc(&d_misc, 256 + 4 * kOvfCap)) != cudaSuccess) {
        cleanup();
        return cuda_fail(e, "graph builder buffers");
    }
    if ((e = cudaMemcpy(d_order, order.data(), n * 4, cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemset(d_cnt, 0, n * 4)) != cudaSuccess || (e = cudaMemset(d_vis, 0, vis_warps * per_warp)) != cudaSuccess ||
        (e = cudaMemset(d_misc, 0, 256 + 4 * kOvfCap)) != cudaSuccess) {
        cleanup();
        return cuda_fail(e, "graph builder set-up");
    }
    a.order = static_cast<const uint32_t*>(d_order);
    a.nbr_ids = ix->d_adj;
    a.nbr_dist = static_cast<float*>(d_dist);
    a.nbr_cnt = static_cast<uint32_t*>(d_cnt);
    a.pool = static_cast<unsigned long long*>(d_pool);
    a.pool_cnt = static_cast<uint32_t*>(d_pcnt);
    a.pool_cap = kPoolCap;
    a.vis = static_cast<uint32_t*>(d_vis);
    a.vis_words = words;
    a.vis_log_cap = kLogCap;
    a.vis_warps = static_cast<uint32_t>(vis_warps);
    uint32_t* rev = static_cast<uint32_t*>(d_rev);
    a.seg_start = rev + 4 * items;
    a.seg_count = static_cast<uint32_t*>(d_misc);
    a.err = static_cast<unsigned int*>(d_misc) + 4;
    a.ovf_count = static_cast<uint32_t*>(d_misc) + 8;
    a.ovf_jobs = static_cast<uint32_t*>(d_misc) + 64;
    a.ovf_cap = kOvfCap;
    a.ovf_pass = 0;
    // The first reverse-prune launch holds 512 candidates per prune (a node's
    // list plus the reverse edges one batch gives it: rarely more), so that
    // many prunes share an SM; larger ones run in the second launch.
    // BSEARCH_GB_REV_PRUNE_CAP (a power of two, 64..4096) sets it (tests use
    // a small one to reach the second launch on small graphs).
    a.rev_prune_cap = 512;
    if (const char* c = std::getenv("BSEARCH_GB_REV_PRUNE_CAP")) {
        const uint32_t v = static_cast<uint32_t>(std::strtoul(c, nullptr, 10));
        if (v >= 64 && v <= 4096 && (v & (v - 1)) == 0) a.rev_prune_cap = v;
    }
    // the batch loop (src/build_graph.cpp:303-369)
    for (uint64_t start = 1; start < n;) {
        const uint64_t end = std::min(std::min(start * 2, start + bound), n);
        a.start = start;
        a.count = end - start;
        e = bsb::graph_build_batch(a, ix->smem_optin, ix->num_sms, d_sort, sort_bytes, rev, rev + items,
                                   rev + 2 * items, rev + 3 * items, nullptr);
        if (e != cudaSuccess) { cleanup(); return cuda_fail(e, "graph build batch"); }
        start = end;
    }
    e = bsb::graph_build_finish(a, ix->smem_optin, ix->num_sms, nullptr);
    unsigned int err = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&err, a.err, 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) { cleanup(); return cuda_fail(e, "graph build"); }
    if (err) {
        cleanup();
        return fail(BS_ERR_KERNEL, "graph builder: %s (flags 0x%x)",
                    (err & bsb::kErrPoolFull) ? "a build search expanded more than 2048 nodes"
                                              : "a prune had more than 16384 candidates", err);
    }
    // missing slots are node 0 (src/build_graph.cpp:371): the tails past each count
    {
        std::vector<uint32_t> cnt(n);
        if ((e = cudaMemcpy(cnt.data(), d_cnt, n * 4, cudaMemcpyDeviceToHost)) != cudaSuccess) { cleanup(); return cuda_fail(e, "graph counts"); }
        std::vector<uint32_t> edges(n * deg);
        if ((e = cudaMemcpy(edges.data(), ix->d_adj, n * deg * 4, cudaMemcpyDeviceToHost)) != cudaSuccess) { cleanup(); return cuda_fail(e, "graph edges"); }
        for (uint64_t u = 0; u < n; ++u)
            for (uint32_t j = cnt[u]; j < deg; ++j) edges[u * deg + j] = 0;
        if ((e = cudaMemcpy(ix->d_adj, edges.data(), n * deg * 4, cudaMemcpyHostToDevice)) != cudaSuccess) { cleanup(); return cuda_fail(e, "graph edges"); }
        if (edges_out) std::memcpy(edges_out, edges.data(), n * deg * 4);
    }
    cleanup();
    // the layouts and the codebook that depended on the old graph
    {
        std::lock_guard<std::mutex> lk(ix->mu);
        cudaFree(ix->d_nb);
        ix->d_nb = nullptr;
        ix->nb_tried = false;
    }
    cudaFree(ix->d_codes); cudaFree(ix->d_factors); cudaFree(ix->d_signs); cudaFree(ix->d_rqb);
    ix->d_codes = nullptr; ix->d_factors = nullptr; ix->d_signs = nullptr; ix->d_rqb = nullptr;
    ix->has_rabitq = false;
    ix->rq_entry = BS_NO_NODE;
    return BS_OK;
}

BS_API bs_status bs_ground_truth(bs_index* ix, const float* queries, uint32_t nq, uint32_t k, uint32_t* ids,
                                 float* dists, void* stream_) {
    if (!ix) return fail(BS_ERR_INVALID_ARGUMENT, "index is NULL");
    if (k == 0 || k > 256) return fail(BS_ERR_UNSUPPORTED, "k must be in 1..256");
    if (nq > 0 && (!queries || !ids)) return fail(BS_ERR_INVALID_ARGUMENT, "queries or ids is NULL");
    if (nq == 0) return BS_OK;
    DeviceGuard g(ix->device);
    if (!g.ok) return fail(BS_ERR_CUDA, "cannot select device %d", ix->device);
    if (any_foreign(ix->device, {queries, ids, dists}))
        return fail(BS_ERR_INVALID_ARGUMENT, "a buffer lives on another GPU than the index (device %d)", ix->device);
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    bsb::GroundTruthArgs a{};
    {
        ModeInfo mi{false, bsb::kHash, 4};
        bs_search_params sp0;
        bs_search_params_default(&sp0);
        LaunchShape shape;
        fill_params(ix, mi, &sp0, 0, a.sp, shape);
        a.sp.nb = nullptr;
    }
    a.nq = nq;
    a.k = k;
    if (bsb::plan_ground_truth(a, ix->smem_optin, ix->num_sms) != cudaSuccess)
        return fail(BS_ERR_UNSUPPORTED, "rows of %d dimensions do not fit the ground-truth kernel", ix->dim);
    const bool q_dev = is_device_ptr(queries, ix->device);
    const bool i_dev = is_device_ptr(ids, ix->device);
    const bool d_dev = dists ? is_device_ptr(dists, ix->device) : true;
    const size_t qbytes = static_cast<size_t>(nq) * ix->dim * 4, obytes = static_cast<size_t>(nq) * k * 4;
    const size_t pbytes = static_cast<size_t>(a.splits) * nq * k * 4;
    size_t off = 0;
    const size_t q_off = off;
    if (!q_dev) off += (qbytes + 255) & ~static_cast<size_t>(255);
    const size_t i_off = off;
    if (!i_dev) off += (obytes + 255) & ~static_cast<size_t>(255);
    const size_t d_off = off;
    if (dists && !d_dev) off += (obytes + 255) & ~static_cast<size_t>(255);
    const size_t pd_off = off;
    off += (pbytes + 255) & ~static_cast<size_t>(255);
    const size_t pi_off = off;
    off += (pbytes + 255) & ~static_cast<size_t>(255);
    char* scratch = nullptr;
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&scratch), off, stream);
    if (e != cudaSuccess) return cuda_fail(e, "ground-truth scratch");
    a.queries = q_dev ? queries : reinterpret_cast<const float*>(scratch + q_off);
    a.out_ids = i_dev ? ids : reinterpret_cast<uint32_t*>(scratch + i_off);
    a.out_dists = !dists ? nullptr : d_dev ? dists : reinterpret_cast<float*>(scratch + d_off);
    a.part_d = reinterpret_cast<float*>(scratch + pd_off);
    a.part_i = reinterpret_cast<uint32_t*>(scratch + pi_off);
    if (!q_dev) e = cudaMemcpyAsync(scratch + q_off, queries, qbytes, cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess) e = bsb::launch_ground_truth(a, ix->num_sms, stream);
    if (e == cudaSuccess && !i_dev) e = cudaMemcpyAsync(ids, scratch + i_off, obytes, cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess && dists && !d_dev)
        e = cudaMemcpyAsync(dists, scratch + d_off, obytes, cudaMemcpyDeviceToHost, stream);
    cudaFreeAsync(scratch, stream);
    if (e == cudaSuccess && (!q_dev || !i_dev || !d_dev)) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return cuda_fail(e, "ground truth");
    return BS_OK;
}

BS_API bs_status bs_index_prepare(bs_index* ix, const char* mode) {
    if (!ix) return fail(BS_ERR_INVALID_ARGUMENT, "index is NULL");
    ModeInfo mi;
    if (!parse_mode(mode, mi)) return fail(BS_ERR_INVALID_ARGUMENT, "Unknown mode: %s", mode ? mode : "(null)");
    DeviceGuard g(ix->device);
    if (!g.ok) return fail(BS_ERR_CUDA, "cannot select device %d", ix->device);
    if (mi.rabitq) {
        if (!ix->has_rabitq) return fail(BS_ERR_INVALID_ARGUMENT, "rabitq mode requires a codebook on the index");
        return BS_OK;
    }
    std::lock_guard<std::mutex> lk(ix->mu);
    return ensure_blocks(ix);
}

BS_API bs_status bs_index_take_errors(bs_index* ix, void* stream_, uint32_t* flags) {
    if (!ix || !flags) return fail(BS_ERR_INVALID_ARGUMENT, "index or flags is NULL");
    DeviceGuard g(ix->device);
    if (!g.ok) return fail(BS_ERR_CUDA, "cannot select device %d", ix->device);
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    unsigned int h = 0;
    cudaError_t e = cudaMemcpyAsync(&h, ix->d_err, sizeof(h), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(ix->d_err, 0, sizeof(h), stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return cuda_fail(e, "error word");
    *flags = h;
    return BS_OK;
}

BS_API void bs_index_destroy(bs_index* ix) { free_index(ix); }

BS_API bs_status bs_search(bs_index* ix, const bs_search_params* prm, const float* queries, uint32_t nq,
                           uint32_t* ids, float* dists, bs_stats* stats, void* stream_) {
    if (!ix || !prm) return fail(BS_ERR_INVALID_ARGUMENT, "index or params is NULL");
    ModeInfo mi;
    if (!parse_mode(prm->mode, mi)) return fail(BS_ERR_INVALID_ARGUMENT, "Unknown mode: %s", prm->mode ? prm->mode : "(null)");
    if (prm->K <= 0) return fail(BS_ERR_INVALID_ARGUMENT, "K must be positive");
    if (prm->topk_size == 0) return fail(BS_ERR_INVALID_ARGUMENT, "topk_size must be positive");
    if (prm->max_iterations < 0) return fail(BS_ERR_INVALID_ARGUMENT, "max_iterations must be >= 0");
    if (mi.rabitq && !ix->has_rabitq) return fail(BS_ERR_INVALID_ARGUMENT, "rabitq mode requires a codebook on the index");
    if (nq > 0 && (!queries || !ids)) return fail(BS_ERR_INVALID_ARGUMENT, "queries or ids is NULL");

    DeviceGuard g(ix->device);
    if (!g.ok) return fail(BS_ERR_CUDA, "cannot select device %d", ix->device);
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);

    uint32_t entry = prm->entry_point;
    if (entry == BS_NO_NODE) {
        if (mi.rabitq && ix->rq_entry != BS_NO_NODE) {
            entry = ix->rq_entry;
        } else {
            const bs_status s = ensure_entry(ix);
            if (s != BS_OK) return s;
            entry = ix->entry;
        }
    }
    if (entry >= ix->n) return fail(BS_ERR_INVALID_ARGUMENT, "entry point %u out of range", entry);
    if (!mi.rabitq) {
        std::lock_guard<std::mutex> lk(ix->mu);
        const bs_status bs = ensure_blocks(ix);
        if (bs != BS_OK) return bs;
    }

    SearchParams p;
    LaunchShape shape;
    fill_params(ix, mi, prm, entry, p, shape);
    p.nq = nq;
    const bool use_team = p.team_qlo <= p.team_qhi;
    char why[256] = {0};
    if (plan(ix, p, shape, why, sizeof(why)) != cudaSuccess)
        return fail(BS_ERR_UNSUPPORTED, "%s", why);

    if (stats) {
        std::memset(stats, 0, sizeof(*stats));
        stats->entry_point = entry;
        stats->integer_exact = use_team ? 1u : 0u;
        stats->row_bytes = ix->u8 ? ix->row_bytes : ix->row_stride * 4u;
        stats->block_bytes = p.nb ? p.nb_stride : p.rq_nb ? p.rq_stride : 0u;
        stats->warps_per_query = shape.block_query ? static_cast<uint32_t>(shape.warps_per_block) : 1u;
    }
    if (nq == 0) return BS_OK;

    cudaError_t e0 = cudaSuccess;
    if (any_foreign(ix->device, {queries, ids, dists}))
        return fail(BS_ERR_INVALID_ARGUMENT, "a buffer lives on another GPU than the index (device %d)", ix->device);
    const bool q_dev = is_device_ptr(queries, ix->device);
    const bool i_dev = is_device_ptr(ids, ix->device);
    const bool d_dev = dists ? is_device_ptr(dists, ix->device) : true;
    // Host buffers that are page-locked and mapped into this device's
    // context are used in place: each warp reads its query over the bus when
    // it starts it and writes its result row back when it ends, so the
    // transfers overlap the search instead of bracketing it.  Pageable
    // buffers go through device staging and whole-batch copies.
    const float* q_map = q_dev ? nullptr : static_cast<const float*>(mapped_host_ptr(queries, ix->device));
    uint32_t* i_map = i_dev ? nullptr : static_cast<uint32_t*>(mapped_host_ptr(ids, ix->device));
    float* d_map = d_dev ? nullptr : static_cast<float*>(mapped_host_ptr(dists, ix->device));
    const bool i_stage = !i_dev && !i_map;
    const bool d_stage = dists && !d_dev && !d_map;
    const size_t qbytes = static_cast<size_t>(nq) * ix->dim * sizeof(float);
    const size_t obytes = static_cast<size_t>(nq) * p.K * sizeof(uint32_t);
    size_t off = 256;   // DevCounters at 0
    const size_t q_off = off;
    if (!q_dev) off += (qbytes + 255) & ~static_cast<size_t>(255);   // staging, or the kernel's query slots
    const size_t i_off = off;
    if (i_stage) off += (obytes + 255) & ~static_cast<size_t>(255);
    const size_t d_off = off;
    if (d_stage) off += (obytes + 255) & ~static_cast<size_t>(255);
    const size_t s_off = off;
    if (mi.rabitq && !p.rq_nb) {
        uint64_t warps = 0;
        e0 = bsb::rabitq_grid_warps(p, shape, ix->num_sms, warps);
        if (e0 != cudaSuccess) return cuda_fail(e0, "rabitq launch shape");
        off += static_cast<size_t>(warps) * p.spill_slots * sizeof(uint32_t);
    }

    char* scratch = nullptr;
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&scratch), off, stream);
    if (e != cudaSuccess) return cuda_fail(e, "search scratch");
    auto release = [&]() { cudaFreeAsync(scratch, stream); };
    p.counters = reinterpret_cast<DevCounters*>(scratch);
    p.queries = q_dev ? queries : reinterpret_cast<const float*>(scratch + q_off);
    p.queries_src = q_map;
    p.out_ids = i_dev ? ids : i_map ? i_map : reinterpret_cast<uint32_t*>(scratch + i_off);
    p.out_dists = !dists ? nullptr : d_dev ? dists : d_map ? d_map : reinterpret_cast<float*>(scratch + d_off);
    p.spill = (mi.rabitq && !p.rq_nb) ? reinterpret_cast<uint32_t*>(scratch + s_off) : nullptr;

    e = cudaMemsetAsync(scratch, 0, sizeof(DevCounters), stream);
    if (e == cudaSuccess && !q_dev && !q_map)
        e = cudaMemcpyAsync(scratch + q_off, queries, qbytes, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) { release(); return cuda_fail(e, "query upload"); }

    if (p.rq_nb) {
        // RaBitQ over node blocks: the index's visited arena, used by one
        // call at a time (stream order through rq_event)
        std::lock_guard<std::mutex> lk(ix->rq_mu);
        uint64_t cap = 0;
        e = bsb::rq_nb_capacity_warps(p, shape, ix->num_sms, cap);
        if (e != cudaSuccess) { release(); return cuda_fail(e, "rabitq launch shape"); }
        const bs_status as = ensure_visited_arena(ix, cap, static_cast<uint32_t>(shape.warps_per_block));
        if (as != BS_OK) { release(); return as; }
        p.vis = ix->d_vis;
        p.vis_words = ix->vis_words;
        p.vis_log_cap = ix->vis_log_cap;
        p.vis_warps = static_cast<uint32_t>(ix->vis_warps);
        e = cudaStreamWaitEvent(stream, ix->rq_event, 0);
        if (e == cudaSuccess) e = bsb::launch_search_rq_nb(p, shape, ix->num_sms, stream);
        if (e == cudaSuccess) e = cudaEventRecord(ix->rq_event, stream);
    } else {
        e = mi.rabitq          ? bsb::launch_search_rabitq(p, shape, ix->num_sms, stream)
            : shape.block_query ? bsb::launch_search_bq(p, shape, ix->num_sms, stream)
            : p.nb              ? bsb::launch_search_nb(p, shape, ix->num_sms, stream)
                                : bsb::launch_search(p, shape, ix->num_sms, stream);
    }
    if (e != cudaSuccess) { release(); return cuda_fail(e, "search launch"); }

    if (i_stage) e = cudaMemcpyAsync(ids, scratch + i_off, obytes, cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess && d_stage)
        e = cudaMemcpyAsync(dists, scratch + d_off, obytes, cudaMemcpyDeviceToHost, stream);
    DevCounters hc{};
    const bool sync = stats || !q_dev || !i_dev || !d_dev;
    if (e == cudaSuccess && sync)
        e = cudaMemcpyAsync(&hc, scratch, sizeof(hc), cudaMemcpyDeviceToHost, stream);
    release();
    if (e != cudaSuccess) return cuda_fail(e, "result download");
    if (!sync) return BS_OK;
    e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return cuda_fail(e, "search");
    if (stats) {
        stats->expansions = hc.expansions;
        stats->distances = hc.distances;
        stats->estimates = hc.estimates;
        stats->rerank = hc.rerank;
        stats->error_flags = hc.error_flags;
        stats->integer_exact = (use_team && hc.team_fallbacks == 0) ? 1u : 0u;
    }
    if (hc.error_flags) return fail(BS_ERR_KERNEL, "search kernel reported error flags 0x%x", hc.error_flags);
    return BS_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free search (bs_search_no_alloc).
//
// Some callers cannot allocate device memory once they are running: a host
// process that reserves the GPU's memory at start-up and forbids later
// allocations (a serving process with a fixed memory budget, or a plugin that
// lives inside a runtime owning all device memory through its own
// allocator), or a latency-critical loop where cudaMalloc's possible
// device-wide blocking, or its failure under memory pressure, is not
// acceptable.  For them the search kernel's scratch -- its work-queue counter,
// statistics and error flags, and on a device's first entry-point computation
// the centroid -- lives in the fixed array below instead of in per-call
// allocations.
//
// The array is a file-scope __device__ variable: every GPU that loads this
// library holds one copy of kFixedScratchBytes until the process exits.  In
// host code its name is only a host-side stand-in, never a device address, so
// the device address is looked up once per device with cudaGetSymbolAddress
// (with that device current) and passed to the kernels.
static constexpr size_t kFixedScratchBytes = 16384;
static constexpr size_t kFixedEntryOffset = 256;       // [0,256): search counters
static constexpr uint32_t kFixedMaxQueries = 1u << 31;  // keeps the u32 work counter from wrapping
static __device__ __align__(256) unsigned char g_fixed_scratch[kFixedScratchBytes];
static_assert(sizeof(DevCounters) <= kFixedEntryOffset, "search counters must fit below the entry scratch");

namespace {

constexpr int kFixedMaxDevices = 64;
std::mutex g_fixed_mu;
unsigned char* g_fixed_addr[kFixedMaxDevices] = {};

// Device address of g_fixed_scratch on `device`, which must be current.
bs_status fixed_scratch(int device, unsigned char** out) {
    if (device < 0 || device >= kFixedMaxDevices)
        return fail(BS_ERR_UNSUPPORTED, "device %d is beyond the %d devices the fixed scratch tracks", device,
                    kFixedMaxDevices);
    std::lock_guard<std::mutex> lk(g_fixed_mu);
    if (!g_fixed_addr[device]) {
        void* addr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&addr, g_fixed_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_fixed_scratch)");
        g_fixed_addr[device] = static_cast<unsigned char*>(addr);
    }
    *out = g_fixed_addr[device];
    return BS_OK;
}

}  // namespace

extern "C" {

BS_API bs_status bs_search_no_alloc(bs_index* ix, const bs_search_params* prm, const float* queries, uint32_t nq,
                                    uint32_t* ids, float* dists, void* stream_) {
    if (!ix || !prm) return fail(BS_ERR_INVALID_ARGUMENT, "index or params is NULL");
    ModeInfo mi;
    if (!parse_mode(prm->mode, mi)) return fail(BS_ERR_INVALID_ARGUMENT, "Unknown mode: %s", prm->mode ? prm->mode : "(null)");
    if (mi.rabitq)
        return fail(BS_ERR_UNSUPPORTED,
                    "rabitq needs visited bitmaps over all node ids per warp, far beyond the %zu-byte fixed scratch; "
                    "use bs_search",
                    kFixedScratchBytes);
    if (prm->K <= 0) return fail(BS_ERR_INVALID_ARGUMENT, "K must be positive");
    if (prm->topk_size == 0) return fail(BS_ERR_INVALID_ARGUMENT, "topk_size must be positive");
    if (prm->max_iterations < 0) return fail(BS_ERR_INVALID_ARGUMENT, "max_iterations must be >= 0");
    if (nq > kFixedMaxQueries)
        return fail(BS_ERR_UNSUPPORTED, "nq %u exceeds the fixed-scratch limit of %u queries per call", nq,
                    kFixedMaxQueries);
    if (nq > 0 && (!queries || !ids)) return fail(BS_ERR_INVALID_ARGUMENT, "queries or ids is NULL");

    DeviceGuard g(ix->device);
    if (!g.ok) return fail(BS_ERR_CUDA, "cannot select device %d", ix->device);
    if (nq > 0 && any_foreign(ix->device, {queries, ids, dists}))
        return fail(BS_ERR_INVALID_ARGUMENT, "a buffer lives on another GPU than the index (device %d)", ix->device);
    if (nq > 0 && (!is_device_ptr(queries, ix->device) || !is_device_ptr(ids, ix->device) ||
                   (dists && !is_device_ptr(dists, ix->device))))
        return fail(BS_ERR_INVALID_ARGUMENT,
                    "bs_search_no_alloc takes device pointers only (host buffers would need staging memory)");
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    unsigned char* scratch = nullptr;
    bs_status s = fixed_scratch(ix->device, &scratch);
    if (s != BS_OK) return s;

    uint32_t entry = prm->entry_point;
    if (entry == BS_NO_NODE) {
        std::lock_guard<std::mutex> lk(ix->mu);
        if (!ix->entry_valid) {
            // centroid (dim floats) + packed argmin key, then the u32 result
            const size_t need = bsb::entry_point_scratch_bytes(ix->n, ix->dim) + 8;
            if (kFixedEntryOffset + need > kFixedScratchBytes)
                return fail(BS_ERR_UNSUPPORTED,
                            "dim %d is too large to compute the entry point in the %zu-byte fixed scratch; "
                            "pass entry_point or call bs_index_entry_point first",
                            ix->dim, kFixedScratchBytes);
            unsigned char* es = scratch + kFixedEntryOffset;
            uint32_t* d_out = reinterpret_cast<uint32_t*>(es + need - 8);
            cudaError_t e = entry_kernels(ix, d_out, reinterpret_cast<float*>(es), stream);
            uint32_t h = 0;
            if (e == cudaSuccess) e = cudaMemcpyAsync(&h, d_out, 4, cudaMemcpyDeviceToHost, stream);
            if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
            if (e != cudaSuccess) return cuda_fail(e, "entry point kernel");
            ix->entry = h;
            ix->entry_valid = true;
        }
        entry = ix->entry;
    }
    if (entry >= ix->n) return fail(BS_ERR_INVALID_ARGUMENT, "entry point %u out of range", entry);
    if (nq == 0) return BS_OK;

    SearchParams p;
    LaunchShape shape;
    fill_params(ix, mi, prm, entry, p, shape);
    p.queries = queries;
    p.nq = nq;
    p.out_ids = ids;
    p.out_dists = dists;
    p.counters = reinterpret_cast<DevCounters*>(scratch);
    char why[256] = {0};
    if (plan(ix, p, shape, why, sizeof(why)) != cudaSuccess)
        return fail(BS_ERR_UNSUPPORTED, "%s", why);

    // the array keeps the previous call's contents: the work queue and the
    // counters must start from zero
    cudaError_t e = cudaMemsetAsync(scratch, 0, sizeof(DevCounters), stream);
    if (e != cudaSuccess) return cuda_fail(e, "fixed scratch reset");
    e = shape.block_query ? bsb::launch_search_bq(p, shape, ix->num_sms, stream)
        : p.nb            ? bsb::launch_search_nb(p, shape, ix->num_sms, stream)
                          : bsb::launch_search(p, shape, ix->num_sms, stream);
    if (e != cudaSuccess) return cuda_fail(e, "search launch");
    return BS_OK;
}

BS_API bs_status bs_merge_shards(const float* dists, const uint32_t* ids, uint32_t shards, uint32_t nq,
                                 uint32_t K, const uint32_t* id_offsets, uint32_t K_out, uint32_t* out_ids,
                                 float* out_dists, void* stream) {
    if (shards == 0 || shards > bsb::kMaxShards)
        return fail(BS_ERR_INVALID_ARGUMENT, "shards must be in 1..%u", bsb::kMaxShards);
    if (K == 0 || K_out == 0 || K_out > static_cast<uint64_t>(shards) * K)
        return fail(BS_ERR_INVALID_ARGUMENT, "need 0 < K_out <= shards * K");
    if (!id_offsets) return fail(BS_ERR_INVALID_ARGUMENT, "id_offsets is NULL");
    if (nq == 0) return BS_OK;
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "device query");
    if (!is_device_ptr(dists, dev) || !is_device_ptr(ids, dev) || !is_device_ptr(out_ids, dev) ||
        (out_dists && !is_device_ptr(out_dists, dev)))
        return fail(BS_ERR_INVALID_ARGUMENT, "bs_merge_shards takes device pointers on the current device");
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "device query");
    bsb::MergeArgs a{};
    a.dists = dists;
    a.ids = ids;
    a.shards = shards;
    a.nq = nq;
    a.K = K;
    a.K_out = K_out;
    for (uint32_t s = 0; s < shards; ++s) a.offsets[s] = id_offsets[s];
    a.out_ids = out_ids;
    a.out_dists = out_dists;
    e = bsb::launch_merge_shards(a, sms, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "merge launch");
    return BS_OK;
}

BS_API bs_status bs_device_alloc(const bs_index* ix, size_t bytes, void** dptr) {
    if (!ix || !dptr) return fail(BS_ERR_INVALID_ARGUMENT, "index or dptr is NULL");
    DeviceGuard g(ix->device);
    const cudaError_t e = cudaMalloc(dptr, bytes ? bytes : 1);
    return e == cudaSuccess ? BS_OK : cuda_fail(e, "bs_device_alloc");
}

BS_API bs_status bs_device_free(const bs_index* ix, void* dptr) {
    if (!ix) return fail(BS_ERR_INVALID_ARGUMENT, "index is NULL");
    DeviceGuard g(ix->device);
    const cudaError_t e = cudaFree(dptr);
    return e == cudaSuccess ? BS_OK : cuda_fail(e, "bs_device_free");
}

BS_API bs_status bs_copy_to_device(const bs_index* ix, void* dst, const void* src, size_t bytes) {
    if (!ix) return fail(BS_ERR_INVALID_ARGUMENT, "index is NULL");
    DeviceGuard g(ix->device);
    const cudaError_t e = cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice);
    return e == cudaSuccess ? BS_OK : cuda_fail(e, "bs_copy_to_device");
}

BS_API bs_status bs_copy_to_host(const bs_index* ix, void* dst, const void* src, size_t bytes) {
    if (!ix) return fail(BS_ERR_INVALID_ARGUMENT, "index is NULL");
    DeviceGuard g(ix->device);
    const cudaError_t e = cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? BS_OK : cuda_fail(e, "bs_copy_to_host");
}

BS_API bs_status bs_device_fill(const bs_index* ix, void* dptr, int byte_value, size_t bytes) {
    if (!ix) return fail(BS_ERR_INVALID_ARGUMENT, "index is NULL");
    DeviceGuard g(ix->device);
    const cudaError_t e = cudaMemset(dptr, byte_value, bytes);
    return e == cudaSuccess ? BS_OK : cuda_fail(e, "bs_device_fill");
}

BS_API bs_status bs_synchronize(const bs_index* ix, void* stream) {
    if (!ix) return fail(BS_ERR_INVALID_ARGUMENT, "index is NULL");
    DeviceGuard g(ix->device);
    const cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? BS_OK : cuda_fail(e, "bs_synchronize");
}

}  // extern "C"
