// bs_ground_truth.cu -- exact brute-force k nearest rows of every query, the
// ground truth a recall figure is measured against (the reference reads it
// from ivecs files made elsewhere, src/gpu_cli.cu:379-381; script/unpack.py).
//
// Distances are the search's own: the reference's sequential fp32 sum
// (include/cpu_search_base.hpp:29-37), or exact integer sums for byte rows
// and integer queries (any order gives the same value); the k best are taken
// by (distance, id).
//
// One warp scores 8 queries against a range of rows, one row per lane, so a
// row is read once for 8 queries (byte rows: 16-byte chunks, one __dp4a per 4
// bytes and query plus the row's own sum of squares).  Keys below a query's
// current k-th key are appended to its candidate buffer in shared memory; a
// full buffer is merged into the query's sorted top-k list by a bitonic sort
// of the two.  The rows are split into ranges so that every SM has work; the
// ranges' lists are merged per query by the shard-merge kernel.
#include <cfloat>
#include <cstdint>

#include "bs_device.cuh"
#include "bs_internal.h"
#include "bs_score.cuh"

namespace bsb {

using namespace dev;

namespace {

constexpr uint32_t kGtQ = 8;        // queries per warp

__device__ __forceinline__ unsigned long long gt_key(float d, uint32_t id) {
    return (static_cast<unsigned long long>(f2ord(d)) << 32) | id;
}

// Sorts k[0, P) ascending, P a power of two (a bitonic sort of one warp over
// shared memory; partner i ^ stride < P).
__device__ __forceinline__ void gt_sort(unsigned long long* k, uint32_t P, unsigned lane) {
    for (uint32_t size = 2; size <= P; size <<= 1) {
        for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
            for (uint32_t i = lane; i < P; i += 32) {
                const uint32_t j = i ^ stride;
                if (j > i) {
                    const unsigned long long x = k[i], y = k[j];
                    if ((x > y) == ((i & size) == 0)) { k[i] = y; k[j] = x; }
                }
            }
            __syncwarp();
        }
    }
}

template <int DM>
__global__ void __launch_bounds__(128) k_gt_partial(const GroundTruthArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const SearchParams& sp = a.sp;
    const unsigned lane = threadIdx.x & 31u;
    unsigned char* ws = smem_raw + static_cast<size_t>(threadIdx.x >> 5) * a.smem_per_warp;
    float* qf = reinterpret_cast<float*>(ws);                                        // [kGtQ][row_stride]
    unsigned char* qb = ws + a.off_qb;                                               // [kGtQ][row_bytes]
    uint32_t* qq = reinterpret_cast<uint32_t*>(ws + a.off_qq);                       // [kGtQ]
    // per query: its sorted list (kcap keys) followed by its candidate buffer
    // (kcap keys): 2 * kcap, a power of two, sorted as one
    unsigned long long* lists = reinterpret_cast<unsigned long long*>(ws + a.off_lists);  // [kGtQ][2 * kcap]
    const uint32_t span = 2u * a.kcap;
    const unsigned lt_mask = (1u << lane) - 1u;

    const uint64_t gw = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const uint64_t groups = (a.nq + kGtQ - 1) / kGtQ;
    if (gw >= groups * a.splits) return;
    const uint32_t g = static_cast<uint32_t>(gw / a.splits), split = static_cast<uint32_t>(gw % a.splits);
    const uint64_t per = (sp.n + a.splits - 1) / a.splits;
    const uint64_t lo = split * per, hi = lo + per < sp.n ? lo + per : sp.n;
    const uint32_t q0 = g * kGtQ;
    const uint32_t nqg = a.nq - q0 < kGtQ ? a.nq - q0 : kGtQ;

    // the group's queries; byte rows also get them packed, when integer
    unsigned team = 0;   // bit j: query j takes the integer-exact path
    for (uint32_t j = 0; j < kGtQ; ++j) {
        float* dst = qf + j * sp.row_stride;
        for (uint32_t d = lane; d < sp.row_stride; d += 32)
            dst[d] = (j < nqg && d < sp.dim) ? a.queries[static_cast<size_t>(q0 + j) * sp.dim + d] : 0.0f;
        __syncwarp();
        const bool tj = DM != kSeq && j < nqg && query_integer_exact(dst, sp.dim, sp.team_qlo, sp.team_qhi);
        team |= tj ? (1u << j) : 0u;
        if (DM == kU8 && tj) {
            pack_query_u8(dst, sp.dim, sp.row_bytes, reinterpret_cast<uint32_t*>(qb + j * (sp.row_bytes + 16u)), lane);
            if (lane == 0) qq[j] = reinterpret_cast<const uint32_t*>(qb + j * (sp.row_bytes + 16u))[sp.row_bytes / 4u];
        }
    }
    for (uint32_t i = lane; i < kGtQ * span; i += 32) lists[i] = kEmptyKey;
    uint32_t nbuf[kGtQ];
    unsigned long long thr[kGtQ];
#pragma unroll
    for (uint32_t j = 0; j < kGtQ; ++j) { nbuf[j] = 0; thr[j] = kEmptyKey; }
    __syncwarp();

    auto flush = [&](uint32_t j) {
        unsigned long long* L = lists + j * span;
        __syncwarp();
        gt_sort(L, span, lane);
        for (uint32_t i = a.kcap + lane; i < span; i += 32) L[i] = kEmptyKey;
        __syncwarp();
        thr[j] = L[a.k - 1];
        nbuf[j] = 0;
    };

    for (uint64_t r0 = lo; r0 < hi; r0 += 32) {
        const uint64_t row = r0 + lane;
        const bool ok = row < hi;
        float d[kGtQ];
        if (DM == kU8) {
            const unsigned char* x = sp.vecs8 + (ok ? row : lo) * sp.row_bytes;
            unsigned xx = 0, qx[kGtQ];
            for (uint32_t j = 0; j < kGtQ; ++j) qx[j] = 0;
            for (uint32_t c = 0; c < sp.row_bytes; c += 16) {
                const uint4 v = *reinterpret_cast<const uint4*>(x + c);
                xx = __dp4a(v.x, v.x, xx); xx = __dp4a(v.y, v.y, xx);
                xx = __dp4a(v.z, v.z, xx); xx = __dp4a(v.w, v.w, xx);
#pragma unroll
                for (uint32_t j = 0; j < kGtQ; ++j) {
                    const uint4 qv = *reinterpret_cast<const uint4*>(qb + j * (sp.row_bytes + 16u) + c);
                    qx[j] = __dp4a(qv.x, v.x, qx[j]); qx[j] = __dp4a(qv.y, v.y, qx[j]);
                    qx[j] = __dp4a(qv.z, v.z, qx[j]); qx[j] = __dp4a(qv.w, v.w, qx[j]);
                }
            }
#pragma unroll
            for (uint32_t j = 0; j < kGtQ; ++j) {
                if ((team >> j) & 1u) {
                    d[j] = static_cast<float>(xx - 2u * qx[j] + qq[j]);
                } else {
                    float s = 0.0f;
                    const float* q = qf + j * sp.row_stride;
                    for (uint32_t t = 0; t < sp.dim; ++t) {
                        const float u = __fsub_rn(q[t], static_cast<float>(x[t]));
                        s = __fadd_rn(s, __fmul_rn(u, u));
                    }
                    d[j] = s;
                }
            }
        } else {
            const float* x = sp.vecs + (ok ? row : lo) * sp.row_stride;
            float s[kGtQ];
            for (uint32_t j = 0; j < kGtQ; ++j) s[j] = 0.0f;
            for (uint32_t t = 0; t < sp.row_stride; t += 4) {
                const float4 v = *reinterpret_cast<const float4*>(x + t);
#pragma unroll
                for (uint32_t j = 0; j < kGtQ; ++j) {
                    const float4 q = *reinterpret_cast<const float4*>(qf + j * sp.row_stride + t);
                    float u;
                    if (DM == kTeam && ((team >> j) & 1u)) {
                        u = q.x - v.x; s[j] = fmaf(u, u, s[j]);
                        u = q.y - v.y; s[j] = fmaf(u, u, s[j]);
                        u = q.z - v.z; s[j] = fmaf(u, u, s[j]);
                        u = q.w - v.w; s[j] = fmaf(u, u, s[j]);
                    } else {
                        u = __fsub_rn(q.x, v.x); s[j] = __fadd_rn(s[j], __fmul_rn(u, u));
                        u = __fsub_rn(q.y, v.y); s[j] = __fadd_rn(s[j], __fmul_rn(u, u));
                        u = __fsub_rn(q.z, v.z); s[j] = __fadd_rn(s[j], __fmul_rn(u, u));
                        u = __fsub_rn(q.w, v.w); s[j] = __fadd_rn(s[j], __fmul_rn(u, u));
                    }
                }
            }
#pragma unroll
            for (uint32_t j = 0; j < kGtQ; ++j) d[j] = s[j];
        }
#pragma unroll
        for (uint32_t j = 0; j < kGtQ; ++j) {
            if (j >= nqg) break;
            const unsigned long long key = gt_key(d[j], static_cast<uint32_t>(row));
            const bool pass = ok && key < thr[j];
            const unsigned bm = __ballot_sync(kFull, pass);
            if (!bm) continue;
            if (nbuf[j] + __popc(bm) > a.kcap) flush(j);
            const bool pass2 = ok && key < thr[j];
            const unsigned bm2 = __ballot_sync(kFull, pass2);
            if (pass2) lists[j * span + a.kcap + nbuf[j] + __popc(bm2 & lt_mask)] = key;
            nbuf[j] += __popc(bm2);
        }
    }
#pragma unroll
    for (uint32_t j = 0; j < kGtQ; ++j) {
        if (j >= nqg) break;
        flush(j);
        const unsigned long long* L = lists + j * span;
        const size_t at = (static_cast<size_t>(split) * a.nq + q0 + j) * a.k;
        for (uint32_t i = lane; i < a.k; i += 32) {
            const unsigned long long key = L[i];
            a.part_i[at + i] = key == kEmptyKey ? kNoNode : static_cast<uint32_t>(key);
            a.part_d[at + i] = key == kEmptyKey ? FLT_MAX : key_dist(key);
        }
    }
}

using GtFn = void (*)(GroundTruthArgs);

GtFn select_gt(int dm) {
    if (dm == kU8) return k_gt_partial<kU8>;
    if (dm == kTeam) return k_gt_partial<kTeam>;
    return k_gt_partial<kSeq>;
}

}  // namespace

cudaError_t plan_ground_truth(GroundTruthArgs& a, size_t smem_optin, int num_sms) {
    const SearchParams& sp = a.sp;
    uint32_t kcap = 32;
    while (kcap < a.k) kcap <<= 1;
    a.kcap = kcap;
    auto a16 = [](uint32_t x) { return (x + 15u) & ~15u; };
    uint32_t off = a16(kGtQ * sp.row_stride * 4u);
    a.off_qb = off;
    off = a16(off + kGtQ * (sp.row_bytes + 16u));
    a.off_qq = off;
    off = a16(off + kGtQ * 4u);
    a.off_lists = off;
    off = a16(off + kGtQ * 2u * kcap * 8u);
    a.smem_per_warp = off;
    a.warps_per_block = static_cast<uint32_t>(smem_optin / off);
    if (a.warps_per_block == 0) return cudaErrorInvalidValue;
    if (a.warps_per_block > 4) a.warps_per_block = 4;
    const uint64_t groups = (static_cast<uint64_t>(a.nq) + kGtQ - 1) / kGtQ;
    const uint64_t want = static_cast<uint64_t>(num_sms) * 16u;
    uint64_t splits = (want + groups - 1) / groups;
    if (splits < 1) splits = 1;
    if (splits > kMaxShards) splits = kMaxShards;
    if (splits > a.sp.n) splits = a.sp.n;
    a.splits = static_cast<uint32_t>(splits);
    return cudaSuccess;
}

cudaError_t launch_ground_truth(const GroundTruthArgs& a, int num_sms, cudaStream_t stream) {
    const int dm = a.sp.vecs8 ? kU8 : (a.sp.team_qlo <= a.sp.team_qhi ? kTeam : kSeq);
    GtFn fn = select_gt(dm);
    const size_t smem = static_cast<size_t>(a.smem_per_warp) * a.warps_per_block;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const uint64_t warps = (static_cast<uint64_t>(a.nq) + kGtQ - 1) / kGtQ * a.splits;
    const unsigned blocks = static_cast<unsigned>((warps + a.warps_per_block - 1) / a.warps_per_block);
    if (blocks) fn<<<blocks, 32 * a.warps_per_block, smem, stream>>>(a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    MergeArgs m{};
    m.dists = a.part_d;
    m.ids = a.part_i;
    m.shards = a.splits;
    m.nq = a.nq;
    m.K = a.k;
    m.K_out = a.k;
    m.out_ids = a.out_ids;
    m.out_dists = a.out_dists;
    return launch_merge_shards(m, num_sms, stream);
}

}  // namespace bsb
