// bs_device.cuh -- warp-level device primitives of the beam search.
//
//  * 64-bit beam keys: (order-preserving fp32 distance, node id, expanded bit)
//    so that every comparison is the reference CPU comparator "(dist, id)"
//    (include/cpu_search_base.hpp:48-51) in one integer compare.
//  * register-resident bitonic sort / merge over a striped warp layout
//    (element p lives in register p/32 of lane p%32); the beam's role is that
//    of RegBitonicTopK (include/topk_reg.cuh) but ordered by (dist, id).
//  * shared-memory visited filters (exact hash set, Bloom filter).
//  * the two distance evaluators (sequential per lane, or 8-lane teams).
#pragma once

#include <cfloat>
#include <cstdint>
#include <cuda_runtime.h>

namespace bsb {
namespace dev {

constexpr unsigned kFull = 0xffffffffu;
constexpr uint64_t kEmptyKey = ~0ull;
constexpr uint32_t kNoNode = 0xffffffffu;

// ---------------------------------------------------------------- beam keys

// Monotone map fp32 -> u32 (negative values flip all bits, others set the
// sign bit).  -0 is folded onto +0 because the reference comparator treats
// them as equal.
__device__ __forceinline__ uint32_t f2ord(float f) {
    uint32_t u = __float_as_uint(f);
    if (u == 0x80000000u) u = 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float ord2f(uint32_t o) {
    const uint32_t u = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
    return __uint_as_float(u);
}

// key = ord(dist) << 32 | id << 1 | expanded.  Node ids are < 2^31, ids are
// unique inside a beam, so the expanded bit never decides an order.
__device__ __forceinline__ uint64_t make_key(float d, uint32_t id) {
    return (static_cast<uint64_t>(f2ord(d)) << 32) | (static_cast<uint64_t>(id) << 1);
}
__device__ __forceinline__ uint32_t key_id(uint64_t k) { return static_cast<uint32_t>(k) >> 1; }
__device__ __forceinline__ float key_dist(uint64_t k) { return ord2f(static_cast<uint32_t>(k >> 32)); }
__device__ __forceinline__ uint64_t kmin(uint64_t a, uint64_t b) { return a < b ? a : b; }
__device__ __forceinline__ uint64_t kmax(uint64_t a, uint64_t b) { return a < b ? b : a; }

// ------------------------------------------------------- bitonic networks

// One compare-exchange stage of a bitonic network of 32*N elements in the
// striped layout.  SIZE is the bitonic block size (direction ascending when
// (p & SIZE) == 0), STRIDE the partner distance.  Both are template constants
// so the whole network unrolls into register moves and shuffles.
template <int N, unsigned SIZE, unsigned STRIDE>
__device__ __forceinline__ void cmpx_stage(uint64_t (&k)[N], unsigned lane) {
    if constexpr (STRIDE >= 32) {
        constexpr unsigned rs = STRIDE >> 5;
#pragma unroll
        for (int r = 0; r < N; ++r) {
            if ((static_cast<unsigned>(r) & rs) == 0) {
                const int r2 = r | static_cast<int>(rs);
                const bool asc = ((static_cast<unsigned>(r) * 32u) & SIZE) == 0;
                const uint64_t lo = kmin(k[r], k[r2]);
                const uint64_t hi = kmax(k[r], k[r2]);
                k[r] = asc ? lo : hi;
                k[r2] = asc ? hi : lo;
            }
        }
    } else {
        const bool lower = (lane & STRIDE) == 0;
#pragma unroll
        for (int r = 0; r < N; ++r) {
            const uint64_t o = __shfl_xor_sync(kFull, k[r], STRIDE);
            const unsigned p = static_cast<unsigned>(r) * 32u + lane;
            const bool asc = (p & SIZE) == 0;
            k[r] = (asc == lower) ? kmin(k[r], o) : kmax(k[r], o);
        }
    }
}

template <int N, unsigned SIZE, unsigned STRIDE>
__device__ __forceinline__ void merge_stages(uint64_t (&k)[N], unsigned lane) {
    if constexpr (STRIDE > 0) {
        cmpx_stage<N, SIZE, STRIDE>(k, lane);
        merge_stages<N, SIZE, STRIDE / 2>(k, lane);
    }
}

template <int N, unsigned SIZE>
__device__ __forceinline__ void sort_stages(uint64_t (&k)[N], unsigned lane) {
    if constexpr (SIZE >= 2) {
        sort_stages<N, SIZE / 2>(k, lane);
        merge_stages<N, SIZE, SIZE / 2>(k, lane);
    }
}

// Full ascending sort of 32*N keys.
template <int N>
__device__ __forceinline__ void sort_asc(uint64_t (&k)[N], unsigned lane) {
    sort_stages<N, 32u * N>(k, lane);
}

// Bitonic 32*N keys -> ascending (one merge pass).
template <int N>
__device__ __forceinline__ void merge_asc(uint64_t (&k)[N], unsigned lane) {
    merge_stages<N, 32u * N, 16u * N>(k, lane);
}

// Keep the `topk` smallest keys of beam (ascending, 32*RX) and cand (any
// order, 32*RY), ascending in beam.  cand is clobbered.
template <int RX, int RY>
__device__ __forceinline__ void beam_merge(uint64_t (&beam)[RX], uint64_t (&cand)[RY],
                                           unsigned lane, unsigned topk) {
    static_assert(RX >= RY, "beam must be at least as wide as the candidate batch");
    sort_asc<RY>(cand, lane);
    // Pair the beam's largest 32*RY positions with the candidates reversed:
    // min() of an ascending and a descending run keeps the smallest half and
    // leaves a bitonic sequence.
#pragma unroll
    for (int r = RX - RY; r < RX; ++r) {
        const uint64_t c = __shfl_xor_sync(kFull, cand[RX - 1 - r], 31);
        beam[r] = kmin(beam[r], c);
    }
    merge_asc<RX>(beam, lane);
#pragma unroll
    for (int r = 0; r < RX; ++r)
        if (static_cast<unsigned>(r) * 32u + lane >= topk) beam[r] = kEmptyKey;
}

// Insert one key c into the ascending beam (kept to `topk` entries): every
// entry above c moves up one position.  A key at or past position topk is
// dropped, so inserting a key that no longer fits leaves the beam unchanged.
template <int RX>
__device__ __forceinline__ void beam_insert1(uint64_t (&beam)[RX], unsigned lane, uint64_t c,
                                             unsigned topk) {
    unsigned pos = 0;
#pragma unroll
    for (int r = 0; r < RX; ++r) pos += __popc(__ballot_sync(kFull, beam[r] < c));
    uint64_t up[RX], last[RX];
#pragma unroll
    for (int r = 0; r < RX; ++r) {
        up[r] = __shfl_up_sync(kFull, beam[r], 1);
        last[r] = __shfl_sync(kFull, beam[r], 31);
    }
#pragma unroll
    for (int r = 0; r < RX; ++r) {
        const unsigned p = static_cast<unsigned>(r) * 32u + lane;
        const uint64_t prev = lane ? up[r] : (r > 0 ? last[r > 0 ? r - 1 : 0] : kEmptyKey);
        const uint64_t nv = p > pos ? prev : (p == pos ? c : beam[r]);
        beam[r] = p >= topk ? kEmptyKey : nv;
    }
}

// Merge `count` candidate keys, already compacted into ckeys[0..count) in
// shared memory, into the beam.  One or two keys are shifted in directly;
// otherwise the keys are sorted with the smallest bitonic network that holds
// them (8, 16, 32 or 32*RY; the empty slots hold kEmptyKey, the largest key,
// so the full candidate array is sorted) and merged as in beam_merge.
template <int RX, int RY>
__device__ __forceinline__ void beam_merge_compact(uint64_t (&beam)[RX], const uint64_t* ckeys,
                                                   unsigned count, unsigned lane, unsigned topk) {
    if (count <= 2) {
        for (unsigned j = 0; j < count; ++j) beam_insert1<RX>(beam, lane, ckeys[j], topk);
        return;
    }
    uint64_t cand[RY];
#pragma unroll
    for (int r = 0; r < RY; ++r) {
        const unsigned s = static_cast<unsigned>(r) * 32u + lane;
        cand[r] = s < count ? ckeys[s] : kEmptyKey;
    }
    if (count <= 8) sort_stages<RY, 8>(cand, lane);
    else if (count <= 16) sort_stages<RY, 16>(cand, lane);
    else if (count <= 32) sort_stages<RY, 32>(cand, lane);
    else sort_stages<RY, 32u * RY>(cand, lane);
#pragma unroll
    for (int r = RX - RY; r < RX; ++r) {
        const uint64_t c = __shfl_xor_sync(kFull, cand[RX - 1 - r], 31);
        beam[r] = kmin(beam[r], c);
    }
    merge_asc<RX>(beam, lane);
#pragma unroll
    for (int r = 0; r < RX; ++r)
        if (static_cast<unsigned>(r) * 32u + lane >= topk) beam[r] = kEmptyKey;
}

// ---- the same networks with the lane-level stages (partner distance < 32)
// as runtime loops: one copy of a stage's code instead of one per stage, for
// kernels whose unrolled networks would not fit the instruction cache (wide
// beams); the register-level stages stay unrolled (their register indices
// must be constants).

template <int N>
__device__ __forceinline__ void cmpx_shfl(uint64_t (&k)[N], unsigned lane, unsigned size, unsigned stride) {
    const bool lower = (lane & stride) == 0;
#pragma unroll
    for (int r = 0; r < N; ++r) {
        const uint64_t o = __shfl_xor_sync(kFull, k[r], stride);
        const unsigned p = static_cast<unsigned>(r) * 32u + lane;
        const bool asc = (p & size) == 0;
        k[r] = (asc == lower) ? kmin(k[r], o) : kmax(k[r], o);
    }
}

template <int N, unsigned SIZE, unsigned STRIDE>
__device__ __forceinline__ void merge_reg_stages(uint64_t (&k)[N], unsigned lane) {
    if constexpr (STRIDE >= 32) {
        cmpx_stage<N, SIZE, STRIDE>(k, lane);
        merge_reg_stages<N, SIZE, STRIDE / 2>(k, lane);
    }
}

// bitonic merge of blocks of SIZE keys (SIZE a power of two, <= 32*N)
template <int N, unsigned SIZE>
__device__ __forceinline__ void merge_rt(uint64_t (&k)[N], unsigned lane) {
    merge_reg_stages<N, SIZE, SIZE / 2>(k, lane);
#pragma unroll 1
    for (unsigned stride = (SIZE / 2 < 16u ? SIZE / 2 : 16u); stride > 0; stride >>= 1)
        cmpx_shfl<N>(k, lane, SIZE, stride);
}

template <int N, unsigned SIZE>
__device__ __forceinline__ void sort_big_rt(uint64_t (&k)[N], unsigned lane) {
    if constexpr (SIZE >= 64) {
        sort_big_rt<N, SIZE / 2>(k, lane);
        merge_rt<N, SIZE>(k, lane);
    }
}

// ascending sort of blocks of SIZE keys (the whole array for SIZE = 32*N)
template <int N, unsigned SIZE>
__device__ __forceinline__ void sort_rt(uint64_t (&k)[N], unsigned lane) {
    constexpr unsigned kLane = SIZE < 32u ? SIZE : 32u;
#pragma unroll 1
    for (unsigned size = 2; size <= kLane; size <<= 1)
#pragma unroll 1
        for (unsigned stride = size >> 1; stride > 0; stride >>= 1) cmpx_shfl<N>(k, lane, size, stride);
    sort_big_rt<N, SIZE>(k, lane);
}

// beam_merge_compact for wide beams (RaBitQ: topk up to 512).  Up to kIns
// keys are shifted in one at a time.  Otherwise the keys are sorted and paired
// with the beam's last rows as in beam_merge_compact; every beam row whose
// largest key is at or below the smallest candidate is left alone (all its
// keys precede every candidate), and the bitonic merge runs only over the
// smallest power-of-two suffix of rows that holds the others.  That suffix,
// an ascending run whose tail was min-paired with the reversed candidates, is
// bitonic, so merging it alone sorts the whole beam.
template <int RX, int S>
__device__ __forceinline__ void merge_suffix(uint64_t (&beam)[RX], unsigned lane) {
    uint64_t sub[S];
#pragma unroll
    for (int i = 0; i < S; ++i) sub[i] = beam[RX - S + i];
    merge_rt<S, 32u * S>(sub, lane);
#pragma unroll
    for (int i = 0; i < S; ++i) beam[RX - S + i] = sub[i];
}

template <int RX, int RY>
__device__ __forceinline__ void beam_merge_compact_wide(uint64_t (&beam)[RX], const uint64_t* ckeys,
                                                        unsigned count, unsigned lane, unsigned topk) {
    constexpr unsigned kIns = RX >= 4 ? 3u : 2u;
    if (count <= kIns) {
        for (unsigned j = 0; j < count; ++j) beam_insert1<RX>(beam, lane, ckeys[j], topk);
        return;
    }
    uint64_t cand[RY];
#pragma unroll
    for (int r = 0; r < RY; ++r) {
        const unsigned s = static_cast<unsigned>(r) * 32u + lane;
        cand[r] = s < count ? ckeys[s] : kEmptyKey;
    }
    if (count <= 32) {
        // sort the first register row in blocks of the smallest power of two
        // that holds the keys (empty slots hold kEmptyKey, the largest key)
        unsigned size = 8;
        while (size < count) size <<= 1;
#pragma unroll 1
        for (unsigned sz = 2; sz <= size; sz <<= 1)
#pragma unroll 1
            for (unsigned stride = sz >> 1; stride > 0; stride >>= 1) cmpx_shfl<RY>(cand, lane, sz, stride);
    } else {
        sort_rt<RY, 32u * RY>(cand, lane);
    }
    const uint64_t cmin = __shfl_sync(kFull, cand[0], 0);
    int r0 = RX;
#pragma unroll
    for (int r = RX - 1; r >= 0; --r)
        if (__shfl_sync(kFull, beam[r], 31) > cmin) r0 = r;
#pragma unroll
    for (int r = RX - RY; r < RX; ++r) {
        const uint64_t c = __shfl_xor_sync(kFull, cand[RX - 1 - r], 31);
        beam[r] = kmin(beam[r], c);
    }
    if (RX >= 2 && RY <= 1 && r0 >= RX - 1) merge_suffix<RX, 1>(beam, lane);
    else if (RX >= 4 && RY <= 2 && r0 >= RX - 2) merge_suffix<RX, (RX >= 4 ? 2 : 1)>(beam, lane);
    else if (RX >= 8 && r0 >= RX - 4) merge_suffix<RX, (RX >= 8 ? 4 : 1)>(beam, lane);
    else merge_rt<RX, 32u * RX>(beam, lane);
#pragma unroll
    for (int r = 0; r < RX; ++r)
        if (static_cast<unsigned>(r) * 32u + lane >= topk) beam[r] = kEmptyKey;
}

// Smallest unexpanded entry: mark it and return its node id.  Branch-free
// over the registers so the beam stays in registers.
template <int RX>
__device__ __forceinline__ bool beam_pick(uint64_t (&beam)[RX], unsigned lane, uint32_t& node) {
    int sel = -1;
    unsigned sel_mask = 0;
#pragma unroll
    for (int r = 0; r < RX; ++r) {
        const bool open = beam[r] != kEmptyKey && (beam[r] & 1ull) == 0;
        const unsigned m = __ballot_sync(kFull, open);
        if (sel < 0 && m != 0) { sel = r; sel_mask = m; }
    }
    if (sel < 0) return false;
    const int src = __ffs(sel_mask) - 1;
    uint32_t mine = 0;
#pragma unroll
    for (int r = 0; r < RX; ++r)
        if (r == sel) mine = static_cast<uint32_t>(beam[r]) >> 1;
    node = __shfl_sync(kFull, mine, src);
    if (static_cast<int>(lane) == src) {
#pragma unroll
        for (int r = 0; r < RX; ++r)
            if (r == sel) beam[r] |= 1ull;
    }
    return true;
}

// beam_pick that also returns the entry the next pick would take if the beam
// did not change (kNoNode when there is none): a speculative prefetch target.
template <int RX>
__device__ __forceinline__ bool beam_pick_next(uint64_t (&beam)[RX], unsigned lane, uint32_t& node,
                                               uint32_t& next) {
    int sel = -1, sel2 = -1;
    unsigned sel_mask = 0, sel2_mask = 0;
#pragma unroll
    for (int r = 0; r < RX; ++r) {
        const bool open = beam[r] != kEmptyKey && (beam[r] & 1ull) == 0;
        const unsigned m = __ballot_sync(kFull, open);
        if (sel >= 0 && sel2 < 0 && m != 0) { sel2 = r; sel2_mask = m; }
        if (sel < 0 && m != 0) { sel = r; sel_mask = m; }
    }
    if (sel < 0) return false;
    const int src = __ffs(sel_mask) - 1;
    const unsigned rest = sel_mask & (sel_mask - 1u);
    int nreg = -1, nsrc = 0;
    if (rest != 0) { nreg = sel; nsrc = __ffs(rest) - 1; }
    else if (sel2 >= 0) { nreg = sel2; nsrc = __ffs(sel2_mask) - 1; }
    uint32_t mine = 0, mine2 = 0;
#pragma unroll
    for (int r = 0; r < RX; ++r) {
        if (r == sel) mine = static_cast<uint32_t>(beam[r]) >> 1;
        if (r == nreg) mine2 = static_cast<uint32_t>(beam[r]) >> 1;
    }
    node = __shfl_sync(kFull, mine, src);
    next = kNoNode;
    if (nreg >= 0) next = __shfl_sync(kFull, mine2, nsrc);
    if (static_cast<int>(lane) == src) {
#pragma unroll
        for (int r = 0; r < RX; ++r)
            if (r == sel) beam[r] |= 1ull;
    }
    return true;
}

// ------------------------------------------------------------ filters

// Exact visited set: linear probing on a power-of-two table of node ids
// (0xffffffff = empty).  Returns 1 when the key was inserted, 0 when it was
// already present.
__device__ __forceinline__ uint32_t hash_slot(uint32_t key, uint32_t shift) {
    return (key * 0x9E3779B1u) >> shift;
}

__device__ __forceinline__ int hash_insert(uint32_t* tab, uint32_t mask, uint32_t shift,
                                           uint32_t key, unsigned& err) {
    uint32_t h = hash_slot(key, shift);
    for (uint32_t i = 0; i <= mask; ++i) {
        // plain read first: a key already present (the common case for
        // neighbours of neighbours) or an occupied slot needs no atomic
        uint32_t v = tab[h];
        if (v == kNoNode) {
            v = atomicCAS(&tab[h], kNoNode, key);
            if (v == kNoNode) return 1;
        }
        if (v == key) return 0;
        h = (h + 1) & mask;
    }
    err |= 1u;   // table full: cannot happen with the host's load bound
    return 1;
}

__device__ __forceinline__ bool hash_contains(const uint32_t* tab, uint32_t mask, uint32_t shift,
                                              uint32_t key) {
    uint32_t h = hash_slot(key, shift);
    for (uint32_t i = 0; i <= mask; ++i) {
        const uint32_t v = tab[h];
        if (v == key) return true;
        if (v == kNoNode) return false;
        h = (h + 1) & mask;
    }
    return false;
}

// Bloom filter with the three hashes of include/filter_bloom.cuh:25-38.
__device__ __forceinline__ void bloom_hashes(uint32_t key, uint32_t mask, uint32_t (&h)[3]) {
    uint32_t a = key;
    a ^= a >> 16; a *= 0x45d9f3bu; a ^= a >> 16;
    uint32_t b = key * 0x9e3779b9u;
    b ^= b >> 16; b *= 0x45d9f3bu; b ^= b >> 16;
    uint32_t c = key * 0x517cc1b7u;
    c ^= c >> 16; c *= 0x45d9f3bu; c ^= c >> 16;
    h[0] = a & mask; h[1] = b & mask; h[2] = c & mask;
}

__device__ __forceinline__ bool bloom_test(const uint32_t* w, uint32_t mask, uint32_t key) {
    uint32_t h[3];
    bloom_hashes(key, mask, h);
    return ((w[h[0] >> 5] >> (h[0] & 31)) & (w[h[1] >> 5] >> (h[1] & 31)) &
            (w[h[2] >> 5] >> (h[2] & 31)) & 1u) != 0;
}

__device__ __forceinline__ void bloom_set(uint32_t* w, uint32_t mask, uint32_t key) {
    uint32_t h[3];
    bloom_hashes(key, mask, h);
    atomicOr(&w[h[0] >> 5], 1u << (h[0] & 31));
    atomicOr(&w[h[1] >> 5], 1u << (h[1] & 31));
    atomicOr(&w[h[2] >> 5], 1u << (h[2] & 31));
}

// ------------------------------------------------------------ memory ops

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
}

__device__ __forceinline__ float4 ldg_stream4(const float* p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];\n"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t ldg_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.global.nc.u32 %0, [%1];\n" : "=r"(v) : "l"(p));
    return v;
}

// ------------------------------------------------------------ distances

// Reference order (include/cpu_search_base.hpp:29-37): sum += diff*diff for
// d = 0..dim-1, every operation rounded on its own (no FMA contraction).
__device__ __forceinline__ float l2_seq(const float* __restrict__ q, const float* __restrict__ x,
                                        uint32_t dim) {
    float s = 0.0f;
    uint32_t d = 0;
    for (; d + 8 <= dim; d += 8) {
        const float4 a0 = *reinterpret_cast<const float4*>(q + d);
        const float4 b0 = *reinterpret_cast<const float4*>(x + d);
        const float4 a1 = *reinterpret_cast<const float4*>(q + d + 4);
        const float4 b1 = *reinterpret_cast<const float4*>(x + d + 4);
        float t;
        t = __fsub_rn(a0.x, b0.x); s = __fadd_rn(s, __fmul_rn(t, t));
        t = __fsub_rn(a0.y, b0.y); s = __fadd_rn(s, __fmul_rn(t, t));
        t = __fsub_rn(a0.z, b0.z); s = __fadd_rn(s, __fmul_rn(t, t));
        t = __fsub_rn(a0.w, b0.w); s = __fadd_rn(s, __fmul_rn(t, t));
        t = __fsub_rn(a1.x, b1.x); s = __fadd_rn(s, __fmul_rn(t, t));
        t = __fsub_rn(a1.y, b1.y); s = __fadd_rn(s, __fmul_rn(t, t));
        t = __fsub_rn(a1.z, b1.z); s = __fadd_rn(s, __fmul_rn(t, t));
        t = __fsub_rn(a1.w, b1.w); s = __fadd_rn(s, __fmul_rn(t, t));
    }
    for (; d < dim; ++d) {
        const float t = __fsub_rn(q[d], x[d]);
        s = __fadd_rn(s, __fmul_rn(t, t));
    }
    return s;
}

}  // namespace dev
}  // namespace bsb
