// bs_merge.cu -- merge of per-shard result lists for an index split into
// shards (one per GPU, each with its own graph over its own rows).
//
// Every query is searched on every shard; each shard returns its K best
// (distance, local id) entries in ascending (distance, id) order, and the
// caller gathers them (NCCL all-gather over NVLink) into
//     dists[s][q][K], ids[s][q][K]    s < shards.
// The merged answer is the K_out smallest (distance, global id) entries over
// all shards, global id = local id + the shard's id offset, with
// 0xffffffff / FLT_MAX past the end -- the order the reference's result lists
// use (include/cpu_search_base.hpp:47-51,75-81).
//
// One warp per query: lane s holds the head of shard s's list; each output
// position is the warp minimum of the heads, after which the winning lane
// advances.  The lists are already sorted, so K_out rounds suffice.
#include <cfloat>
#include <cstdint>

#include "bs_device.cuh"
#include "bs_internal.h"

namespace bsb {

using namespace dev;

namespace {

__device__ __forceinline__ uint64_t shard_key(const MergeArgs& a, uint32_t s, uint32_t q, uint32_t pos) {
    if (pos >= a.K) return kEmptyKey;
    const size_t at = (static_cast<size_t>(s) * a.nq + q) * a.K + pos;
    const uint32_t id = a.ids[at];
    if (id == kNoNode) return kEmptyKey;
    // (ordered distance, global id): 32-bit global ids, no expanded bit here
    return (static_cast<uint64_t>(f2ord(a.dists[at])) << 32) | (id + a.offsets[s]);
}

__global__ void k_merge_shards(const MergeArgs a) {
    const unsigned lane = threadIdx.x & 31u;
    const uint64_t warp = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = (static_cast<uint64_t>(gridDim.x) * blockDim.x) >> 5;
    for (uint64_t q = warp; q < a.nq; q += nwarps) {
        const uint32_t qi = static_cast<uint32_t>(q);
        uint32_t pos = 0;
        uint64_t head = lane < a.shards ? shard_key(a, lane, qi, 0) : kEmptyKey;
        uint32_t* oid = a.out_ids + q * a.K_out;
        float* odist = a.out_dists ? a.out_dists + q * a.K_out : nullptr;
        for (uint32_t k = 0; k < a.K_out; ++k) {
            uint64_t m = head;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = kmin(m, __shfl_xor_sync(kFull, m, o));
            if (lane == 0) {
                oid[k] = m == kEmptyKey ? kNoNode : static_cast<uint32_t>(m);
                if (odist) odist[k] = m == kEmptyKey ? FLT_MAX : key_dist(m);
            }
            // keys are unique (shards hold disjoint ids), so one lane wins
            if (m != kEmptyKey && head == m) head = shard_key(a, lane, qi, ++pos);
        }
    }
}

}  // namespace

cudaError_t launch_merge_shards(const MergeArgs& a, int num_sms, cudaStream_t stream) {
    if (a.nq == 0 || a.K_out == 0) return cudaSuccess;
    const uint64_t blocks_needed = (static_cast<uint64_t>(a.nq) + 7) / 8;   // 8 warps per block
    const uint64_t cap = static_cast<uint64_t>(num_sms) * 8;
    const unsigned blocks = static_cast<unsigned>(blocks_needed < cap ? blocks_needed : cap);
    k_merge_shards<<<blocks, 256, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace bsb
