// Push of a finished block of C into the same rows of every peer's C, over NVLink,
// by plain 16-byte loads from this GPU's memory and 16-byte stores into the peers'
// memory (addresses of peer buffers mapped into this process, e.g. symmetric
// memory).  No TMA and no multicast: every load reads this GPU's own memory.
//
// The row-sharded multi-GPU GEMM all-gathers C: each rank's rows must reach every
// other rank.  Copy engines (one cudaMemcpyAsync per peer) take no SM but at 8
// GPUs moved only about 400 GB/s into each GPU when every rank pushed to all its
// peers at once; this kernel runs on the SMs the GEMM leaves free
// (matmul_set_sm_limit) and sends each 16-byte vector to the peers in the order
// rank + 1, rank + 2, ... starting at a CTA-dependent peer, so that the stores of
// the CTAs spread over all peers at any moment.
#pragma once

#include <cstddef>
#include <cstdint>

#include "ptx.cuh"

namespace b200 {

constexpr int PP_MAX_PEERS = 7;
constexpr int PP_THREADS = 512;

struct PeerPushJob {
    const float4 *src;                  // this GPU's block (16-byte aligned)
    float4 *dst[PP_MAX_PEERS];          // the same block in each peer's buffer
    int peers;
    long long count;                    // 16-byte vectors in the block
};

__global__ void __launch_bounds__(PP_THREADS) peer_push_kernel(const PeerPushJob job)
{
    const long long stride = static_cast<long long>(gridDim.x) * PP_THREADS;
    const int first = static_cast<int>(blockIdx.x) % (job.peers > 0 ? job.peers : 1);
    for (long long i = static_cast<long long>(blockIdx.x) * PP_THREADS + threadIdx.x; i < job.count; i += stride) {
        const float4 v = job.src[i];
        for (int j = 0; j < job.peers; ++j) {
            int p = first + j;
            if (p >= job.peers)
                p -= job.peers;
            job.dst[p][i] = v;
        }
    }
    // The peers read these rows after a collective that follows this kernel on the
    // stream; make the stores visible beyond this GPU before the kernel ends.
    __threadfence_system();
}

} // namespace b200
