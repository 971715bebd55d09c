// peer.cu -- the sequence-sharded exchange over NVLink peer memory (sm_100a).
//
// imi_peer_allgather replaces an NCCL all-gather of one equally sized block
// per rank (the candidate records, then the attention partials of every
// decode layer).  Every rank's source block lives in memory that every peer
// has mapped (symmetric memory); each rank also owns `world` flag words that
// the peers write.  One launch on every rank:
//   * every CTA first publishes this rank's epoch e into flag word `rank` of
//     every peer (a release store over NVLink) -- this rank's block, written
//     by earlier kernels in the stream, is ready;
//   * CTA (s, c) waits, bounded, until its own flag word s reaches e (peer s
//     is ready), then copies chunk c of peer s's block into dst with 16-byte
//     loads straight from the peer's memory;
//   * the last CTA to finish (a ticket) advances the local epoch.
// Every CTA signals, so no CTA depends on another being resident.  A wait
// that gives up sets bit 0 of `status` and skips its copy.
//
// Reuse: the two exchanges of a layer alternate, and each starts only after
// every peer has started it, which is after that peer finished the previous
// one -- so once a rank passes an exchange, no peer still reads the block of
// the other kind, and it may be rewritten.
#include "common.cuh"
#include "imi_internal.h"

namespace imi {

constexpr int PG_THREADS = 256;
constexpr int PG_UNROLL = 8;              // 16-byte loads in flight per thread
constexpr long long PG_CHUNK = (long long)PG_THREADS * PG_UNROLL * 16;  // bytes per CTA (32 KB)
constexpr int PG_WAIT_LIMIT = 1 << 24;     // polls (about 100 ns each) before giving up

__global__ void __launch_bounds__(PG_THREADS) imi_peer_allgather_kernel(const __grid_constant__ PeerGatherArgs a) {
    const int s = blockIdx.x;  // source rank
    const unsigned e = *a.epoch + 1u;
    __shared__ int ok;
    if (threadIdx.x < a.world) {  // publish: this rank's block is ready for epoch e
        unsigned* f = a.flag_peers[threadIdx.x] + a.rank;
        __threadfence_system();
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(e) : "memory");
    }
    if (threadIdx.x == 0) {
        const unsigned* mine = a.flag_peers[a.rank] + s;
        int good = 0;
        for (int i = 0; i < PG_WAIT_LIMIT; ++i) {
            unsigned v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
            if ((int)(v - e) >= 0) {
                good = 1;
                break;
            }
            __nanosleep(64);
        }
        ok = good;
        if (!good && a.status) atomicOr(a.status, 1);
    }
    __syncthreads();
    if (ok) {
        const long long c0 = (long long)blockIdx.y * PG_CHUNK;
        const long long c1 = min((long long)a.bytes, c0 + PG_CHUNK);
        const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const unsigned char*>(a.src_peers[s]) + c0);
        uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(a.dst) + (long long)s * (long long)a.bytes + c0);
        const int n16 = (int)((c1 - c0) / 16);
        uint4 v[PG_UNROLL];  // every load in flight before the first store
#pragma unroll
        for (int u = 0; u < PG_UNROLL; ++u) {
            const int i = threadIdx.x + u * PG_THREADS;
            if (i < n16) v[u] = __ldcv(src + i);
        }
#pragma unroll
        for (int u = 0; u < PG_UNROLL; ++u) {
            const int i = threadIdx.x + u * PG_THREADS;
            if (i < n16) dst[i] = v[u];
        }
    }
    // the last CTA advances the epoch for the next launch
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned total = gridDim.x * gridDim.y;
        if (atomicAdd(a.ticket, 1u) == total - 1u) {
            *a.ticket = 0u;
            *a.epoch = e;
        }
    }
}

long long peer_gather_chunks(long long bytes) { return (bytes + PG_CHUNK - 1) / PG_CHUNK; }

cudaError_t launch_peer_allgather(const PeerGatherArgs& a, cudaStream_t st) {
    imi_peer_allgather_kernel<<<dim3(a.world, (unsigned)peer_gather_chunks(a.bytes)), PG_THREADS, 0, st>>>(a);
    return cudaGetLastError();
}

}  // namespace imi
