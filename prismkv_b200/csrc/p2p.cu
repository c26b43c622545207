// All-gather of a small fixed-size device buffer between the ranks of one
// node over NVLink peer memory: the exchange step of the sequence-sharded
// decode (the routing picks and the attention's (m, l, o) partials), done
// with plain peer stores and one flag per (parity, rank) instead of a
// library collective.
//
// Each rank owns an exchange region in its own device memory, opened by
// every other rank through a CUDA IPC handle:
//   [0, 256)    flags[2][P] uint32: the epoch of rank q's last put into
//               parity p's slot (written by rank q over NVLink)
//   [256, 264)  ctr (uint32, this rank's last completed epoch), arrivals
//   [512, ...)  recv[2][P][slot]: rank q's buffer for epochs of parity p
// One launch of p2p_allgather_kernel (P CTAs) is one epoch e = ctr + 1 on
// every rank: CTA q stores this rank's buffer into rank q's recv[e & 1][me]
// (every thread fences its stores at system scope), publishes it with a
// release store of e into rank q's flags[e & 1][me], waits -- bounded -- for
// rank q's acquire-visible flag in its own region, and copies recv[e & 1][q]
// to out[q].  The last CTA to finish advances ctr.
//
// Two parity slots suffice: rank a writes parity (e & 1) of rank b again at
// epoch e + 2, which a starts only after its epoch e + 1 waited for b's put
// of e + 1, which b issues only after its epoch e finished reading.  Every
// rank runs the same sequence of epochs (the same calls, eager or replayed
// in a CUDA graph), so the epochs agree without any host exchange.
//
// A wait gives up after max_spins polls (a sleep of ~64 ns each), sets
// PK_STATUS_EXCHANGE_TIMEOUT in the caller's status word and lets the CTA
// finish; the host raises on it.  Ranks are separate GPUs: the waits are
// never between launches on one device.
#include <cstring>

#include "common.cuh"

namespace pk {

constexpr int kP2PMax = 8;
constexpr int kP2PHeader = 512;
constexpr int kP2PThreads = 512;

struct PeerBases {
    uint64_t b[kP2PMax];
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__global__ void __launch_bounds__(kP2PThreads)
p2p_allgather_kernel(const uint4* __restrict__ src, int64_t n16, int64_t slot, int me, int P, PeerBases peers,
                     uint8_t* __restrict__ local, uint4* __restrict__ out, int* __restrict__ status,
                     long long max_spins) {
    const int q = blockIdx.x, tid = threadIdx.x;
    __shared__ uint32_t epoch_s;
    uint32_t* lflags = reinterpret_cast<uint32_t*>(local);
    uint32_t* lctr = reinterpret_cast<uint32_t*>(local + 256);
    uint32_t* larrive = lctr + 1;
    if (tid == 0) epoch_s = *reinterpret_cast<volatile uint32_t*>(lctr) + 1u;
    __syncthreads();
    const uint32_t e = epoch_s, par = e & 1u;
    // 1. This rank's buffer into rank q's slot [par][me].
    uint8_t* qbase = reinterpret_cast<uint8_t*>(peers.b[q]);
    uint4* dq = reinterpret_cast<uint4*>(qbase + kP2PHeader + ((int64_t)par * P + me) * slot);
    for (int64_t i = tid; i < n16; i += kP2PThreads) dq[i] = src[i];
    __threadfence_system();
    __syncthreads();
    if (tid == 0) {
        st_release_sys(reinterpret_cast<uint32_t*>(qbase) + par * P + me, e);
        // 2. Rank q's buffer in this rank's slot [par][q].
        const uint32_t* f = lflags + par * P + q;
        long long it = 0;
        while (ld_acquire_sys(f) != e) {
            if (++it >= max_spins) {
                atomicOr(status, PK_STATUS_EXCHANGE_TIMEOUT);
                break;
            }
            __nanosleep(64);
        }
    }
    __syncthreads();
    // 3. Copy it out (L2 reads: the data arrived over NVLink).
    const uint4* sq = reinterpret_cast<const uint4*>(local + kP2PHeader + ((int64_t)par * P + q) * slot);
    uint4* oq = out + (int64_t)q * n16;
    for (int64_t i = tid; i < n16; i += kP2PThreads) oq[i] = __ldcg(sq + i);
    // 4. The last CTA advances the epoch (read by the next launch).
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(larrive, 1u) == (uint32_t)(P - 1)) {
            *reinterpret_cast<volatile uint32_t*>(larrive) = 0u;
            *reinterpret_cast<volatile uint32_t*>(lctr) = e;
        }
    }
}

}  // namespace pk

using namespace pk;

static int64_t p2p_slot(int64_t bytes) { return (bytes + 255) / 256 * 256; }

extern "C" size_t pk_p2p_region_bytes(int P, int64_t bytes) {
    if (P < 1 || P > kP2PMax || bytes < 0) return 0;
    return (size_t)kP2PHeader + (size_t)2 * P * p2p_slot(bytes);
}

extern "C" int pk_p2p_alloc(uint64_t bytes, uint64_t ptr_out) {
    if (!bytes || !ptr_out) return PK_ERR_ARG;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return (int)e;
    e = cudaMemset(p, 0, bytes);
    if (e != cudaSuccess) {
        cudaFree(p);
        return (int)e;
    }
    *reinterpret_cast<uint64_t*>(ptr_out) = (uint64_t)p;
    return PK_OK;
}

extern "C" int pk_p2p_free(uint64_t ptr) {
    if (!ptr) return PK_ERR_ARG;
    return (int)cudaFree((void*)ptr);
}

extern "C" int pk_p2p_handle(uint64_t ptr, uint64_t handle_out) {
    if (!ptr || !handle_out) return PK_ERR_ARG;
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, (void*)ptr);
    if (e != cudaSuccess) return (int)e;
    memcpy((void*)handle_out, &h, sizeof(h));
    return PK_OK;
}

extern "C" int pk_p2p_open(uint64_t handle, uint64_t ptr_out) {
    if (!handle || !ptr_out) return PK_ERR_ARG;
    cudaIpcMemHandle_t h;
    memcpy(&h, (const void*)handle, sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return (int)e;
    *reinterpret_cast<uint64_t*>(ptr_out) = (uint64_t)p;
    return PK_OK;
}

extern "C" int pk_p2p_close(uint64_t ptr) {
    if (!ptr) return PK_ERR_ARG;
    return (int)cudaIpcCloseMemHandle((void*)ptr);
}

extern "C" int pk_p2p_allgather(uint64_t src, int64_t bytes, int rank, int P, uint64_t peer_bases,
                                uint64_t local_base, uint64_t out, uint64_t status, int64_t max_spins,
                                uint64_t stream) {
    if (P < 1 || P > kP2PMax || rank < 0 || rank >= P || bytes <= 0 || bytes % 16 || max_spins < 1)
        return PK_ERR_ARG;
    if (!src || !peer_bases || !local_base || !out || !status || (src | out | local_base) % 16) return PK_ERR_ARG;
    PeerBases pb = {};
    const uint64_t* hb = reinterpret_cast<const uint64_t*>(peer_bases);
    for (int q = 0; q < P; ++q) {
        if (!hb[q] || hb[q] % 256) return PK_ERR_ARG;
        pb.b[q] = hb[q];
    }
    if (pb.b[rank] != local_base) return PK_ERR_ARG;
    p2p_allgather_kernel<<<P, kP2PThreads, 0, (cudaStream_t)stream>>>(
        (const uint4*)src, bytes / 16, p2p_slot(bytes), rank, P, pb, (uint8_t*)local_base, (uint4*)out,
        (int*)status, (long long)max_spins);
    PK_CHECK_LAUNCH();
    return PK_OK;
}
