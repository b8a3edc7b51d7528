// Peer-memory all-gather between the GPUs of one box, for the vocab-sharded sampler's phase
// exchange (the rank-major all-gather of vocab_shard.py's protocol) without a collective library.
//
// Every rank owns one exchange buffer, allocated here and mapped into every other rank's process
// (CUDA IPC): 512 bytes of arrival words (uint64, one per source rank) and then the gathered
// region, world slots of the phase's record bytes.  One launch per phase: the CTAs copy this
// rank's records straight into slot `rank` of every peer's buffer with plain stores over NVLink,
// the last CTA to finish makes those stores visible system-wide, then stores the phase's sequence
// number into arrival word `rank` of every peer, and waits (bounded) until every peer's word in
// its own buffer has reached the sequence number.  The next kernel on the stream then reads the
// gathered region.  No TMA and no cluster copies touch peer memory, and no NVLink multicast
// object is involved.

#include <cstring>

#include "enx_internal.cuh"

namespace enx {

constexpr uint32_t kPeerHeader = 512;  // arrival words (64 x u64) before the gathered region
constexpr uint32_t kPeerMaxWorld = 8;
constexpr uint32_t kPeerCtas = 16;
constexpr uint32_t kPeerSpin = 1u << 24;

__device__ uint32_t g_peer_done;  // CTAs of the current launch that finished their copies

__global__ void __launch_bounds__(256) k_peer_allgather(const uint4* __restrict__ send, uint32_t vecs,
                                                        const unsigned long long* __restrict__ peers, uint32_t world,
                                                        uint32_t rank, unsigned long long seq, uint32_t* err) {
    __shared__ bool last;
    // my records -> slot `rank` of every buffer (my own included), 16 bytes per store
    for (uint32_t p = 0; p < world; ++p) {
        uint4* dst = reinterpret_cast<uint4*>(peers[p] + kPeerHeader) + (size_t)rank * vecs;
        for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < vecs; i += gridDim.x * blockDim.x) dst[i] = send[i];
    }
    __threadfence_system();  // this thread's stores, visible to every GPU before the count below
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(&g_peer_done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    if (threadIdx.x == 0) g_peer_done = 0;  // the next launch starts from zero (stream order)
    __threadfence_system();
    if (threadIdx.x < world) {  // arrival word `rank` of every buffer
        unsigned long long* w = reinterpret_cast<unsigned long long*>(peers[threadIdx.x]) + rank;
        asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(w), "l"(seq) : "memory");
    }
    if (threadIdx.x < world) {  // wait for every rank's word in my buffer (bounded)
        const unsigned long long* w = reinterpret_cast<const unsigned long long*>(peers[rank]) + threadIdx.x;
        for (uint32_t it = 0;; ++it) {
            unsigned long long v;
            asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(w) : "memory");
            if (v >= seq) break;
            if (it >= kPeerSpin) {
                atomicMax(err, 4u);
                break;
            }
        }
    }
    __syncthreads();
}

}  // namespace enx

using namespace enx;

#define CHECK_ARG(cond, msg)                                   \
    do {                                                       \
        if (!(cond)) return ::enx::fail(ENX_ERR_INVALID, msg); \
    } while (0)

extern "C" enx_status enx_peer_alloc(size_t bytes, void** ptr, uint8_t* handle) {
    CHECK_ARG(ptr && handle, "enx_peer_alloc: null pointer");
    void* p = nullptr;
    ENX_CUDA(cudaMalloc(&p, bytes + kPeerHeader));
    ENX_CUDA(cudaMemset(p, 0, bytes + kPeerHeader));
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        ENX_CUDA(e);
    }
    std::memcpy(handle, &h, sizeof(h));
    *ptr = p;
    return ENX_OK;
}

extern "C" enx_status enx_peer_open(const uint8_t* handle, void** ptr) {
    CHECK_ARG(ptr && handle, "enx_peer_open: null pointer");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    ENX_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return ENX_OK;
}

extern "C" enx_status enx_peer_close(void* ptr, int opened) {
    if (!ptr) return ENX_OK;
    ENX_CUDA(opened ? cudaIpcCloseMemHandle(ptr) : cudaFree(ptr));
    return ENX_OK;
}

extern "C" enx_status enx_peer_allgather(const void* send, size_t bytes, const unsigned long long* peers, uint32_t world,
                                         uint32_t rank, unsigned long long seq, uint32_t* err, void* stream) {
    CHECK_ARG(send && peers && err, "enx_peer_allgather: null pointer");
    CHECK_ARG(world >= 1 && world <= kPeerMaxWorld && rank < world, "enx_peer_allgather: world of 1-8 ranks");
    CHECK_ARG(bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(send) & 15) == 0,
              "enx_peer_allgather: records must be 16-byte aligned multiples of 16 bytes");
    const uint32_t vecs = (uint32_t)(bytes / 16);
    k_peer_allgather<<<kPeerCtas, 256, 0, as_stream(stream)>>>(reinterpret_cast<const uint4*>(send), vecs, peers, world,
                                                              rank, seq, err);
    ENX_CUDA(cudaGetLastError());
    return ENX_OK;
}
