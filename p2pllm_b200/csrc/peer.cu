// A barrier between the GPUs of one node over NVLink peer memory, for the collectives fused into the kernels (the
// GEMM epilogue that stores its rows of y into every rank's y, the hop that stores a member's part into the next
// step's ranks). Each rank owns a flag array with one 32-bit slot per rank, in memory every rank can write (CUDA IPC
// or symmetric allocations). p2p_peer_barrier(epoch) on rank `me`:
//
//   thread r != me:  __threadfence_system(), then st.release.sys flags[r][me] = epoch  (rank r learns: me is done)
//   thread r != me:  spin on ld.acquire.sys flags[me][r] until it equals epoch          (me learns: r is done)
//
// Everything this rank's stream ran before the barrier -- the stores of earlier kernels into peers' memory included
// -- is visible to a peer once that peer's wait for this rank ends. The spin is bounded (timeout of %globaltimer):
// past it the kernel records the rank it gave up on and returns, so a rank that died or never came ends the wait with
// an error status (p2p_peer_status) instead of a hang. Epochs grow by one a barrier; flags are never cleared.
//
// Two ranks' barriers wait on each other: they must run on different GPUs (one process per GPU), never as two
// launches on one GPU.
#include "common.cuh"

namespace p2p {
namespace {

constexpr int kMaxRanks = 8;

__device__ int g_peer_error;     // 1 + the rank a wait gave up on, since the last reset (0: none)

struct PeerFlags {
    uint32_t* flags[kMaxRanks];  // rank r's flag array (kMaxRanks slots), as this GPU addresses it
};

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__global__ void peer_barrier_kernel(PeerFlags f, int n, int me, uint32_t epoch, uint64_t timeout_ns) {
    const int r = threadIdx.x;
    if (r >= n || r == me) return;
    __threadfence_system();
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f.flags[r] + me), "r"(epoch) : "memory");
    const uint32_t* mine = f.flags[me] + r;
    const uint64_t t0 = now_ns();
    for (;;) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
        if (v == epoch) break;
        if (now_ns() - t0 > timeout_ns) {
            atomicCAS(&g_peer_error, 0, 1 + r);
            break;
        }
        __nanosleep(200);
    }
}

struct PushDst {
    char* y[kMaxRanks];   // the other ranks' y buffers, as this GPU addresses them
    int n;
};

// Columns [col0, col0 + width) of tokens rows of y (row stride ld elements) from this rank's buffer to every other
// rank's: 16-byte loads and stores, the grid striding over (row, 16-byte chunk) pairs, each chunk to every peer.
__global__ void __launch_bounds__(256) peer_push_kernel(const char* __restrict__ src, const __grid_constant__ PushDst dst,
                                                        int64_t tokens, int64_t row_bytes, int64_t ld_bytes,
                                                        int64_t col0_bytes) {
    const int64_t chunks = row_bytes / 16;
    const int64_t total = tokens * chunks;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / chunks, c = i - t * chunks;
        const int64_t at = t * ld_bytes + col0_bytes + c * 16;
        const uint4 v = *reinterpret_cast<const uint4*>(src + at);
        for (int k = 0; k < dst.n; ++k) *reinterpret_cast<uint4*>(dst.y[k] + at) = v;
    }
}

}  // namespace
}  // namespace p2p

using namespace p2p;

extern "C" int p2p_peer_push(const void* y, void* const* peers, int n_peers, int64_t tokens, int64_t col0,
                             int64_t width, int64_t ldy, int dtype, void* stream) {
    P2P_REQUIRE(y && peers && n_peers >= 0 && n_peers < kMaxRanks, "p2p_peer_push: 0 to %d peers", kMaxRanks - 1);
    P2P_REQUIRE(dtype_ok(dtype) && tokens >= 0 && col0 >= 0 && width >= 0 && col0 + width <= ldy,
                "p2p_peer_push: columns %lld.. (%lld) of rows of %lld", (long long)col0, (long long)width,
                (long long)ldy);
    const int64_t es = dtype_size(dtype);
    P2P_REQUIRE((col0 * es) % 16 == 0 && (width * es) % 16 == 0 && (ldy * es) % 16 == 0 && aligned16(y),
                "p2p_peer_push: the columns, the row stride and y must be 16-byte aligned");
    if (tokens == 0 || width == 0 || n_peers == 0) return P2P_OK;
    PushDst d = {};
    d.n = n_peers;
    for (int k = 0; k < n_peers; ++k) {
        P2P_REQUIRE(peers[k] && aligned16(peers[k]), "p2p_peer_push: peer buffer %d is null or misaligned", k);
        d.y[k] = reinterpret_cast<char*>(peers[k]);
    }
    const int64_t total = tokens * (width * es / 16);
    const int64_t want = (total + 255) / 256;
    const int64_t cap = (int64_t)sm_count() * 4;
    peer_push_kernel<<<(unsigned)(want < cap ? want : cap), 256, 0, as_stream(stream)>>>(
        reinterpret_cast<const char*>(y), d, tokens, width * es, ldy * es, col0 * es);
    return launch_status("p2p_peer_push");
}

extern "C" int p2p_peer_barrier(void* const* flags, int n_ranks, int me, uint32_t epoch, int64_t timeout_us,
                                void* stream) {
    P2P_REQUIRE(flags && n_ranks >= 1 && n_ranks <= kMaxRanks && me >= 0 && me < n_ranks,
                "p2p_peer_barrier: %d ranks, rank %d", n_ranks, me);
    P2P_REQUIRE(timeout_us >= 1000 && timeout_us <= 60000000, "p2p_peer_barrier: a time limit of 1 ms to 60 s");
    if (n_ranks == 1) return P2P_OK;
    PeerFlags f = {};
    for (int r = 0; r < n_ranks; ++r) {
        P2P_REQUIRE(flags[r] && (reinterpret_cast<uintptr_t>(flags[r]) & 3) == 0, "p2p_peer_barrier: flags of rank %d",
                    r);
        f.flags[r] = reinterpret_cast<uint32_t*>(flags[r]);
    }
    peer_barrier_kernel<<<1, 32, 0, as_stream(stream)>>>(f, n_ranks, me, epoch, (uint64_t)timeout_us * 1000ull);
    return launch_status("p2p_peer_barrier");
}

extern "C" int p2p_peer_status(int reset, void* stream) {
    cudaStream_t st = as_stream(stream);
    int v = 0;
    if (cudaMemcpyFromSymbolAsync(&v, g_peer_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return fail(P2P_ECUDA, "p2p_peer_status: %s", cudaGetErrorString(cudaGetLastError()));
    if (reset && v) {
        const int zero = 0;
        cudaMemcpyToSymbolAsync(g_peer_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
        cudaStreamSynchronize(st);
    }
    if (v) return fail(P2P_ECUDA, "p2p_peer_barrier: the wait for rank %d timed out", v - 1);
    return P2P_OK;
}
