// The hidden-state hop of a layer-parallel plan over NVLink peer memory, with the sender's part and the receiver's sum
// fused into it (p2p/route.py:1254-1274 makes a member's part, 800-810 sends it to every rank of the next step,
// 825-831 sums the parts a rank receives in fp32 in member order).
//
// Every rank owns an inbox in memory that every rank of the job addresses (a symmetric allocation):
//
//   [128, 256)   freed[n_ranks]    u32: + 1 for every receiver CTA that has consumed a pass of ours (index: receiver)
//   [256, ...)   slots[n_ranks][ring][slot_bytes]: the part of sender s for pass p sits in slot [s][p % ring], every
//                32 bits of it as one 64-bit word whose upper half is the flag p + 1
//
// p2p_hop_send (one launch on the sender): each CTA first waits until every destination has consumed pass
// p - ring of this sender (so the slot is free), then computes its share of the part -- a copy or fp32 sum of parts,
// a member's difference dtype(y - x), or the whole group combine of p2p/replica.py:81-85 -- and stores it straight
// into every destination's slot over NVLink as flagged words. No fence and no counter: a 64-bit word is written at
// once, so the receiver knows a word has arrived when it carries this pass's flag. p2p_hop_recv (one launch on the
// receiver): each thread polls its own words until they carry the flag (so the work starts as the data lands, word
// by word), adds the parts in fp32 in member order into `out` (rounded once, to the model dtype), and after a CTA
// barrier one thread frees the slots (adds 1 to every source's freed[me] with a release). Both kernels run
// hop_grid(n) CTAs, so a pass is freed at (p + 1) * grid; counters only grow (compared modulo 2^32). Slots take
// twice the part's bytes.
//
// Every wait is bounded (%globaltimer): past its limit the thread records the site and the rank it gave up on and
// returns without storing or signalling, so the peer's own wait runs out too and both hosts read an error from
// p2p_hop_status instead of a hang; every later hop on that GPU then returns at once until the status is reset.
// A sender and its receiver must run on different GPUs (one process per GPU), or, on one GPU, in stream order with
// the send first -- a wait that depends on a later launch on the same GPU is never made.
#include "elementwise.cuh"

namespace p2p {
namespace {

constexpr int kHopBlock = 256;
constexpr int kHopRanks = 8;
constexpr int kFreedAt = 128;
constexpr int kSlotsAt = 256;
constexpr int kMaxHopCtas = 128;

__device__ int g_hop_error;  // 0, or 1 + the site of the first wait that gave up: 1 send (free slot), 2 recv (parts)
__device__ int g_hop_rank;   // the rank that wait was for

struct HopPeers {
    char* inbox[kHopRanks];  // the inboxes of the listed ranks, as this GPU addresses them
    int rank[kHopRanks];     // their ranks, in the order given (member order for sources)
    int n;
};

__device__ __forceinline__ uint64_t hop_now() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Spins until *p has reached `target` (modulo 2^32), at most limit_ns; false if it gave up.
__device__ bool wait_count(const uint32_t* p, uint32_t target, uint64_t limit_ns) {
    const uint64_t t0 = hop_now();
    for (;;) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
        if ((int32_t)(v - target) >= 0) return true;
        if (hop_now() - t0 > limit_ns) return false;
        __nanosleep(32);
    }
}

__device__ __forceinline__ void signal(uint32_t* p) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(1u) : "memory");
}

// A wait on this GPU gave up since the last reset: later hops return at once (no stores, no signals) instead of each
// waiting out its own limit, until p2p_hop_status(reset) clears it.
__device__ __forceinline__ bool hop_failed() { return *reinterpret_cast<volatile int*>(&g_hop_error) != 0; }

__device__ __forceinline__ void gave_up(int site, int rank) {
    if (atomicCAS(&g_hop_error, 0, site) == 0) atomicExch(&g_hop_rank, rank);
}

template <typename T, int MODE>
__global__ void __launch_bounds__(kHopBlock) hop_send_kernel(const __grid_constant__ Parts parts,
                                                              const void* __restrict__ h,
                                                              const void* __restrict__ hc, int64_t n_vec,
                                                              const __grid_constant__ HopPeers dst,
                                                              const char* my_inbox, int me, uint32_t pass_arg,
                                                              const uint32_t* pass_at, int ring, int64_t slot_bytes,
                                                              uint64_t wait_ns) {
    constexpr int VEC = 16 / sizeof(T);
    const uint32_t pass = pass_at ? *pass_at : pass_arg;
    __shared__ int go;
    if (threadIdx.x == 0) {
        bool ok = !hop_failed();
        if (ok && pass >= (uint32_t)ring) {
            const uint32_t target = (pass - (uint32_t)ring + 1u) * gridDim.x;
            for (int d = 0; d < dst.n && ok; ++d) {
                ok = wait_count(reinterpret_cast<const uint32_t*>(my_inbox + kFreedAt) + dst.rank[d], target, wait_ns);
                if (!ok) gave_up(1, dst.rank[d]);
            }
        }
        go = ok;
    }
    __syncthreads();
    if (!go) return;
    const int64_t slot = kSlotsAt + ((int64_t)me * ring + (int64_t)(pass % (uint32_t)ring)) * slot_bytes;
    const uint64_t flag = (uint64_t)(pass + 1u) << 32;
    for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < n_vec; v += (int64_t)gridDim.x * blockDim.x) {
        float total[VEC];
        member_value<T, VEC, MODE>(parts, h, hc, v * VEC, total);
        const uint4 raw = pack_vec<T, VEC>(total);
        const uint64_t w0 = flag | raw.x, w1 = flag | raw.y, w2 = flag | raw.z, w3 = flag | raw.w;
        for (int d = 0; d < dst.n; ++d) {
            char* at = dst.inbox[d] + slot + v * 32;
            asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(at), "l"(w0), "l"(w1) : "memory");
            asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(at + 16), "l"(w2), "l"(w3) : "memory");
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(kHopBlock) hop_recv_kernel(const __grid_constant__ HopPeers src,
                                                              const char* my_inbox, int me, uint32_t pass_arg,
                                                              const uint32_t* pass_at, int ring, int64_t slot_bytes,
                                                              int64_t n_vec, void* __restrict__ out, uint64_t wait_ns) {
    constexpr int VEC = 16 / sizeof(T);
    const uint32_t pass = pass_at ? *pass_at : pass_arg;
    __shared__ int failed;
    if (threadIdx.x == 0) failed = hop_failed();
    __syncthreads();
    if (failed) return;
    const int64_t ring_at = (int64_t)(pass % (uint32_t)ring) * slot_bytes;
    const uint32_t want = pass + 1u;
    bool ok = true;
    for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < n_vec && ok; v += (int64_t)gridDim.x * blockDim.x) {
        float total[VEC];
        for (int s = 0; s < src.n && ok; ++s) {
            // four flagged words: each 64-bit word is written at once, so a word whose flag is this pass's carries
            // this pass's 32 bits of data
            const char* at = my_inbox + kSlotsAt + (int64_t)src.rank[s] * ring * slot_bytes + ring_at + v * 32;
            uint64_t w0, w1, w2, w3;
            uint64_t t0 = 0;
            for (;;) {
                asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(at) : "memory");
                asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(w2), "=l"(w3) : "l"(at + 16) : "memory");
                if ((uint32_t)(w0 >> 32) == want && (uint32_t)(w1 >> 32) == want && (uint32_t)(w2 >> 32) == want &&
                    (uint32_t)(w3 >> 32) == want)
                    break;
                const uint64_t now = hop_now();
                if (t0 == 0) t0 = now;
                if (now - t0 > wait_ns || hop_failed()) {
                    gave_up(2, src.rank[s]);
                    ok = false;
                    break;
                }
            }
            if (!ok) break;
            const uint4 raw = make_uint4((uint32_t)w0, (uint32_t)w1, (uint32_t)w2, (uint32_t)w3);
            const T* e = reinterpret_cast<const T*>(&raw);
            if (s == 0) {
#pragma unroll
                for (int q = 0; q < VEC; ++q) total[q] = to_f32(e[q]);
            } else {
#pragma unroll
                for (int q = 0; q < VEC; ++q) total[q] += to_f32(e[q]);
            }
        }
        if (ok) store_vec<T, VEC>(out, v * VEC, total);
    }
    if (!ok) atomicExch(&failed, 1);
    __syncthreads();                            // every read of the slots is done before the slots are freed
    if (threadIdx.x == 0 && !failed) {
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        for (int s = 0; s < src.n; ++s) signal(reinterpret_cast<uint32_t*>(src.inbox[s] + kFreedAt) + me);
    }
}

__global__ void hop_advance_kernel(uint32_t* counters, int n) {
    if ((int)threadIdx.x < n) counters[threadIdx.x] += 1u;
}

// A slot holds every 32 bits of a part as one 64-bit word with the pass's flag in its upper half.
int64_t slot_bytes_of(int64_t cap_elems, int dtype) { return (cap_elems * dtype_size(dtype) * 2 + 255) / 256 * 256; }

// CTAs of a hop over n elements, the same on both sides (a pass is freed at (p + 1) * grid): four 16-byte vectors a
// thread (one a thread, with four times the CTAs, measured 2.6 us slower one way at 174 KB).
int hop_grid(int64_t n_elem, int dtype) {
    const int64_t n_vec = n_elem * dtype_size(dtype) / 16;
    const int64_t g = (n_vec + kHopBlock * 4 - 1) / (kHopBlock * 4);
    return (int)(g < 1 ? 1 : g > kMaxHopCtas ? kMaxHopCtas : g);
}

int fill_peers(HopPeers& hp, void* const* inboxes, int n_ranks, const int* list, int n, const char* what) {
    if (!list || n < 1 || n > n_ranks) return fail(P2P_EINVAL, "p2p_hop_%s: 1 to %d ranks, got %d", what, n_ranks, n);
    hp.n = n;
    for (int k = 0; k < n; ++k) {
        const int r = list[k];
        if (r < 0 || r >= n_ranks) return fail(P2P_EINVAL, "p2p_hop_%s: rank %d of %d", what, r, n_ranks);
        for (int j = 0; j < k; ++j)
            if (list[j] == r) return fail(P2P_EINVAL, "p2p_hop_%s: rank %d listed twice", what, r);
        hp.rank[k] = r;
        hp.inbox[k] = reinterpret_cast<char*>(inboxes[r]);
    }
    return P2P_OK;
}

int check_common(void* const* inboxes, int n_ranks, int me, int ring, int64_t cap_elems, int dtype, int64_t n_elem,
                 int64_t wait_us, const char* what) {
    P2P_REQUIRE(inboxes && n_ranks >= 1 && n_ranks <= kHopRanks && me >= 0 && me < n_ranks,
                "p2p_hop_%s: %d ranks (1 to %d), rank %d", what, n_ranks, kHopRanks, me);
    P2P_REQUIRE(dtype_ok(dtype), "p2p_hop_%s: dtype %d", what, dtype);
    P2P_REQUIRE(ring >= 1 && ring <= 64, "p2p_hop_%s: a ring of 1 to 64 slots, got %d", what, ring);
    P2P_REQUIRE(n_elem >= 1 && n_elem <= cap_elems, "p2p_hop_%s: %lld elements, slots hold %lld", what,
                (long long)n_elem, (long long)cap_elems);
    P2P_REQUIRE((n_elem * dtype_size(dtype)) % 16 == 0, "p2p_hop_%s: the part must be a multiple of 16 bytes", what);
    P2P_REQUIRE(wait_us >= 1000 && wait_us <= 60000000, "p2p_hop_%s: a time limit of 1 ms to 60 s", what);
    for (int r = 0; r < n_ranks; ++r)
        P2P_REQUIRE(inboxes[r] && (reinterpret_cast<uintptr_t>(inboxes[r]) & 255) == 0,
                    "p2p_hop_%s: inbox of rank %d is null or not 256-byte aligned", what, r);
    return P2P_OK;
}

}  // namespace
}  // namespace p2p

using namespace p2p;

extern "C" size_t p2p_hop_inbox_bytes(int n_ranks, int64_t cap_elems, int dtype, int ring) {
    if (n_ranks < 1 || n_ranks > kHopRanks || cap_elems < 1 || !dtype_ok(dtype) || ring < 1 || ring > 64) return 0;
    return (size_t)kSlotsAt + (size_t)n_ranks * (size_t)ring * (size_t)slot_bytes_of(cap_elems, dtype);
}

extern "C" int p2p_hop_send(int mode, const void* const* parts, int n_parts, const void* h, const void* h_copy,
                            int dtype, int64_t n_elem, void* const* inboxes, int n_ranks, int me, const int* dsts,
                            int n_dst, uint32_t pass, const uint32_t* pass_at, int ring, int64_t cap_elems,
                            int64_t wait_us, void* stream) {
    if (int e = check_common(inboxes, n_ranks, me, ring, cap_elems, dtype, n_elem, wait_us, "send")) return e;
    HopPeers dst;
    if (int e = fill_peers(dst, inboxes, n_ranks, dsts, n_dst, "send")) return e;
    Parts p;
    if (int e = fill_parts(p, parts, n_parts)) return e;
    for (int k = 0; k < n_parts; ++k) P2P_REQUIRE(aligned16(parts[k]), "p2p_hop_send: part %d is not 16-byte aligned", k);
    switch (mode) {
        case P2P_PART_SUM: break;
        case P2P_PART_DIFF:
            P2P_REQUIRE(n_parts == 1 && h && aligned16(h), "p2p_hop_send: a difference takes one part and an aligned x");
            break;
        case P2P_PART_COMBINE:
            P2P_REQUIRE(n_parts >= 2 && h_copy && aligned16(h_copy) && (n_parts == 2 || (h && aligned16(h))),
                        "p2p_hop_send: a combine takes 2 or more parts, h_copy, and h beyond 2 members");
            break;
        default: return fail(P2P_EINVAL, "p2p_hop_send: mode %d (sum 0, difference 1, combine 2)", mode);
    }
    const int64_t n_vec = n_elem * dtype_size(dtype) / 16;
    const int64_t sb = slot_bytes_of(cap_elems, dtype);
    const uint64_t wait_ns = (uint64_t)wait_us * 1000ull;
    const int grid = hop_grid(n_elem, dtype);
    const char* mine = reinterpret_cast<const char*>(inboxes[me]);
    cudaStream_t st = as_stream(stream);
    P2P_DISPATCH(dtype, {
        switch (mode) {
            case P2P_PART_SUM:
                hop_send_kernel<scalar_t, kSum><<<grid, kHopBlock, 0, st>>>(p, nullptr, nullptr, n_vec, dst, mine, me,
                                                                           pass, pass_at, ring, sb, wait_ns);
                break;
            case P2P_PART_DIFF:
                hop_send_kernel<scalar_t, kDiff><<<grid, kHopBlock, 0, st>>>(p, h, nullptr, n_vec, dst, mine, me, pass,
                                                                            pass_at, ring, sb, wait_ns);
                break;
            default:
                hop_send_kernel<scalar_t, kReplica><<<grid, kHopBlock, 0, st>>>(p, h, h_copy, n_vec, dst, mine, me,
                                                                               pass, pass_at, ring, sb, wait_ns);
        }
    });
    return launch_status("p2p_hop_send");
}

extern "C" int p2p_hop_recv(void* const* inboxes, int n_ranks, int me, const int* srcs, int n_src, uint32_t pass,
                            const uint32_t* pass_at, int ring, int64_t cap_elems, int dtype, int64_t n_elem, void* out,
                            int64_t wait_us, void* stream) {
    if (int e = check_common(inboxes, n_ranks, me, ring, cap_elems, dtype, n_elem, wait_us, "recv")) return e;
    HopPeers src;
    if (int e = fill_peers(src, inboxes, n_ranks, srcs, n_src, "recv")) return e;
    P2P_REQUIRE(out && aligned16(out), "p2p_hop_recv: out is null or not 16-byte aligned");
    const int64_t n_vec = n_elem * dtype_size(dtype) / 16;
    const int grid = hop_grid(n_elem, dtype);
    const char* mine = reinterpret_cast<const char*>(inboxes[me]);
    P2P_DISPATCH(dtype, {
        hop_recv_kernel<scalar_t><<<grid, kHopBlock, 0, as_stream(stream)>>>(
            src, mine, me, pass, pass_at, ring, slot_bytes_of(cap_elems, dtype), n_vec, out, (uint64_t)wait_us * 1000ull);
    });
    return launch_status("p2p_hop_recv");
}

extern "C" int p2p_hop_advance(uint32_t* counters, int n, void* stream) {
    P2P_REQUIRE(counters && n >= 1 && n <= 32, "p2p_hop_advance: 1 to 32 counters");
    hop_advance_kernel<<<1, 32, 0, as_stream(stream)>>>(counters, n);
    return launch_status("p2p_hop_advance");
}

extern "C" int p2p_hop_status(int reset, void* stream) {
    cudaStream_t st = as_stream(stream);
    int v[2] = {0, 0};
    if (cudaMemcpyFromSymbolAsync(&v[0], g_hop_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaMemcpyFromSymbolAsync(&v[1], g_hop_rank, sizeof(int), 0, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return fail(P2P_ECUDA, "p2p_hop_status: %s", cudaGetErrorString(cudaGetLastError()));
    if (reset && v[0]) {
        const int zero = 0;
        cudaMemcpyToSymbolAsync(g_hop_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
        cudaStreamSynchronize(st);
    }
    if (v[0] == 1) return fail(P2P_ECUDA, "p2p_hop_send: the wait for rank %d to free its slot timed out", v[1]);
    if (v[0]) return fail(P2P_ECUDA, "p2p_hop_recv: the wait for rank %d's part timed out", v[1]);
    return P2P_OK;
}
