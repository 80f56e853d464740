// Device-side building blocks of the sm_100a GEMMs (spmm_tc.cu, spmm_mask.cu): mbarriers with bounded waits, TMA and
// bulk copies, tcgen05 MMAs with operands in shared or tensor memory, TMEM loads and stores, cluster (DSMEM) access.
#pragma once
#include <cuda.h>
#include <stdint.h>

#include <type_traits>

#include "common.cuh"

namespace p2p {
namespace sm100 {

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The shared::cluster address of `saddr` (this CTA's shared memory) in cluster CTA `rank`.
__device__ __forceinline__ uint32_t cluster_addr(uint32_t saddr, int rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}

__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// One test of the phase; a thread whose phase is not complete sleeps in hardware (up to the suspend-time hint, in ns)
// until it completes, instead of spinning on the issue slots its warp scheduler shares with working warps.
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}

// Ring position of the next item: `step` slots on (step <= n), the phase bit flipping at each wrap. Kept in
// registers, so the single-thread roles do no divisions by the runtime ring sizes.
__device__ __forceinline__ void advance(int& slot, uint32_t& phase, int step, int n) {
    slot += step;
    if (slot >= n) {
        slot -= n;
        phase ^= 1u;
    }
}

__device__ __forceinline__ void sts_u16(uint32_t addr, uint32_t v) {
    asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"((unsigned short)v) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
        : "memory");
}

// Shared-memory matrix descriptor of a K-major tile in the 128-byte swizzle layout: rows of 128 bytes, 8-row atoms of
// 1024 bytes (stride byte offset), version 1, swizzle mode 2 (128B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor of kind::f16: D fp32, A and B bf16 (or both f16), both K-major, M = 128, N.
template <typename T> __device__ __forceinline__ uint32_t idesc_f16(int n) {
    constexpr uint32_t ab = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
    return (1u << 4) | (ab << 7) | (ab << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
        "[%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}


// How a launch's pipeline waits are bounded: past limit_ns a wait records its site in *site (the first one wins) and
// this launch's sequence number in *failed; every later wait of the same launch then gives up at once.
struct WaitCtl {
    int* site;
    unsigned* failed;
    uint64_t limit_ns;
    unsigned seq;
};

__device__ __forceinline__ void give_up(int where, const WaitCtl& w) {
    atomicCAS(w.site, 0, where);
    atomicExch(w.failed, w.seq);
}

// Waits for the phase of parity `parity`; true once it completed. Past the limit, or at once when another wait of the
// same launch has given up, it records `where` and returns false: the caller then issues no further work.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int where, const WaitCtl& w) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = now_ns();
    while (!mbar_try(bar, parity)) {
        if (*(volatile unsigned*)w.failed == w.seq || now_ns() - t0 > w.limit_ns) {
            give_up(where, w);
            return false;
        }
    }
    return true;
}

// Waits for asynchronous work this CTA already issued (a copy landing, its MMAs completing), which finishes on its
// own: bounded by the limit only, even after another wait gave up, so the CTA never exits with that work in flight.
__device__ __forceinline__ bool mbar_drain(uint32_t bar, uint32_t parity, int where, const WaitCtl& w) {
    const uint64_t t0 = now_ns();
    while (!mbar_try(bar, parity)) {
        if (now_ns() - t0 > w.limit_ns) {
            give_up(where, w);
            return false;
        }
    }
    return true;
}

// One bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned) from global to this CTA's shared memory,
// completing as transactions on `bar`.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// A 16-bit load from shared memory, zero-extended into a 32-bit register.
__device__ __forceinline__ uint32_t lds_u16(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint4 lds_v4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}

// kind::f16 MMA with A (M = 128 rows, K = 16) in tensor memory at a_tmem, B from the shared-memory descriptor.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 16 lanes x 256 bits four times along the columns: thread t writes lanes base + t / 4 (registers 4 r, 4 r + 1) and
// base + 8 + t / 4 (4 r + 2, 4 r + 3), columns 8 r + 2 (t % 4) and + 1 of repetition r.
__device__ __forceinline__ void tmem_st_16x256b_x4(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int c0, int c1) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(c0), "r"(c1), "r"(src)
                 : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

}  // namespace sm100
}  // namespace p2p
