// Inline-PTX building blocks for the Blackwell (sm_100a) tensor-core kernels:
// mbarriers with bounded waits, TMA tiled loads (no multicast), tcgen05 MMA /
// TMEM allocation / TMEM loads, and the shared-memory matrix descriptor.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace snnb {
namespace tc {

// Spin limits of the mbarrier waits, in SM clock cycles.
//  - Progress waits (a stage's copies, an accumulator, a free ring slot) give up after the
//    per-device limit g_wait_limit: ~2 s at the B200's 1.9 GHz SM clock unless the host set
//    another with snnb_set_wait_limit.  The value is read only once a wait has to spin.
//  - Drain waits (after a failure: for copies or MMAs already issued, which complete on
//    their own; or for the whole kernel's last commit) always use DRAIN_LIMIT_CYCLES, so a
//    short progress limit can never let a CTA exit with copies still landing in its
//    shared memory.
constexpr unsigned long long DEFAULT_WAIT_LIMIT = 4000000000ull;
constexpr unsigned long long DRAIN_LIMIT_CYCLES = 4000000000ull;
constexpr long long WAIT_LIMIT_CYCLES = (long long)DEFAULT_WAIT_LIMIT;

// One copy per translation unit that includes this header (no relocatable device code);
// snnb_set_wait_limit writes every copy on the current device through the setters that
// each unit registers at load time.
static __device__ unsigned long long g_wait_limit = DEFAULT_WAIT_LIMIT;
static cudaError_t set_wait_limit_tu(unsigned long long cycles) {
    return cudaMemcpyToSymbol(g_wait_limit, &cycles, sizeof(cycles));
}
static const int g_wait_limit_setter_registered = register_wait_limit_setter(&set_wait_limit_tu);

// The limit a wait uses: the run-time progress limit, or the fixed drain limit.
template <bool DRAIN>
__device__ __forceinline__ const unsigned long long* wait_limit_ptr() {
    if constexpr (DRAIN) {
        return nullptr;
    } else {
        return &g_wait_limit;
    }
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: returns false (after writing SNNB_ERR_TIMEOUT to the device status word
// and raising the CTA's abort flag) if the phase does not complete within
// WAIT_LIMIT_CYCLES, or if another role of the CTA has already aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int* status) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    uint32_t it = 0;
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((++it & 255u) == 0) {
            if (*abort_flag) return false;
            if ((unsigned long long)(clock64() - t0) > *(volatile unsigned long long*)&g_wait_limit) {
                atomicExch(status, SNNB_ERR_TIMEOUT);
                *abort_flag = 1;
                return false;
            }
        }
    }
}

// One lane of a converged warp (elect.sync): the lane that issues a TMA copy, an MMA or a
// commit for the whole warp.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "elect.sync _|p, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(pred));
    return pred != 0;
}

// Bounded wait of a whole converged warp, as one asm block: the lanes spin on try_wait and
// agree through votes, so every lane leaves together and compiled code never branches on a
// per-lane value (a branch there costs the MMA issuer its warp-uniform registers: each
// tcgen05.mma issued after it took ~4x longer).  Returns 1 when the phase completed, 0 after
// WAIT_LIMIT_CYCLES or at once when skip != 0 (an earlier wait of this warp failed).
template <bool DRAIN = false>
__device__ __forceinline__ uint32_t mbar_wait_warp(uint32_t bar, uint32_t parity, uint32_t skip) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t.reg .u64 t0, t1, lim;\n\t"
        "setp.ne.u32 q, %3, 0;\n\t"
        "@q bra WFAIL_%=;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "vote.sync.all.pred p, p, 0xffffffff;\n\t"
        "@p bra WOK_%=;\n\t"
        "mov.u64 lim, %4;\n\t"
        "setp.eq.u64 q, %5, 0;\n\t"
        "@!q ld.volatile.u64 lim, [%5];\n\t"
        "mov.u64 t0, %%clock64;\n\t"
        "WLOOP_%=:\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "vote.sync.all.pred p, p, 0xffffffff;\n\t"
        "@p bra WOK_%=;\n\t"
        "mov.u64 t1, %%clock64;\n\t"
        "sub.u64 t1, t1, t0;\n\t"
        "setp.lt.u64 q, t1, lim;\n\t"
        "vote.sync.any.pred q, q, 0xffffffff;\n\t"
        "@q bra WLOOP_%=;\n\t"
        "WFAIL_%=:\n\t"
        "mov.u32 %0, 0;\n\t"
        "bra.uni WEND_%=;\n\t"
        "WOK_%=:\n\t"
        "mov.u32 %0, 1;\n\t"
        "WEND_%=:\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(skip), "l"(DRAIN_LIMIT_CYCLES),
          "l"(wait_limit_ptr<DRAIN>())
        : "memory");
    return ok;
}

// The same bounded wait for one thread (the elected lane of the MMA warp: only it touches
// the stage it waits for).  No votes, so it adds nothing to the issue path when the phase
// has already completed.
__device__ __forceinline__ uint32_t mbar_wait_lane(uint32_t bar, uint32_t parity, uint32_t skip) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t.reg .u64 t0, t1, lim;\n\t"
        "setp.ne.u32 q, %3, 0;\n\t"
        "@q bra LFAIL_%=;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "@p bra LOK_%=;\n\t"
        "ld.volatile.u64 lim, [%4];\n\t"
        "mov.u64 t0, %%clock64;\n\t"
        "LLOOP_%=:\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "@p bra LOK_%=;\n\t"
        "mov.u64 t1, %%clock64;\n\t"
        "sub.u64 t1, t1, t0;\n\t"
        "setp.lt.u64 q, t1, lim;\n\t"
        "@q bra LLOOP_%=;\n\t"
        "LFAIL_%=:\n\t"
        "mov.u32 %0, 0;\n\t"
        "bra.uni LEND_%=;\n\t"
        "LOK_%=:\n\t"
        "mov.u32 %0, 1;\n\t"
        "LEND_%=:\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(skip), "l"(&g_wait_limit)
        : "memory");
    return ok;
}

// ---- TMA (tiled, no multicast) ------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* tm, uint32_t bar,
                                            int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(c0), "r"(c1)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* tm, uint32_t bar,
                                            int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* tm, uint32_t bar,
                                            int c0, int c1, int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}
__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* tm, uint32_t bar,
                                            int c0, int c1, int c2, int c3, int c4) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
        : "memory");
}
// Bulk prefetch of [src, src + bytes) into L2 (src 16-byte aligned, bytes a multiple of 16).
// Tiled TMA store from shared memory (bulk-group completion; coordinates >= 0, elements
// outside the tensor are not written).  The writing threads fence their shared-memory
// stores to the async proxy (fence_proxy_async_smem) and synchronise before one thread
// issues the store.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* tm, uint32_t src, int c0, int c1,
                                             int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(tm),
        "r"(src), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until at most N committed bulk groups still READ their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until at most N committed bulk groups are incomplete (their writes done).
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(src)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* tm) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}

// ---- tcgen05 ------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, bf16 x bf16 -> f32, one instruction per call.
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
    const uint32_t z = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
        : "memory");
}
// Arrive once on an mbarrier when every tcgen05.mma issued so far by this thread is done.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// 32 lanes x 32 consecutive 32-bit columns: thread i gets row (lane base + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&r)[32]) {
    uint32_t u[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]),
          "=r"(u[7]), "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]),
          "=r"(u[14]), "=r"(u[15]), "=r"(u[16]), "=r"(u[17]), "=r"(u[18]), "=r"(u[19]),
          "=r"(u[20]), "=r"(u[21]), "=r"(u[22]), "=r"(u[23]), "=r"(u[24]), "=r"(u[25]),
          "=r"(u[26]), "=r"(u[27]), "=r"(u[28]), "=r"(u[29]), "=r"(u[30]), "=r"(u[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) r[i] = __uint_as_float(u[i]);
}
// Ties later uses of r to this point of the instruction stream: after tcgen05.wait::ld, so
// that no use of an asynchronously loaded register is scheduled before the wait.
__device__ __forceinline__ void reg_fence16(float (&r)[16]) {
    asm volatile(""
                 : "+f"(r[0]), "+f"(r[1]), "+f"(r[2]), "+f"(r[3]), "+f"(r[4]), "+f"(r[5]),
                   "+f"(r[6]), "+f"(r[7]), "+f"(r[8]), "+f"(r[9]), "+f"(r[10]), "+f"(r[11]),
                   "+f"(r[12]), "+f"(r[13]), "+f"(r[14]), "+f"(r[15])
                 :
                 : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&r)[16]) {
    uint32_t u[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15}, [%16];"
        : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]),
          "=r"(u[7]), "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]),
          "=r"(u[14]), "=r"(u[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) r[i] = __uint_as_float(u[i]);
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the 128-byte
// swizzle (rows of 128 bytes, 8-row / 1024-byte swizzle atoms, tile 1024-byte aligned):
// start address >> 4 in bits [0,14), leading byte offset 16 B (unused for swizzled
// K-major), stride byte offset 1024 B in bits [32,46), descriptor version 1 in bits
// [46,48), layout SWIZZLE_128B (= 2) in bits [61,64).
__device__ __forceinline__ uint64_t sdesc_k_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor of kind::f16 with bf16 A and B (K-major), f32 accumulator.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
    return (1u << 4)                       // D format: f32
         | (1u << 7)                       // A format: bf16
         | (1u << 10)                      // B format: bf16
         | ((uint32_t)(N >> 3) << 17)      // N / 8
         | ((uint32_t)(M >> 4) << 24);     // M / 16
}

// ---- CTA pairs: a cluster of 2 CTAs issuing tcgen05 with cta_group::2 ------------------
// The even CTA (rank 0) issues the M = 256 MMAs; operand rows 0-127 of A and the first half
// of B's rows come from its shared memory, the rest from the odd CTA's at the same offsets,
// and each CTA's TMEM receives its own 128 accumulator rows.
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Every thread of both CTAs: barrier across the cluster (release / acquire).
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
}
// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
                 : "memory");
}
// 8-byte asynchronous global -> shared copy; src_bytes 0 writes zeros and reads nothing.
__device__ __forceinline__ void cp_async_8(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst),
                 "l"(reinterpret_cast<uint64_t>(src)), "r"(src_bytes)
                 : "memory");
}
// Waits for this thread's cp.async copies.
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;" ::: "memory");
}
// Makes this thread's earlier generic-proxy shared-memory writes visible to the async proxy
// (tcgen05.mma operand reads, TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Orders this thread's earlier shared-memory writes (and those its CTA barrier made visible
// to it) before its later arrivals on other CTAs' barriers.
__device__ __forceinline__ void fence_acq_rel_cluster() {
    asm volatile("fence.acq_rel.cluster;" ::: "memory");
}
// 16 bytes of another CTA's shared memory (a mapa address).
__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t cluster_addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(cluster_addr));
    return v;
}
// mbar_wait_warp with cluster-scope acquire: for a barrier other CTAs of the cluster arrive
// on after writing shared memory this warp then reads.
__device__ __forceinline__ uint32_t mbar_wait_warp_cluster(uint32_t bar, uint32_t parity,
                                                           uint32_t skip) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t.reg .u64 t0, t1, lim;\n\t"
        "setp.ne.u32 q, %3, 0;\n\t"
        "@q bra CFAIL_%=;\n\t"
        "ld.volatile.u64 lim, [%4];\n\t"
        "mov.u64 t0, %%clock64;\n\t"
        "CLOOP_%=:\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "vote.sync.all.pred p, p, 0xffffffff;\n\t"
        "@p bra COK_%=;\n\t"
        "mov.u64 t1, %%clock64;\n\t"
        "sub.u64 t1, t1, t0;\n\t"
        "setp.lt.u64 q, t1, lim;\n\t"
        "vote.sync.any.pred q, q, 0xffffffff;\n\t"
        "@q bra CLOOP_%=;\n\t"
        "CFAIL_%=:\n\t"
        "mov.u32 %0, 0;\n\t"
        "bra.uni CEND_%=;\n\t"
        "COK_%=:\n\t"
        "mov.u32 %0, 1;\n\t"
        "CEND_%=:\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(skip), "l"(&g_wait_limit)
        : "memory");
    return ok;
}
// Tiled loads into this CTA's shared memory whose completion bytes are counted on the
// mbarrier at `bar` (a shared::cluster address: the pair's even CTA); no multicast.
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* tm, uint32_t bar,
                                                 int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}
__device__ __forceinline__ void tma_load_5d_pair(uint32_t dst, const CUtensorMap* tm, uint32_t bar,
                                                 int c0, int c1, int c2, int c3, int c4) {
    asm volatile(
        "cp.async.bulk.tensor.5d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
        : "memory");
}
// TMEM of a pair: one warp (same warp index) in each CTA issues these together.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
// D (+)= A * B^T over the pair (M = 256), issued by one thread of the even CTA.
__device__ __forceinline__ void umma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                               uint32_t idesc, uint32_t accumulate) {
    const uint32_t z = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n\t}\n"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z),
        "r"(z), "r"(z), "r"(z), "r"(z), "r"(z)
        : "memory");
}
// Arrive once on the mbarrier at offset `bar` of every CTA in `cta_mask` when the pair MMAs
// issued so far by this thread are done.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar, uint16_t cta_mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        " [%0], %1;" ::"r"(bar), "h"(cta_mask)
        : "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Named barrier with an OR reduction: every one of `threads` threads passes its predicate
// and all of them get true if any passed true.  Used after bounded waits so that the
// threads of a role agree on aborting and none is left waiting at a later barrier.
__device__ __forceinline__ bool named_bar_any(int id, int threads, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}\n"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(id), "r"(threads)
        : "memory");
    return r != 0;
}

}  // namespace tc

// Host: device pointer of this library's status word on the current device
// (nullptr on failure).  Kernels with bounded waits record SNNB_ERR_TIMEOUT there.
int* device_status_ptr();

// Host: encode a tiled TMA descriptor (bf16 or f32 elements, 128-byte swizzle,
// zero fill out of bounds; elem_strides: per-dimension traversal strides, nullptr = all 1).
// Returns SNNB_OK or an error status.
int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                CUtensorMapSwizzle swizzle, const uint32_t* elem_strides = nullptr);

}  // namespace snnb
