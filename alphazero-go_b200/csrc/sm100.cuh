// Blackwell (sm_100a) building blocks written as inline PTX: mbarriers with
// bounded waits, TMA tile loads, and the tcgen05 tensor-core instructions
// (TMEM allocation, MMA issue, commit, TMEM loads) with their shared-memory
// and instruction descriptors.
//
// Every wait here is bounded by %globaltimer: a wait that runs past its
// limit records an error code in a global word and returns false, so a
// kernel that loses a barrier arrival ends with an error status instead of
// hanging the GPU.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>

#include "kernels.hpp"

namespace azb {

// How long one wait may block before the kernel gives up (nanoseconds).
constexpr uint64_t kWaitLimitNs = 1000ull * 1000ull * 1000ull;   // 1 s


__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ------------------------------------------ programmatic dependent launch

// Waits until the kernels this one was launched after (with programmatic
// stream serialization) have completed and their memory is visible; no-op
// when there are none. Every kernel of a pass calls it before it touches an
// activation another kernel wrote or reads.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Lets the next kernel of the stream start launching (its CTAs take SMs as
// this kernel's free them and run up to their own grid_dependency_wait).
__device__ __forceinline__ void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------------ mbarrier

// A position in a ring of pipeline stages: the stage and the parity of
// its current phase, advanced by a compare instead of a division.
struct Ring {
    uint32_t idx = 0, phase = 0;
    __device__ __forceinline__ void next(uint32_t stages) {
        if (++idx == stages) {
            idx = 0;
            phase ^= 1u;
        }
    }
};


__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes barrier initialisation visible to the async proxy (TMA, tcgen05).
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Waits for the phase with the given parity to complete, for at most
// kWaitLimitNs. On timeout records `code` in *err (first error wins) and
// returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = global_timer();
    for (;;) {
        for (int i = 0; i < 32; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (global_timer() - start > kWaitLimitNs) {
            atomicCAS(err, 0, code);
            return false;
        }
    }
}

// --------------------------------------------------------------------- TMA

// Brings the 128-byte line holding `p` into L2.
__device__ __forceinline__ void prefetch_l2(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<uint64_t>(p)));
}

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// A 2D tile of `map` at element coordinates (x, y) into shared memory at
// `dst`, completing `bytes` of transaction on `bar`. x is a multiple of 16
// bytes' worth of elements in every call of this engine (channel chunks of
// 128 bytes). Rows outside the tensor (negative y included) read as zero.
__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, void* dst, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// `bytes` (a multiple of 16) from global memory at `src` into shared memory
// at `dst` (both 16-byte aligned) as one bulk copy, completing on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// A 2D tile from shared memory at `src` to `map` at element coordinates
// (x, y) >= 0, in this thread's current bulk group; rows or columns outside
// the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(src)), "r"(x), "r"(y)
                 : "memory");
}

// Closes this thread's current bulk group.
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Waits until at most kPending of this thread's bulk groups still read
// shared memory (their sources may then be overwritten).
template <int kPending>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(kPending) : "memory");
}

// Waits until every bulk group of this thread has completed its writes.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Orders this thread's earlier shared-memory writes before later async-proxy
// (TMA, tensor core) accesses of them.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Orders this thread's global-memory accesses in the generic proxy with its
// async-proxy (TMA) accesses of global memory, both ways.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// -------------------------------------------------- counters between CTAs

// Adds v to *flag with release semantics at GPU scope: this thread's earlier
// writes are visible to a thread that reads the sum with acquire.
__device__ __forceinline__ void flag_add_release(unsigned* flag, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(flag), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned flag_load_acquire(const unsigned* flag) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    return v;
}

// Waits until *flag >= target, for at most half of kWaitLimitNs: a wait for
// another CTA's work starves this CTA's own pipeline waits (bounded by
// kWaitLimitNs), so it must run out first for the error word to name the
// cause. On timeout records `code` in *err (first error wins) and returns
// false.
__device__ __forceinline__ bool flag_wait(const unsigned* flag, unsigned target, int* err, int code) {
    if (flag_load_acquire(flag) >= target) return true;
    const uint64_t start = global_timer();
    for (;;) {
        __nanosleep(100);
        if (flag_load_acquire(flag) >= target) return true;
        if (global_timer() - start > kWaitLimitNs / 2) {
            atomicCAS(err, 0, code);
            return false;
        }
    }
}

// ------------------------------------------------------------------ tcgen05

// Allocates `ncols` TMEM columns (a power of two >= 32) for this CTA and
// writes the base address to shared memory at `dst`. Whole warp.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

// Whole warp.
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D (TMEM, fp32) (+)= A (smem, K-major) . B (smem, K-major)^T, one thread.
// kind::f16 covers bf16 x bf16; kind::tf32 covers tf32 x tf32.
template <bool kBf16>
__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    if constexpr (kBf16) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
            ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
            ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    }
}

// Arrives once on `bar` when every tcgen05.mma this thread issued so far has
// completed (their shared-memory operands may then be overwritten).
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane (warp-collective:
// lane i of the warp reads lane (taddr.lane + i)).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// After tmem_wait_ld: ties registers a tcgen05.ld wrote to the wait, so no
// use of them is scheduled before it (to the compiler they are written at
// the load).
template <int K>
__device__ __forceinline__ void tmem_hold(uint32_t (&v)[K]) {
#pragma unroll
    for (int i = 0; i < K; ++i) asm volatile("" : "+r"(v[i]));
}

// 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}

// The store counterpart: 32 consecutive 32-bit columns of this thread's lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
        "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
        "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ------------------------------------------------- CTA pairs (cta_group::2)
//
// The two CTAs of a 2-CTA cluster compute one M = 256 tile together: each
// stages its own 128 rows of A and half of B; the pair's leader (rank 0)
// issues the MMAs, which read both CTAs' shared memory and write both CTAs'
// TMEM. Each helper below addresses one CTA's barrier or memory at a time.

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// All threads of both CTAs: everything before (barrier inits, remote
// arrivals) is visible to everything after.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The shared::cluster address of this CTA's shared-memory location `saddr`
// as seen in cluster CTA `rank`.
__device__ __forceinline__ uint32_t mapa(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}

// Arrive on an mbarrier given by its shared::cluster address (possibly the
// peer CTA's), releasing this thread's prior work at cluster scope.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// mbar_wait with cluster-scope acquire: for barriers the peer CTA arrives on.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* err, int code) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t start = global_timer();
    for (;;) {
        for (int i = 0; i < 32; ++i)
            if (mbar_try_wait_cluster(bar, parity)) return true;
        if (global_timer() - start > kWaitLimitNs) {
            atomicCAS(err, 0, code);
            return false;
        }
    }
}

// A 2D TMA tile into THIS CTA's shared memory, its transaction bytes
// completing on the pair leader's barrier (`leader_bar`: a shared::cluster
// address in rank 0). The tile lands in this CTA only.
__device__ __forceinline__ void tma_load_2d_pair(const CUtensorMap* map, void* dst, uint32_t leader_bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(x), "r"(y)
        : "memory");
}

// TMEM for a CTA pair: the same columns in both CTAs. Issued by the same warp
// of both CTAs.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D (both CTAs' TMEM) (+)= A (both CTAs' shared memory, M = 256) . B (both
// halves)^T. Issued by one thread of the leader.
template <bool kBf16>
__device__ __forceinline__ void umma_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    if constexpr (kBf16) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
            ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
            ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    }
}

// Arrives once on the mbarrier at shared::cluster address `bar` (this CTA's
// or the peer's) when the pair MMAs issued so far by this thread complete.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// Shared-memory matrix descriptor for a K-major operand in the 128-byte
// swizzle layout that TMA writes with CU_TENSOR_MAP_SWIZZLE_128B: rows of
// 128 bytes, 8-row (1024-byte) swizzle atoms stacked along M/N (stride byte
// offset 1024), leading byte offset unused (1). Bits 46-48 hold the fixed
// value 0b001; bits 61-63 the swizzle mode (2 = 128-byte). The start address
// may sit at ANY 128-byte row of a 1024-byte-aligned buffer with the matrix
// base offset left at 0: the tensor core takes the swizzle phase from the
// address bits themselves, exactly as TMA applied it (the single-CTA probe
// checks every row shift against exact sums; setting the base offset to
// (address >> 7) & 7 instead gives wrong products). The conv's nine taps are
// such row-shifted views of one staged halo tile.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, int base_offset_mode = 0) {
    uint64_t d = static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
    d |= 1ull << 16;                      // leading byte offset (unused for swizzled K-major)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;   // stride byte offset: one 8-row atom
    d |= 1ull << 46;                      // fixed 0b001
    if (base_offset_mode) d |= static_cast<uint64_t>((saddr >> 7) & 7u) << 49;
    d |= 2ull << 61;                      // SWIZZLE_128B
    return d;
}

// Instruction descriptor: fp32 accumulator, K-major A and B, M = 128 (one
// CTA) or 256 (a CTA pair). a/b format 1 = bf16 (kind::f16), 2 = tf32.
__host__ __device__ constexpr uint32_t umma_idesc(int n, bool bf16, int m = 128) {
    return (1u << 4)                               // D format: f32
           | ((bf16 ? 1u : 2u) << 7)               // A format
           | ((bf16 ? 1u : 2u) << 10)              // B format
           | (static_cast<uint32_t>(n >> 3) << 17) // N / 8
           | (static_cast<uint32_t>(m >> 4) << 24);     // M / 16
}

// Two IEEE round-to-nearest additions in one instruction (add.rn.f32x2,
// sm_100): element-wise the same results as two __fadd_rn.
__device__ __forceinline__ float2 fadd2_rn(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// The same for subtraction (sub.rn.f32x2). (No packed multiply here: on
// this toolchain a mul.rn.f32x2 feeding an add.rn.f32x2 is contracted into
// one fused multiply-add, one rounding where two were asked for; scalar
// __fmul_rn / __fadd_rn are not.)
__device__ __forceinline__ float2 fsub2_rn(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %5};\n\t"
        "sub.rn.f32x2 rd, ra, rb;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// Two IEEE fused multiply-adds in one instruction (fma.rn.f32x2): element
// for element __fmaf_rn(a, b, c).
__device__ __forceinline__ float2 ffma2_rn(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %5};\n\t"
        "mov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

// Round-to-nearest (ties away) to tf32, as cvt.rna.tf32.f32 does; the low
// 13 bits of the result are zero, so a tf32 MMA reads it exactly.
__device__ __forceinline__ float to_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

} // namespace azb
