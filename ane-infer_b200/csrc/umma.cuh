// umma.cuh -- thin PTX wrappers for the sm_100a tensor-core path: mbarriers, bulk async
// copies, tcgen05 TMEM allocation / MMA / commit / load, and the shared-memory matrix
// descriptors of K-major, 128-byte-swizzled f16 operands.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace ab2 {

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Programmatic dependent launch: a kernel launched with programmatic stream serialization
// may start while its predecessor runs; pdl_wait() blocks until the predecessor grid has
// completed and its writes are visible (a no-op for ordinary launches). pdl_trigger() lets
// the successor grid start launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// ------------------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait that suspends the thread until the phase completes or `hint_ns` elapses, so a
// waiting thread sleeps instead of occupying issue slots
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar` for at most limit_ns (2 s unless a test shortens it);
// false on timeout. A timeout means a lost arrival; the caller records an error code and
// abandons the tile instead of waiting forever.
constexpr uint32_t kWaitLimitNs = 2000000000u;  // 2 s
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t limit_ns = kWaitLimitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
        if (globaltimer_ns() - t0 > limit_ns) return false;
    }
}

// ------------------------------------------------------------------------------ bulk copy
// global -> shared, completion counted in bytes on `bar` (size and addresses 16-byte aligned)
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// L2 prefetch of [src, src + bytes) (16-byte aligned, size a multiple of 16), fire and forget
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// This CTA's share (CTA `part` of `parts`) of an L2 prefetch of `bytes` bytes at `src`, in
// 32 KB pieces: how kernels pull the weights of the next GEMM on the stream into L2 while
// their own work still runs, so that GEMM's pipeline fills from L2 instead of HBM.
__device__ __forceinline__ void prefetch_share_l2(const void* src, int64_t bytes, int part, int parts) {
    if (!src || bytes <= 0) return;
    const int64_t per = ((bytes + parts - 1) / parts + 15) / 16 * 16;
    const int64_t lo = (int64_t)part * per, hi = lo + per < bytes ? lo + per : bytes;
    for (int64_t o = lo; o < hi; o += 32768) {
        const int64_t n = hi - o < 32768 ? hi - o : 32768;
        bulk_prefetch_l2(static_cast<const uint8_t*>(src) + o, (uint32_t)((n + 15) / 16 * 16));
    }
}

// shared -> global bulk operations of the calling thread's bulk async-group (addresses 16-byte
// aligned, size a multiple of 16): a plain copy, or an f32 add into global memory performed
// at L2; bulk_commit closes the group; bulk_wait_all waits until its writes are complete, and
// bulk_wait_read only until its shared-memory sources have been read (then the staging buffer
// may be reused or the CTA may exit; the writes are visible to dependent grids once this grid
// has completed)
__device__ __forceinline__ void bulk_s2g(void* dst_gmem, const void* src_smem, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst_gmem), "r"(smem_u32(src_smem)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_reduce_add_f32(float* dst_gmem, const float* src_smem, uint32_t bytes) {
    asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(dst_gmem),
                 "r"(smem_u32(src_smem)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ------------------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem desc], f16 inputs, f32 accumulate. A (M=128 x K=16) sits in
// TMEM lane = row, 8 consecutive 32-bit columns each holding the f16 pair (k even, k odd)
__device__ __forceinline__ void umma_ts_f16(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// arrive on `bar` once all previously issued tcgen05.mma of this thread have completed
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// Instruction descriptor of kind::f16: f16 A and B (K-major), f32 D, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N) {
    return (1u << 4)                      // D format f32
           | (0u << 7) | (0u << 10)       // A, B format f16
           | ((uint32_t)(N >> 3) << 17)   // N / 8
           | ((uint32_t)(M >> 4) << 24);  // M / 16
}

// Shared-memory descriptor of a K-major, 128B-swizzled operand whose 8-row groups are
// 1024 bytes apart (rows of 64 f16 = 128 bytes). The start address advances by 32 bytes
// per K16 step inside the swizzle atom.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);      // start address
    d |= (uint64_t)1u << 16;                          // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024u >> 4) << 32;                // stride byte offset: 8 rows x 128 B
    d |= (uint64_t)1u << 46;                          // descriptor version for sm_100
    d |= (uint64_t)2u << 61;                          // SWIZZLE_128B
    return d;
}

}  // namespace ab2
