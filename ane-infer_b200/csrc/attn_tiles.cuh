// attn_tiles.cuh -- pieces shared by the tensor-core attention kernels over the bf16 KV cache
// (attn_mma.cu: decode, attn_prefill.cu: prefill): the TMA tile load, ldmatrix and
// mma.m16n8k16 bf16 wrappers, the bf16 hi/lo split, and the split-partial layout.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>

#include <cstdint>

#include "common.cuh"
#include "umma.cuh"

namespace ab2 {

constexpr int kT = 64;      // cache tokens per tile (a TMA box is 64 tokens x 64 dims, 128-byte swizzle)
constexpr int kGQ = 4;      // query heads per kv head
constexpr int kMaxSplits = 64;  // splits per (sequence, kv head)
// floats of one split partial of a (row, kv head): m[kGQ], l[kGQ], unnormalised O[kGQ][HD]
__host__ __device__ constexpr size_t attn_part_floats(int hd) { return (size_t)kGQ * 2 + (size_t)kGQ * hd; }

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}
// f32 -> (hi, lo) bf16 parts with x = hi + lo to about 2^-17 relative
__device__ __forceinline__ void split_bf16(float x, float& hi, float& lo) {
    hi = __bfloat162float(__float2bfloat16_rn(x));
    lo = x - hi;
}

// byte address of the 16-byte chunk `chunk` (8 dims) of token row `row` in a tile of the bf16
// cache loaded as HD / 64 boxes of [64 tokens][64 dims] with the 128-byte swizzle
__device__ __forceinline__ uint32_t kv_tile_addr(uint32_t base, int row, int chunk) {
    return base + (chunk >> 3) * 8192 + row * 128 + (((chunk & 7) ^ (row & 7)) << 4);
}

}  // namespace ab2
