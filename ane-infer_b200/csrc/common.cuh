// common.cuh -- shared device helpers and the on-device data layouts of the B200 decode backend.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ab2 {

constexpr int kWarp = 32;
constexpr unsigned kFull = 0xffffffffu;

// ----------------------------------------------------------------------------------------
// Packed Q8_0 weight layout ("q8p"), written once at upload by q8_repack_kernel.
//
// A GGUF Q8_0 tensor of M rows x K cols is stored as 34-byte blocks [f16 d][32 x i8 q]
// (crates/gguf/src/dequant.rs:29-38). On the device it is split and reordered so that one
// warp reads one 16-row x 32-col tile (an "m16 x kb" tile: 16 rows, one Q8_0 block per row)
// with a single coalesced 16-byte load per lane, already in the register order of the A
// operand of mma.m16n8k16:
//
//   qs  : uint8 [M16][KB][32 lanes][16]   (M16 = ceil(M/16), KB = K/32); lane = 4*g + t
//         bytes  0..7  -> k16 step 0: a0 = (row g,   cols 2t,2t+1), a1 = (row g+8, cols 2t,2t+1),
//                                     a2 = (row g,   cols 2t+8,+9), a3 = (row g+8, cols 2t+8,+9)
//         bytes  8..15 -> k16 step 1: same with cols + 16
//         each byte holds q ^ 0x80 (offset binary: q + 128), so two bytes become an exact
//         f16 pair with one PRMT and one HSUB2 (see q8_unpack).
//   d   : uint32 [M16][KB][8 g]  -> low half = f16 d of row g, high half = f16 d of row g+8
//
// Rows >= M are zero-padded (q = 0, d = 0).
constexpr int kQ8TileBytes = 512;  // one m16 x kb tile of qs

// ----------------------------------------------------------------------------------------
// Activation fragment layout ("xfrag"): the B operand of mma.m16n8k16 for a GEMM with K
// inputs and up to NB batch rows, in f16 with an exact-to-2^-22 hi/lo split of each f32
// activation (x = hi + lo, hi = f16(x), lo = f16(x - hi)).
//
//   xfrag : uint4 [KB][NTILE][32 lanes]; within a k32 block, lane (g = n, t) holds
//           { b0(k16 step 0), b1(k16 step 0), b0(k16 step 1), b1(k16 step 1) },
//           b0 = (k = 2t, 2t+1), b1 = (k = 2t+8, 2t+9), column n = g.
//   "packed" mode (batch <= 4, NTILE = 1): column n = b for hi, n = 4 + b for lo.
//   "stacked" mode (batch > 4, NTILE = 2*NT, NT = ceil(batch/8)): tiles [0, NT) hold the
//           hi parts of batch rows 8j..8j+7 (n = b % 8), tiles [NT, 2NT) the lo parts.
struct XfragShape {
    int kb;      // K / 32
    int ntile;   // tiles per k32 block
    int packed;  // 1: packed mode, 0: stacked mode
    int nt;      // NT (stacked) or 1 (packed)
};

__host__ __device__ inline XfragShape xfrag_shape(int K, int batch) {
    XfragShape s;
    s.kb = K / 32;
    s.packed = batch <= 4 ? 1 : 0;
    s.nt = s.packed ? 1 : (batch + 7) / 8;
    s.ntile = s.packed ? 1 : 2 * s.nt;
    return s;
}

__host__ __device__ inline size_t xfrag_bytes(int K, int batch) {
    XfragShape s = xfrag_shape(K, batch);
    return (size_t)s.kb * s.ntile * 32 * 16;
}

// byte offset of the f16 element (batch row b, input k, part hl: 0 = hi, 1 = lo)
__device__ __forceinline__ size_t xfrag_offset(const XfragShape& s, int b, int k, int hl) {
    int kb = k >> 5, kk = k & 31;
    int s16 = kk >> 4, r = kk & 15;
    int ihi = r >> 3, r8 = r & 7;
    int t = r8 >> 1, p = r8 & 1;
    int tile, n;
    if (s.packed) {
        tile = 0;
        n = b + 4 * hl;
    } else {
        tile = hl * s.nt + (b >> 3);
        n = b & 7;
    }
    int lane = n * 4 + t;
    return ((((size_t)kb * s.ntile + tile) * 32 + lane) * 16) + (s16 * 2 + ihi) * 4 + p * 2;
}

__device__ __forceinline__ void xfrag_store(uint8_t* xf, const XfragShape& s, int b, int k, float v) {
    __half hi = __float2half_rn(v);
    __half lo = __float2half_rn(v - __half2float(hi));
    *reinterpret_cast<__half*>(xf + xfrag_offset(s, b, k, 0)) = hi;
    *reinterpret_cast<__half*>(xf + xfrag_offset(s, b, k, 1)) = lo;
}

// ----------------------------------------------------------------------------------------
// Activation layout of the tcgen05 GEMM ("x16"): the B operand in f16, stored exactly as the
// shared-memory image of K-major 128-byte-swizzled tiles, so one bulk copy per 64-wide K tile
// lands it ready for tcgen05.mma: [K/64][npad rows][128 B], where the 16-byte chunk j of row n
// is stored at chunk position j ^ (n % 8).
// the tcgen05 GEMM takes the activations as its N operand: 64 rows for a batch of up to 64,
// 128 rows for 65..128 (a prefill step)
__host__ __device__ inline int x16_npad(int batch) { return batch > 64 ? 128 : 64; }
__host__ __device__ inline size_t x16_bytes(int K, int batch) {
    return (size_t)((K + 63) / 64) * x16_npad(batch) * 128;
}
__device__ __forceinline__ size_t x16_offset(int npad, int b, int k) {
    const int kt = k >> 6, kk = k & 63, j = kk >> 3, e = kk & 7;
    return ((size_t)kt * npad + b) * 128 + ((j ^ (b & 7)) << 4) + e * 2;
}

// Where a kernel writes the activations of the next GEMM: xfrag (mma.sync path, exact
// weights, f16 hi/lo activations) for small batches, x16 (tcgen05 path) for large ones.
struct ActOut {
    uint8_t* buf = nullptr;
    int x16 = 0;
    int npad = 16;
    XfragShape xs{};
};

__host__ __device__ inline ActOut act_out(uint8_t* buf, int K, int batch, bool x16) {
    ActOut o;
    o.buf = buf;
    o.x16 = x16 ? 1 : 0;
    o.npad = x16_npad(batch);
    o.xs = xfrag_shape(K, batch);
    return o;
}

__device__ __forceinline__ void act_store(const ActOut& o, int b, int k, float v) {
    if (o.x16)
        *reinterpret_cast<__half*>(o.buf + x16_offset(o.npad, b, k)) = __float2half_rn(v);
    else
        xfrag_store(o.buf, o.xs, b, k, v);
}

// ----------------------------------------------------------------------------------------
// f16 / bf16 helpers
__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ float f16bits_to_f32(uint32_t h16) {
    return __half2float(__ushort_as_half((unsigned short)(h16 & 0xffffu)));
}

// Two offset-binary bytes of w (selected by sel) -> an exact f16 pair (q0, q1).
// prmt builds 0x64XX for each byte XX, i.e. f16 value 1024 + (q + 128); subtracting
// 1152 leaves q exactly.
template <uint32_t SEL>
__device__ __forceinline__ uint32_t q8_pair_to_h2(uint32_t w) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(w), "r"(0x64646464u), "n"(SEL));
    __half2 h = *reinterpret_cast<__half2*>(&r);
    const __half2 off = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
    h = __hsub2(h, off);
    return *reinterpret_cast<uint32_t*>(&h);
}

// 16 packed bytes -> A fragments for two k16 steps (a[0..3] step 0, a[4..7] step 1)
__device__ __forceinline__ void q8_unpack(const uint4& q, uint32_t a[8]) {
    a[0] = q8_pair_to_h2<0x4140>(q.x);
    a[1] = q8_pair_to_h2<0x4342>(q.x);
    a[2] = q8_pair_to_h2<0x4140>(q.y);
    a[3] = q8_pair_to_h2<0x4342>(q.y);
    a[4] = q8_pair_to_h2<0x4140>(q.z);
    a[5] = q8_pair_to_h2<0x4342>(q.z);
    a[6] = q8_pair_to_h2<0x4140>(q.w);
    a[7] = q8_pair_to_h2<0x4342>(q.w);
}

// D(16x8 f32) += A(16x16 f16) * B(16x8 f16)
__device__ __forceinline__ void mma_f16(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ----------------------------------------------------------------------------------------
// math in the reference's f32 form (crates/engine/src/deltanet.rs:10-23)
__device__ __forceinline__ float ref_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float ref_silu(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float ref_softplus(float x) { return logf(1.0f + expf(x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
    return v;
}

// block-wide sum for blockDim.x == NT threads; red must hold NT/32 floats
template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < NT / 32; i++) s += red[i];
    return s;
}

// f32::total_cmp ordering key (greedy_sample, crates/cli/src/main.rs:1767-1785)
__device__ __forceinline__ int32_t total_key(float f) {
    int32_t b = __float_as_int(f);
    return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
}

}  // namespace ab2
