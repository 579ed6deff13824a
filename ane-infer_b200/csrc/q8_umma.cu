// q8_umma.cu -- batched Q8_0 dequant-GEMM on the 5th-generation tensor cores (tcgen05).
//
// D[128 rows][N] = W[128 rows][K] * X[N][K]^T per CTA (N = batch padded to 16/32/64):
//   * warp 0 streams each 128x64 weight tile (int8 + f16 scales, 8.5 KB, contiguous in the
//     "q8t" layout) and the matching 64-wide activation tile (already in the swizzled smem
//     image, the "x16" layout) into a 3-stage ring with cp.async.bulk + mbarrier tx counts;
//   * warps 2-5 turn each weight tile into the f16 A operand (w = q * d rounded once to f16;
//     q is exact in f16 and the product is one correctly rounded f16 multiply) in the
//     K-major 128B-swizzled layout, then fence the writes to the async proxy;
//   * warp 1 allocates the TMEM accumulator and one lane issues tcgen05.mma (M=128, N, K=16)
//     x4 per tile, committing each stage back to the producer;
//   * after the K loop warps 2-5 read their 32-lane TMEM quarter and run the epilogue
//     (store / residual add / SwiGLU into the next GEMM's activations), or write split-K
//     partials that the last CTA of the m-tile sums in split order.
// Every mbarrier wait is bounded; on a timeout the CTA records an error code, drains its
// own copies and MMAs (again bounded), frees its TMEM and returns.
#include "common.cuh"
#include "kernels.h"
#include "umma.cuh"

namespace ab2 {

constexpr int kTileRows = 128;
constexpr int kTileK = 64;
constexpr int kWTileBytes = 8192 + 512;  // [4 chunks][128 rows][16 B] int8 + [128 rows][2] f16
constexpr int kStages = 3;        // ~99 KB smem: two CTAs per SM
constexpr int kUmmaThreads = 192;        // warp 0 producer, warp 1 MMA, warps 2-5 convert + epilogue

// ------------------------------------------------------------------------------ repack
// one thread per source (row, Q8_0 block): row -> dst row R = base + (row/grp)*stride + row%grp,
// block kb -> tile kt = kb/2, chunks 2*(kb%2) and 2*(kb%2)+1, scale slot kb%2
__global__ void q8t_repack_kernel(const uint8_t* __restrict__ src, int64_t rows, int KB, uint8_t* __restrict__ dst,
                                  int KT, int64_t base, int64_t grp, int64_t stride) {
    int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (id >= rows * KB) return;
    const int64_t r = id / KB;
    const int kb = (int)(id % KB);
    const uint8_t* blk = src + id * 34;
    const int64_t R = base + (r / grp) * stride + (r % grp);
    const int64_t mt = R / kTileRows;
    const int rr = (int)(R % kTileRows);
    const int kt = kb >> 1, half = kb & 1;
    uint8_t* tile = dst + ((size_t)mt * KT + kt) * kWTileBytes;
#pragma unroll
    for (int c2 = 0; c2 < 2; c2++) {
        uint8_t* chunk = tile + ((size_t)(half * 2 + c2) * kTileRows + rr) * 16;
#pragma unroll
        for (int i = 0; i < 16; i++) chunk[i] = (uint8_t)(blk[2 + c2 * 16 + i] ^ 0x80u);
    }
    tile[8192 + rr * 4 + half * 2 + 0] = blk[0];
    tile[8192 + rr * 4 + half * 2 + 1] = blk[1];
}

void launch_q8t_repack(const uint8_t* src, int64_t rows, int KB, Q8Weight& w, int64_t base, int64_t grp,
                       int64_t stride, cudaStream_t st) {
    int64_t n = rows * KB;
    q8t_repack_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(src, rows, KB, w.qt, w.KT, base, grp, stride);
}

// ------------------------------------------------------------------------------ kernel
struct UmmaSmem {
    // offsets from the 1024-aligned dynamic smem base
    static constexpr int a_off(int s) { return s * 16384; }
    static constexpr int b_off(int s, int N) { return kStages * 16384 + s * N * 128; }
    static constexpr int w_off(int s, int N) { return kStages * 16384 + kStages * N * 128 + s * kWTileBytes; }
    static constexpr int bar_off(int N) { return w_off(kStages, N); }
    // full[S], conv[S], freed[S], acc, + tmem slot
    static constexpr int bytes(int N) { return bar_off(N) + (3 * kStages + 1) * 8 + 16; }
};

template <int N>
__global__ void __launch_bounds__(kUmmaThreads, 2)
    q8_umma_gemm_kernel(const uint8_t* __restrict__ wt, int KT, int MT, const uint8_t* __restrict__ x16, int batch,
                        int kt_per_split, float* __restrict__ ws, unsigned* __restrict__ tickets,
                        unsigned* __restrict__ err, GemmEpi ep) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + UmmaSmem::bar_off(N));
    uint64_t* conv = full + kStages;
    uint64_t* freed = conv + kStages;
    uint64_t* accb = freed + kStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accb + 1);
    __shared__ int s_abort;
    __shared__ unsigned s_last;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = blockIdx.x, split = blockIdx.y, nsplit = gridDim.y;
    const int kt0 = split * kt_per_split, kt1 = min(KT, kt0 + kt_per_split);
    const int ntiles = kt1 - kt0;
    constexpr uint32_t kCols = N < 32 ? 32 : N;

    if (threadIdx.x == 0) {
        s_abort = 0;
        for (int s = 0; s < kStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&conv[s], 128);
            mbar_init(&freed[s], 1);
        }
        mbar_init(accb, 1);
        mbar_fence_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, kCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- producer
        if (lane == 0) {
            const uint8_t* wsrc = wt + ((size_t)mt * KT) * kWTileBytes;
            int i = 0;
            for (; i < ntiles; i++) {
                const int s = i % kStages;
                if (i >= kStages && !mbar_wait(&freed[s], ((i / kStages) - 1) & 1)) {
                    atomicOr(err, 1u);
                    s_abort = 1;
                    break;
                }
                if (*(volatile int*)&s_abort) break;
                mbar_arrive_expect_tx(&full[s], kWTileBytes + N * 128);
                bulk_g2s(smem + UmmaSmem::w_off(s, N), wsrc + (size_t)(kt0 + i) * kWTileBytes, kWTileBytes, &full[s]);
                bulk_g2s(smem + UmmaSmem::b_off(s, N), x16 + (size_t)(kt0 + i) * N * 128, N * 128, &full[s]);
            }
            // drain: the last min(i, S) issued stages must have landed before the CTA exits
            for (int j = max(0, i - kStages); j < i; j++)
                if (!mbar_wait(&full[j % kStages], (j / kStages) & 1)) atomicOr(err, 2u);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(kTileRows, N);
            int i = 0;
            for (; i < ntiles; i++) {
                const int s = i % kStages;
                if (!mbar_wait(&conv[s], (i / kStages) & 1)) {
                    atomicOr(err, 4u);
                    s_abort = 1;
                    break;
                }
                if (*(volatile int*)&s_abort) break;
                tc_fence_after();
                const uint32_t a0 = smem_u32(smem + UmmaSmem::a_off(s));
                const uint32_t b0 = smem_u32(smem + UmmaSmem::b_off(s, N));
#pragma unroll
                for (int k = 0; k < kTileK / 16; k++)
                    umma_f16(tmem, umma_desc_sw128(a0 + k * 32), umma_desc_sw128(b0 + k * 32), idesc,
                             (i > 0 || k > 0) ? 1u : 0u);
                umma_commit(&freed[s]);
            }
            umma_commit(accb);  // arrives once every MMA issued above has completed
        }
    } else {
        // ---------------- converters (warps 2-5): row r of the 128-row tile
        const int q = warp & 3;
        const int r = q * 32 + lane;
        for (int i = 0; i < ntiles; i++) {
            const int s = i % kStages;
            if (!mbar_wait(&full[s], (i / kStages) & 1)) {
                atomicOr(err, 8u);
                s_abort = 1;
                break;
            }
            if (*(volatile int*)&s_abort) break;
            const uint8_t* wb = smem + UmmaSmem::w_off(s, N);
            uint8_t* ab = smem + UmmaSmem::a_off(s);
            const uint32_t dd = *reinterpret_cast<const uint32_t*>(wb + 8192 + r * 4);
            const __half2 d0 = __halves2half2(__ushort_as_half((unsigned short)(dd & 0xffffu)),
                                              __ushort_as_half((unsigned short)(dd & 0xffffu)));
            const __half2 d1 = __halves2half2(__ushort_as_half((unsigned short)(dd >> 16)),
                                              __ushort_as_half((unsigned short)(dd >> 16)));
            uint8_t* arow = ab + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const uint4 qv = *reinterpret_cast<const uint4*>(wb + ((size_t)c * kTileRows + r) * 16);
                const __half2 dh = c < 2 ? d0 : d1;
                uint32_t h[8];
                h[0] = q8_pair_to_h2<0x4140>(qv.x);
                h[1] = q8_pair_to_h2<0x4342>(qv.x);
                h[2] = q8_pair_to_h2<0x4140>(qv.y);
                h[3] = q8_pair_to_h2<0x4342>(qv.y);
                h[4] = q8_pair_to_h2<0x4140>(qv.z);
                h[5] = q8_pair_to_h2<0x4342>(qv.z);
                h[6] = q8_pair_to_h2<0x4140>(qv.w);
                h[7] = q8_pair_to_h2<0x4342>(qv.w);
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    __half2 x = *reinterpret_cast<__half2*>(&h[e]);
                    x = __hmul2(x, dh);
                    h[e] = *reinterpret_cast<uint32_t*>(&x);
                }
                const int j0 = 2 * c, j1 = 2 * c + 1;
                *reinterpret_cast<uint4*>(arow + ((j0 ^ (r & 7)) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
                *reinterpret_cast<uint4*>(arow + ((j1 ^ (r & 7)) << 4)) = make_uint4(h[4], h[5], h[6], h[7]);
            }
            fence_proxy_async_smem();
            mbar_arrive(&conv[s]);
        }
    }

    // ---------------- epilogue: warps 2-5 hold rows q*32 + lane
    float v[N];
    const bool epi = warp >= 2;
    bool have = false;
    if (epi) {
        const int q = warp & 3;
        if (!*(volatile int*)&s_abort && ntiles > 0) {
            if (mbar_wait(accb, 0)) {
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < N; c += 16) tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + c, v + c);
                have = true;
            } else {
                atomicOr(err, 16u);
                s_abort = 1;
            }
        } else if (ntiles <= 0) {
#pragma unroll
            for (int c = 0; c < N; c++) v[c] = 0.0f;
            have = true;
        }
    }
    // the MMA warp waits (bounded) for its own MMAs before TMEM is released
    if (warp == 1 && lane == 0 && *(volatile int*)&s_abort && ntiles > 0) {
        if (!mbar_wait(accb, 0)) atomicOr(err, 32u);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kCols);
        tmem_relinquish();
    }
    if (s_abort) return;

    const int r = (warp & 3) * 32 + lane;
    if (nsplit > 1) {
        if (epi && have) {
#pragma unroll
            for (int c = 0; c < N; c++) __stcg(&ws[(((size_t)split * MT + mt) * N + c) * kTileRows + r], v[c]);
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            const unsigned prev = atomicAdd(&tickets[mt], 1u);
            s_last = (prev == (unsigned)nsplit - 1u) ? 1u : 0u;
        }
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        if (epi) {
#pragma unroll
            for (int c = 0; c < N; c++) v[c] = 0.0f;
            for (int sp = 0; sp < nsplit; sp++)
#pragma unroll
                for (int c = 0; c < N; c++) v[c] += __ldcg(&ws[(((size_t)sp * MT + mt) * N + c) * kTileRows + r]);
        }
        if (threadIdx.x == 0) tickets[mt] = 0u;
    }
    if (!epi) return;

    if (ep.mode == EPI_SWIGLU) {
        // rows 0..63 of the tile are gate rows, 64..127 the matching up rows (q8t interleave)
        float* xch = reinterpret_cast<float*>(smem);  // operand buffers are free now
        if (r >= 64)
#pragma unroll
            for (int c = 0; c < N; c++) xch[c * 64 + (r - 64)] = v[c];
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (r < 64) {
            const int o = mt * 64 + r;
            if (o < ep.m_out) {
#pragma unroll
                for (int c = 0; c < N; c++) {
                    if (c >= batch) break;
                    const float g = v[c], u = xch[c * 64 + r];
                    const float h = (g / (1.0f + expf(-g))) * u;
                    act_store(ep.out, c, o, h);
                    if (ep.y) ep.y[(size_t)c * ep.ldy + o] = h;
                }
            }
        }
        return;
    }
    const int m = mt * kTileRows + r;
    if (m >= ep.m_out) return;
#pragma unroll
    for (int c = 0; c < N; c++) {
        if (c >= batch) break;
        float* yp = ep.y + (size_t)c * ep.ldy + m;
        if (ep.mode == EPI_RESID)
            *yp += v[c];
        else
            *yp = v[c];
    }
}

// ------------------------------------------------------------------------------ launcher
int umma_npad(int batch) { return batch <= 16 ? 16 : (batch <= 32 ? 32 : 64); }

// K splits so that the grid fills the two CTA slots of every SM once, with at least two K
// tiles per split and at most 8 splits (the last CTA of an m-tile sums the partials)
int umma_nsplit(int MT, int KT, int num_sms) {
    int s = (2 * num_sms) / MT;
    if (s > 8) s = 8;
    if (s > KT / 2) s = KT / 2;
    if (s <= 1) return 1;
    int per = (KT + s - 1) / s;
    return (KT + per - 1) / per;
}

size_t umma_ws_floats(int MT, int KT, int num_sms) {
    int ns = umma_nsplit(MT, KT, num_sms);
    return ns > 1 ? (size_t)ns * MT * 64 * kTileRows : 0;
}

template <int N>
static int launch_umma_t(const Q8Weight& w, const uint8_t* x16, int batch, float* ws, unsigned* tickets,
                         unsigned* err, const GemmEpi& ep, int num_sms, cudaStream_t st) {
    const int smem = UmmaSmem::bytes(N) + 1024;
    static bool attr_set[64] = {};  // per template instance and device, before the first launch
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev & 63]) {
        if (cudaFuncSetAttribute(q8_umma_gemm_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess)
            return -1;
        attr_set[dev & 63] = true;
    }
    const int ns = umma_nsplit(w.MT, w.KT, num_sms);
    const int per = (w.KT + ns - 1) / ns;
    dim3 grid(w.MT, ns);
    q8_umma_gemm_kernel<N><<<grid, kUmmaThreads, smem, st>>>(w.qt, w.KT, w.MT, x16, batch, per, ws, tickets, err, ep);
    return 0;
}

int launch_q8_umma(const Q8Weight& w, const uint8_t* x16, int batch, float* ws, unsigned* tickets, unsigned* err,
                   const GemmEpi& ep, int num_sms, cudaStream_t st) {
    switch (umma_npad(batch)) {
        case 16: return launch_umma_t<16>(w, x16, batch, ws, tickets, err, ep, num_sms, st);
        case 32: return launch_umma_t<32>(w, x16, batch, ws, tickets, err, ep, num_sms, st);
        default: return launch_umma_t<64>(w, x16, batch, ws, tickets, err, ep, num_sms, st);
    }
}

}  // namespace ab2
