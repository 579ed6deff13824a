// q8_umma.cu -- batched Q8_0 dequant-GEMM on the 5th-generation tensor cores (tcgen05).
//
// D[128 rows][N] = W[128 rows][K-range] * X[N][K-range]^T per CTA (N = batch padded to
// 16/32/64), with the accumulator in TMEM:
//   * warp 0 streams the 128x64 weight tiles (int8 + f16 scales, 8.5 KB each, contiguous in
//     the "q8t" layout) into an 8-deep ring with cp.async.bulk. Weights never depend on the
//     previous kernel, so under programmatic dependent launch this ring fills while the
//     predecessor is still running;
//   * warp 10 waits for the predecessor (griddepcontrol.wait) and streams the matching
//     activation tiles (already the swizzled shared-memory image, the "x16" layout);
//   * warps 2-9 turn each weight tile into the f16 A operand (w = q * d, one correctly
//     rounded f16 multiply of exact f16 values) in the K-major 128B-swizzled layout, release
//     the weight stage, fence the writes to the async proxy and hand the operand stage on
//     (a 4-deep A/B ring, so MMA completion latency stays off the critical path);
//   * warp 1 allocates TMEM and one lane issues tcgen05.mma (M=128, N, K=16) x4 per tile,
//     committing each operand stage back to its producers;
//   * warps 2-9 then read their TMEM lane quarter (half the columns each) and run the epilogue. With K split
//     across CTAs the partial sums are added with red.global.add into the residual stream
//     (or into an output the caller has zeroed); SwiGLU is never split.
// Every mbarrier wait is bounded; on a timeout the CTA records an error code, drains its
// own copies and MMAs (again bounded), frees its TMEM and returns.
#include "common.cuh"
#include "kernels.h"
#include "umma.cuh"

namespace ab2 {

constexpr int kTileRows = 128;
constexpr int kTileK = 64;
constexpr int kWTileBytes = 8192 + 512;  // [4 chunks][128 rows][16 B] int8 + [128 rows][2] f16
constexpr int kWStages = 8;              // raw weight ring (70 KB)
constexpr int kAStages = 4;              // f16 operand ring, A and B tiles (96 KB at N = 64)
constexpr int kWarpW = 0, kWarpMma = 1, kWarpConv0 = 2, kConvWarps = 8, kWarpB = 10;
constexpr int kUmmaThreads = 11 * 32;    // weights, MMA, 8 x convert + epilogue, activations

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
struct UmmaSmem {  // offsets from the 1024-aligned dynamic shared-memory base
    static constexpr int a_off(int s) { return s * 16384; }
    static constexpr int b_off(int s, int N) { return kAStages * 16384 + s * N * 128; }
    static constexpr int w_off(int s, int N) { return kAStages * (16384 + N * 128) + s * kWTileBytes; }
    static constexpr int bar_off(int N) { return w_off(kWStages, N); }
    // w_full[W], w_free[W], a_full[A], b_full[A], ab_free[A], acc, tmem slot
    static constexpr int n_bars() { return 2 * kWStages + 3 * kAStages + 1; }
    static constexpr int bytes(int N) { return bar_off(N) + n_bars() * 8 + 16; }
};

template <int N>
__global__ void __launch_bounds__(kUmmaThreads, 1)
    q8_umma_gemm_kernel(const uint8_t* __restrict__ wt, int KT, const uint8_t* __restrict__ x16, int batch,
                        int kt_per_split, unsigned* __restrict__ err, GemmEpi ep) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* w_full = reinterpret_cast<uint64_t*>(smem + UmmaSmem::bar_off(N));
    uint64_t* w_free = w_full + kWStages;
    uint64_t* a_full = w_free + kWStages;
    uint64_t* b_full = a_full + kAStages;
    uint64_t* ab_free = b_full + kAStages;
    uint64_t* accb = ab_free + kAStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accb + 1);
    __shared__ int s_abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = blockIdx.x, split = blockIdx.y, nsplit = gridDim.y;
    const int kt0 = split * kt_per_split, kt1 = min(KT, kt0 + kt_per_split);
    const int ntiles = kt1 - kt0;
    constexpr uint32_t kCols = N < 32 ? 32 : N;
    constexpr int kConvThreads = kConvWarps * 32;

    if (threadIdx.x == 0) {
        s_abort = 0;
        for (int s = 0; s < kWStages; s++) {
            mbar_init(&w_full[s], 1);
            mbar_init(&w_free[s], kConvThreads);
        }
        for (int s = 0; s < kAStages; s++) {
            mbar_init(&a_full[s], kConvThreads);
            mbar_init(&b_full[s], 1);
            mbar_init(&ab_free[s], 1);
        }
        mbar_init(accb, 1);
        mbar_fence_init();
    }
    if (warp == kWarpMma) tmem_alloc(tmem_slot, kCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_trigger();

    if (warp == kWarpW) {
        // ---------------- weight producer (independent of the predecessor kernel)
        if (lane == 0) {
            const uint8_t* wsrc = wt + ((size_t)mt * KT + kt0) * kWTileBytes;
            int i = 0;
            for (; i < ntiles; i++) {
                const int s = i % kWStages;
                if (i >= kWStages && !mbar_wait(&w_free[s], ((i / kWStages) - 1) & 1)) {
                    atomicOr(err, 1u);
                    s_abort = 1;
                    break;
                }
                if (*(volatile int*)&s_abort) break;
                mbar_arrive_expect_tx(&w_full[s], kWTileBytes);
                bulk_g2s(smem + UmmaSmem::w_off(s, N), wsrc + (size_t)i * kWTileBytes, kWTileBytes, &w_full[s]);
            }
            for (int j = max(0, i - kWStages); j < i; j++)  // issued copies land before exit
                if (!mbar_wait(&w_full[j % kWStages], (j / kWStages) & 1)) atomicOr(err, 2u);
        }
    } else if (warp == kWarpB) {
        // ---------------- activation producer (after the predecessor has completed)
        if (lane == 0) {
            pdl_wait();
            int i = 0;
            for (; i < ntiles; i++) {
                const int s = i % kAStages;
                if (i >= kAStages && !mbar_wait(&ab_free[s], ((i / kAStages) - 1) & 1)) {
                    atomicOr(err, 4u);
                    s_abort = 1;
                    break;
                }
                if (*(volatile int*)&s_abort) break;
                mbar_arrive_expect_tx(&b_full[s], N * 128);
                bulk_g2s(smem + UmmaSmem::b_off(s, N), x16 + (size_t)(kt0 + i) * N * 128, N * 128, &b_full[s]);
            }
            for (int j = max(0, i - kAStages); j < i; j++)
                if (!mbar_wait(&b_full[j % kAStages], (j / kAStages) & 1)) atomicOr(err, 8u);
        }
    } else if (warp == kWarpMma) {
        // ---------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(kTileRows, N);
            for (int i = 0; i < ntiles; i++) {
                const int s = i % kAStages;
                const uint32_t ph = (i / kAStages) & 1;
                if (!mbar_wait(&a_full[s], ph) || !mbar_wait(&b_full[s], ph)) {
                    atomicOr(err, 16u);
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
                umma_commit(&ab_free[s]);
            }
            umma_commit(accb);  // arrives once every MMA issued above has completed
        }
    } else {
        // ---------------- converters (warps 2..9): row r of the tile, 16-column chunks 2h, 2h+1
        const int r = (warp & 3) * 32 + lane;
        const int h = (warp - kWarpConv0) >> 2;
        for (int i = 0; i < ntiles; i++) {
            const int sw = i % kWStages, sa = i % kAStages;
            if (!mbar_wait(&w_full[sw], (i / kWStages) & 1) ||
                (i >= kAStages && !mbar_wait(&ab_free[sa], ((i / kAStages) - 1) & 1))) {
                atomicOr(err, 32u);
                s_abort = 1;
                break;
            }
            if (*(volatile int*)&s_abort) break;
            const uint8_t* wb = smem + UmmaSmem::w_off(sw, N);
            uint4 qv[2];
#pragma unroll
            for (int c = 0; c < 2; c++)
                qv[c] = *reinterpret_cast<const uint4*>(wb + ((size_t)(2 * h + c) * kTileRows + r) * 16);
            const uint32_t dd = *reinterpret_cast<const uint32_t*>(wb + 8192 + r * 4);
            mbar_arrive(&w_free[sw]);  // the raw weight stage has been read
            const unsigned short dbits = (unsigned short)(h ? (dd >> 16) : (dd & 0xffffu));
            const __half2 dh = __halves2half2(__ushort_as_half(dbits), __ushort_as_half(dbits));
            uint8_t* arow = smem + UmmaSmem::a_off(sa) + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
            for (int c = 0; c < 2; c++) {
                uint32_t hv[8];
                hv[0] = q8_pair_to_h2<0x4140>(qv[c].x);
                hv[1] = q8_pair_to_h2<0x4342>(qv[c].x);
                hv[2] = q8_pair_to_h2<0x4140>(qv[c].y);
                hv[3] = q8_pair_to_h2<0x4342>(qv[c].y);
                hv[4] = q8_pair_to_h2<0x4140>(qv[c].z);
                hv[5] = q8_pair_to_h2<0x4342>(qv[c].z);
                hv[6] = q8_pair_to_h2<0x4140>(qv[c].w);
                hv[7] = q8_pair_to_h2<0x4342>(qv[c].w);
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    __half2 x = *reinterpret_cast<__half2*>(&hv[e]);
                    x = __hmul2(x, dh);
                    hv[e] = *reinterpret_cast<uint32_t*>(&x);
                }
                const int j0 = 4 * h + 2 * c, j1 = j0 + 1;  // 8-column chunks of the 64-wide row
                *reinterpret_cast<uint4*>(arow + ((j0 ^ (r & 7)) << 4)) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
                *reinterpret_cast<uint4*>(arow + ((j1 ^ (r & 7)) << 4)) = make_uint4(hv[4], hv[5], hv[6], hv[7]);
            }
            fence_proxy_async_smem();
            mbar_arrive(&a_full[sa]);
        }
    }

    // ---------------- epilogue: converter warps; row q*32 + lane, columns [h*N/2, (h+1)*N/2)
    constexpr int CPH = N / 2;
    float v[CPH];
    const bool epi = warp >= kWarpConv0 && warp < kWarpConv0 + kConvWarps;
    const int h = epi ? (warp - kWarpConv0) >> 2 : 0;
    if (epi) {
        const int q = warp & 3;
        if (!*(volatile int*)&s_abort) {
            if (mbar_wait(accb, 0)) {
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < CPH; c += 8)
                    tmem_ld8(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * CPH + c), v + c);
            } else {
                atomicOr(err, 64u);
                s_abort = 1;
            }
        }
    }
    // the MMA lane waits (bounded) for its own MMAs before TMEM is released
    if (warp == kWarpMma && lane == 0 && *(volatile int*)&s_abort) {
        if (!mbar_wait(accb, 0)) atomicOr(err, 128u);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kWarpMma) {
        tc_fence_after();
        tmem_dealloc(tmem, kCols);
        tmem_relinquish();
    }
    if (s_abort || !epi) return;
    pdl_wait();  // outputs may be read or written by earlier kernels of the stream

    const int r = (warp & 3) * 32 + lane;
    const int c0 = h * CPH;
    if (ep.mode == EPI_SWIGLU) {
        // rows 0..63 of the tile are gate rows, 64..127 the matching up rows (q8t interleave)
        float* xch = reinterpret_cast<float*>(smem);  // the operand ring is idle now
        if (r >= 64)
#pragma unroll
            for (int c = 0; c < CPH; c++) xch[(c0 + c) * 64 + (r - 64)] = v[c];
        asm volatile("bar.sync 1, %0;" ::"n"(kConvThreads) : "memory");
        if (r < 64) {
            const int o = mt * 64 + r;
            if (o < ep.m_out) {
#pragma unroll
                for (int c = 0; c < CPH; c++) {
                    if (c0 + c >= batch) break;
                    const float g = v[c], u = xch[(c0 + c) * 64 + r];
                    const float hval = (g / (1.0f + expf(-g))) * u;
                    act_store(ep.out, c0 + c, o, hval);
                    if (ep.y) ep.y[(size_t)(c0 + c) * ep.ldy + o] = hval;
                }
            }
        }
        return;
    }
    const int m = mt * kTileRows + r;
    if (m >= ep.m_out) return;
#pragma unroll
    for (int c = 0; c < CPH; c++) {
        if (c0 + c >= batch) break;
        float* yp = ep.y + (size_t)(c0 + c) * ep.ldy + m;
        if (nsplit > 1)
            atomicAdd(yp, v[c]);  // result unused: compiles to a fire-and-forget reduction
        else if (ep.mode == EPI_RESID)
            *yp += v[c];
        else
            *yp = v[c];
    }
}

// ------------------------------------------------------------------------------ launcher
int umma_npad(int batch) { return batch <= 16 ? 16 : (batch <= 32 ? 32 : 64); }

// K splits so the grid covers the SMs about once (one CTA per SM), at least 4 K tiles per
// split and at most 16 splits. SwiGLU epilogues are never split.
int umma_nsplit(int MT, int KT, int mode, int num_sms) {
    if (mode == EPI_SWIGLU) return 1;
    int s = num_sms / MT;
    if (s > 16) s = 16;
    if (s > KT / 4) s = KT / 4;
    if (s <= 1) return 1;
    int per = (KT + s - 1) / s;
    return (KT + per - 1) / per;
}

template <int N>
static int launch_umma_t(const Q8Weight& w, const uint8_t* x16, int batch, unsigned* err, const GemmEpi& ep,
                         int num_sms, cudaStream_t st) {
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
    const int ns = umma_nsplit(w.MT, w.KT, ep.mode, num_sms);
    const int per = (w.KT + ns - 1) / ns;
    if (launch_pdl(q8_umma_gemm_kernel<N>, dim3(w.MT, ns), dim3(kUmmaThreads), smem, st, w.qt, w.KT, x16, batch,
                   per, err, ep) != cudaSuccess)
        return -2;
    return 0;
}

int launch_q8_umma(const Q8Weight& w, const uint8_t* x16, int batch, unsigned* err, const GemmEpi& ep, int num_sms,
                   cudaStream_t st) {
    switch (umma_npad(batch)) {
        case 16: return launch_umma_t<16>(w, x16, batch, err, ep, num_sms, st);
        case 32: return launch_umma_t<32>(w, x16, batch, err, ep, num_sms, st);
        default: return launch_umma_t<64>(w, x16, batch, err, ep, num_sms, st);
    }
}

}  // namespace ab2
