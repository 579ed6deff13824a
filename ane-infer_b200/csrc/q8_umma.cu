// q8_umma.cu -- batched Q8_0 dequant-GEMM on the 5th-generation tensor cores (tcgen05).
//
// Y[b][m] = sum_k X[b][k] W[m][k] for a batch of up to 64 sequences. The weights are the
// N = 256 side of every MMA and the activations the M = 64 side:
// D[64 x 256] (+)= X[64 x 16] W[256 x 16]^T, 4096 weights per instruction. Measured on B200,
// one tcgen05.mma of kind f16 takes about max(45, N/2) cycles whatever M (64 or 128).
// W is stored in 128-row x 64-column Q8_0 tiles (the "q8u" layout, 8.5 KB each) grouped in
// row-tile pairs: K tile kt of pair p is the contiguous 17 KB block (p*KT + kt)*17408. The
// work units are (pair, K split); a CTA takes units blockIdx.x, blockIdx.x + gridDim.x, ...
// (one unit per CTA for the layer weights, several for the vocabulary projection), and
// streams all of their K tiles through one pipeline:
//   * warp 5 copies one 17 KB pair block per stage into a 5-deep ring (copies of 16 KB or
//     more are needed to reach HBM bandwidth). Weights never depend on the previous kernel,
//     so under programmatic dependent launch the ring fills while the predecessor runs;
//   * warp 9 waits for the predecessor (griddepcontrol.wait) and copies the activations,
//     already the swizzled shared-memory image, four K tiles (32 KB) at a time. Each
//     activation tile serves 256 weight rows, so it costs half a byte per weight byte;
//   * eight converter warps (one weight row per thread) turn the raw tiles into the f16 B
//     operand (w = q*d, one correctly rounded f16 multiply of exact f16 values), K-major with
//     the 128-byte swizzle;
//   * warp 1 allocates TMEM and one lane issues 4 x tcgen05.mma (M=64, N=256, K=16) per
//     stage into one of two TMEM accumulators, alternating per unit so the epilogue of one
//     unit overlaps the MMAs of the next;
//   * four epilogue warps drain the accumulators (TMEM lanes 0-15 of each warp's quarter hold
//     16 batch rows). A unit covering all of K writes its outputs (STORE y = Wx, RESID
//     y += Wx). Units of a K split, and every unit of an EPI_ADD call, add their partial sums
//     into y with fire-and-forget vector reductions (the caller zeroes a STORE output; an
//     EPI_ADD output is kept zeroed by its consumer). The SwiGLU gate/up projection runs as
//     EPI_ADD into an f32 scratch, followed by launch_glu.
// Every mbarrier wait is bounded; on a timeout the CTA records an error code, drains its
// own copies and MMAs (again bounded), frees its TMEM and returns.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "umma.cuh"

namespace ab2 {

constexpr int kRows = kUTileRows;                 // 128 weight rows per tile
constexpr int kPairRows = 2 * kRows;              // 256 weight rows per unit (the MMA's N)
constexpr int kTileK = 64;
constexpr int kBatchRows = 64;                    // the MMA's M: activation rows (batch padded to 64)
constexpr int kStageTiles = 2;                    // weight tiles per pipeline stage: one K tile of a pair
constexpr int kWStageBytes = kStageTiles * kUTileBytes;
constexpr int kWStages = 5;                       // raw weight ring (85 KB)
constexpr int kBStages = 2;                       // f16 weight operand ring (64 KB)
constexpr int kAGroup = 4;                        // activation K tiles per copy
constexpr int kAStages = 2;                       // activation ring (64 KB)
constexpr int kBTileBytes = kRows * kTileK * 2;   // 16 KB
constexpr int kATileBytes = kBatchRows * kTileK * 2;  // 8 KB
// Warp roles. A warp runs on scheduler (warp % 4); the MMA warp's scheduler gets only the
// light roles (the two copy producers and one epilogue warp), so its single issuing thread
// is not slowed by the always-busy converter warps. Epilogue warp w reads TMEM lanes
// 32*(w % 4) .. +31, so the four epilogue warps cover the four residues.
constexpr int kWarpMma = 1, kWarpW = 5, kWarpA = 9, kConvWarps = 8, kEpiWarps = 4;
__device__ __forceinline__ int conv_index(int warp) {  // converter warps 0,2,3,4,6,7,8,10 -> 0..7, else -1
    switch (warp) {
        case 0: return 0;
        case 2: return 1;
        case 3: return 2;
        case 4: return 3;
        case 6: return 4;
        case 7: return 5;
        case 8: return 6;
        case 10: return 7;
        default: return -1;
    }
}
__device__ __forceinline__ bool is_epi(int warp) { return warp >= 11; }
__device__ __forceinline__ int epi_index(int warp) { return warp - 11; }
constexpr int kUmmaThreads = 15 * 32;
constexpr uint32_t kTmemCols = 512;               // two accumulators of 256 columns
constexpr int kEpiBar = 1;                        // named barrier of the epilogue warps
constexpr int kStageLd = kPairRows + 4;           // floats per staged accumulator row (16-byte pad)
constexpr int kMinKTilesPerSplit = 4;
static_assert(kConvWarps * 32 == kStageTiles * kRows, "one converter thread per weight row of a stage");

// ------------------------------------------------------------------------------ repack
// one thread per source (row, Q8_0 block): row -> dst row R = base + (row/grp)*stride + row%grp,
// block kb -> tile kt = kb/2, chunks 2*(kb%2) and 2*(kb%2)+1, scale slot kb%2
__global__ void q8u_repack_kernel(const uint8_t* __restrict__ src, int64_t rows, int KB, uint8_t* __restrict__ dst,
                                  int KT, int64_t base, int64_t grp, int64_t stride) {
    int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (id >= rows * KB) return;
    const int64_t r = id / KB;
    const int kb = (int)(id % KB);
    const uint8_t* blk = src + id * 34;
    const int64_t R = base + (r / grp) * stride + (r % grp);
    const int64_t mt = R / kRows;
    const int rr = (int)(R % kRows);
    const int kt = kb >> 1, half = kb & 1;
    uint8_t* tile = dst + (((size_t)(mt >> 1) * KT + kt) * 2 + (mt & 1)) * kUTileBytes;
#pragma unroll
    for (int c2 = 0; c2 < 2; c2++) {
        uint8_t* chunk = tile + ((size_t)(half * 2 + c2) * kRows + rr) * 16;
#pragma unroll
        for (int i = 0; i < 16; i++) chunk[i] = (uint8_t)(blk[2 + c2 * 16 + i] ^ 0x80u);
    }
    tile[4 * kRows * 16 + rr * 4 + half * 2 + 0] = blk[0];
    tile[4 * kRows * 16 + rr * 4 + half * 2 + 1] = blk[1];
}

void launch_q8t_repack(const uint8_t* src, int64_t rows, int KB, Q8Weight& w, int64_t base, int64_t grp,
                       int64_t stride, cudaStream_t st) {
    int64_t n = rows * KB;
    q8u_repack_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(src, rows, KB, w.qt, w.KT, base, grp, stride);
}

// ------------------------------------------------------------------------------ kernel
struct UmmaSmem {  // offsets from the 1024-aligned dynamic shared-memory base
    static constexpr int w_off(int s) { return s * kWStageBytes; }
    static constexpr int b_base() { return (kWStages * kWStageBytes + 1023) / 1024 * 1024; }
    static constexpr int b_off(int s) { return b_base() + s * kStageTiles * kBTileBytes; }
    static constexpr int a_off(int s) { return b_off(kBStages) + s * kAGroup * kATileBytes; }
    static constexpr int bar_off() { return a_off(kAStages); }
    // w_full/w_free[W], b_full/b_free[B], a_full/a_free[A], acc_full/acc_free[2], mma_done, tmem slot
    static constexpr int n_bars() { return 2 * kWStages + 2 * kBStages + 2 * kAStages + 4 + 1; }
    static constexpr int bytes() { return bar_off() + n_bars() * 8 + 16; }
};
static_assert(kBTileBytes % 1024 == 0 && kATileBytes % 1024 == 0, "operand tiles must stay 1024-aligned");
static_assert(kBatchRows * kStageLd * 4 <= UmmaSmem::bar_off() - UmmaSmem::b_off(0),
              "the staged accumulator fits in the operand rings");

// Unit u = (row tile u / KS, K split u % KS) covers the len K tiles from k0. A CTA takes
// units blockIdx.x, blockIdx.x + G, ...; every role walks them with plain nested loops
// (pipeline stages and activation groups never span two units), because per-tile
// bookkeeping in the issuing threads sits directly on the pipeline's critical path.
__device__ __forceinline__ void unit_range(int u, int KS, int kper, int KT, int& mt, int& k0, int& len) {
    mt = u / KS;
    k0 = (u % KS) * kper;
    len = min(KT, k0 + kper) - k0;
}

// 32 lanes x 32 columns of f32 from TMEM (this warp's lane quarter)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float v[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// fire-and-forget vector reduction into global memory (no value returned, so consecutive
// reductions of a thread do not wait for one another)
__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}

// 32 consecutive outputs y[m0 .. m0+31] of one batch row (m0 a multiple of 32):
// mode 0 store, 1 add in place, 2 add with reductions (other CTAs add to the same outputs)
__device__ __forceinline__ void epi_out32(float* __restrict__ yrow, int m0, int m_out, int how, const float v[32]) {
    if (m0 + 32 <= m_out && (reinterpret_cast<uintptr_t>(yrow + m0) & 15) == 0) {
        float4* p = reinterpret_cast<float4*>(yrow + m0);
#pragma unroll
        for (int j = 0; j < 8; j++) {
            float4 o = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            if (how == 2) {
                red_add_v4(yrow + m0 + 4 * j, o.x, o.y, o.z, o.w);
                continue;
            }
            if (how == 1) {
                const float4 a = p[j];
                o.x += a.x;
                o.y += a.y;
                o.z += a.z;
                o.w += a.w;
            }
            p[j] = o;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; j++) {
            if (m0 + j >= m_out) break;
            if (how == 2)
                atomicAdd(yrow + m0 + j, v[j]);  // result unused: compiles to a reduction
            else
                yrow[m0 + j] = how == 1 ? yrow[m0 + j] + v[j] : v[j];
        }
    }
}

__global__ void __launch_bounds__(kUmmaThreads, 1)
    q8_umma_gemm_kernel(const uint8_t* __restrict__ wt, int MP, int KT, int KS, const uint8_t* __restrict__ x16,
                        int batch, unsigned* __restrict__ err, GemmEpi ep) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* w_full = reinterpret_cast<uint64_t*>(smem + UmmaSmem::bar_off());
    uint64_t* w_free = w_full + kWStages;
    uint64_t* b_full = w_free + kWStages;
    uint64_t* b_free = b_full + kBStages;
    uint64_t* a_full = b_free + kBStages;
    uint64_t* a_free = a_full + kAStages;
    uint64_t* acc_full = a_free + kAStages;
    uint64_t* acc_free = acc_full + 2;
    uint64_t* mma_done = acc_free + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
    __shared__ int s_abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, U = MP * KS;  // MP row-tile pairs
    const int kper = (KT + KS - 1) / KS;

    if (threadIdx.x == 0) {
        s_abort = 0;
        for (int s = 0; s < kWStages; s++) {
            mbar_init(&w_full[s], 1);
            mbar_init(&w_free[s], kConvWarps * 32);
        }
        for (int s = 0; s < kBStages; s++) {
            mbar_init(&b_full[s], kConvWarps * 32);
            mbar_init(&b_free[s], 1);
        }
        for (int s = 0; s < kAStages; s++) {
            mbar_init(&a_full[s], 1);
            mbar_init(&a_free[s], 1);
        }
        for (int j = 0; j < 2; j++) {
            mbar_init(&acc_full[j], 1);
            mbar_init(&acc_free[j], kEpiWarps * 32);
        }
        mbar_init(mma_done, 1);
        mbar_fence_init();
    }
    if (warp == kWarpMma) tmem_alloc(tmem_slot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_trigger();

    if (warp == kWarpW) {
        // ---------------- weight producer (independent of the predecessor kernel)
        if (lane == 0) {
            int st = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < U && ok; u += G) {
                int mt, k0, len;
                unit_range(u, KS, kper, KT, mt, k0, len);
                const uint8_t* src = wt + ((size_t)mt * KT + k0) * kWStageBytes;  // the unit's blocks are contiguous
                for (int q = 0; q < len; q++, st++) {
                    const int s = st % kWStages;
                    // once the ring is full, pull this CTA's share of the next GEMM's weights
                    // into L2 (this launch is latency-bound, so the extra HBM reads are free)
                    if (st == kWStages) prefetch_share_l2(ep.pf, ep.pf_bytes, blockIdx.x, G);
                    if (st >= kWStages && !mbar_wait(&w_free[s], ((st / kWStages) - 1) & 1)) {
                        atomicOr(err, 1u);
                        s_abort = 1;
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&w_full[s], kWStageBytes);
                    bulk_g2s(smem + UmmaSmem::w_off(s), src + (size_t)q * kWStageBytes, kWStageBytes, &w_full[s]);
                }
            }
            if (st <= kWStages) prefetch_share_l2(ep.pf, ep.pf_bytes, blockIdx.x, G);
            for (int j = max(0, st - kWStages); j < st; j++)  // issued copies land before exit
                if (!mbar_wait(&w_full[j % kWStages], (j / kWStages) & 1)) atomicOr(err, 2u);
        }
    } else if (warp == kWarpA) {
        // ---------------- activation producer (after the predecessor has completed)
        if (lane == 0) {
            pdl_wait();
            int g = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < U && ok; u += G) {
                int mt, k0, len;
                unit_range(u, KS, kper, KT, mt, k0, len);
                for (int q = 0; q < len; q += kAGroup, g++) {
                    const int s = g % kAStages;
                    if (g >= kAStages && !mbar_wait(&a_free[s], ((g / kAStages) - 1) & 1)) {
                        atomicOr(err, 4u);
                        s_abort = 1;
                        ok = false;
                        break;
                    }
                    const uint32_t bytes = (uint32_t)min(kAGroup, len - q) * kATileBytes;
                    mbar_arrive_expect_tx(&a_full[s], bytes);
                    bulk_g2s(smem + UmmaSmem::a_off(s), x16 + (size_t)(k0 + q) * kATileBytes, bytes, &a_full[s]);
                }
            }
            for (int j = max(0, g - kAStages); j < g; j++)
                if (!mbar_wait(&a_full[j % kAStages], (j / kAStages) & 1)) atomicOr(err, 8u);
        }
    } else if (warp == kWarpMma) {
        // ---------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(kBatchRows, kPairRows);
            int st = 0, g = 0, j = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < U && ok; u += G, j++) {
                int mt, k0, len;
                unit_range(u, KS, kper, KT, mt, k0, len);
                if (j >= 2) {
                    if (!mbar_wait(&acc_free[j & 1], ((j >> 1) - 1) & 1)) {
                        atomicOr(err, 16u);
                        ok = false;
                        break;
                    }
                    tc_fence_after();  // the epilogue's TMEM loads of this accumulator are done
                }
                const uint32_t d = tmem + (uint32_t)((j & 1) * kPairRows);
                for (int q = 0; q < len; q++, st++) {
                    const int sb = st % kBStages, ua = q % kAGroup, sa = g % kAStages;
                    if (!mbar_wait(&b_full[sb], (st / kBStages) & 1) ||
                        (ua == 0 && !mbar_wait(&a_full[sa], (g / kAStages) & 1))) {
                        atomicOr(err, 32u);
                        ok = false;
                        break;
                    }
                    // the pair's two 128-row operand tiles are adjacent: one N = 256 operand
                    const uint32_t a0 = smem_u32(smem + UmmaSmem::a_off(sa) + ua * kATileBytes);
                    const uint32_t b0 = smem_u32(smem + UmmaSmem::b_off(sb));
#pragma unroll
                    for (int k = 0; k < kTileK / 16; k++)
                        umma_f16(d, umma_desc_sw128(a0 + k * 32), umma_desc_sw128(b0 + k * 32), idesc,
                                 (q > 0 || k > 0) ? 1u : 0u);
                    if (ua == kAGroup - 1 || q == len - 1) {
                        umma_commit(&a_free[sa]);
                        g++;
                    }
                    umma_commit(&b_free[sb]);
                }
                umma_commit(&acc_full[j & 1]);
            }
            if (!ok) s_abort = 1;
            umma_commit(mma_done);  // every MMA issued above has completed before TMEM is freed
            if (!mbar_wait(mma_done, 0)) atomicOr(err, 64u);
        }
    } else if (conv_index(warp) >= 0) {
        // ---------------- converters: weight row r of stage tile t -> one 128-byte swizzled row
        const int ci = conv_index(warp);
        const int t = ci >> 2;
        const int r = (ci & 3) * 32 + lane;
        int st = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < U && ok; u += G) {
          int mt, k0, len;
          unit_range(u, KS, kper, KT, mt, k0, len);
          for (int q = 0; q < len; q++, st++) {
            const int sw = st % kWStages, sb = st % kBStages;
            const bool mine = true;
            if (!mbar_wait(&w_full[sw], (st / kWStages) & 1)) {
                atomicOr(err, 128u);
                s_abort = 1;
                ok = false;
                break;
            }
            const uint8_t* wb = smem + UmmaSmem::w_off(sw) + t * kUTileBytes;
            uint4 qv[4];
            uint32_t dd = 0;
            if (mine) {
#pragma unroll
                for (int c = 0; c < 4; c++)
                    qv[c] = *reinterpret_cast<const uint4*>(wb + ((size_t)c * kRows + r) * 16);
                dd = *reinterpret_cast<const uint32_t*>(wb + 4 * kRows * 16 + r * 4);
            }
            uint32_t hv[4][8];
            if (mine) {
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const unsigned short dbits = (unsigned short)(c >= 2 ? (dd >> 16) : (dd & 0xffffu));
                    const __half2 dh = __halves2half2(__ushort_as_half(dbits), __ushort_as_half(dbits));
                    q8_unpack(qv[c], hv[c]);
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        __half2 x = *reinterpret_cast<__half2*>(&hv[c][e]);
                        x = __hmul2(x, dh);
                        hv[c][e] = *reinterpret_cast<uint32_t*>(&x);
                    }
                }
            }
            if (st >= kBStages && !mbar_wait(&b_free[sb], ((st / kBStages) - 1) & 1)) {
                atomicOr(err, 256u);
                s_abort = 1;
                ok = false;
                break;
            }
            if (mine) {
                // row r of the K-major 128B-swizzled operand: 16-byte chunk j (k 8j..8j+7) at j ^ (r % 8)
                uint8_t* brow = smem + UmmaSmem::b_off(sb) + t * kBTileBytes + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const int j0 = 2 * c, j1 = 2 * c + 1;
                    *reinterpret_cast<uint4*>(brow + ((j0 ^ (r & 7)) << 4)) =
                        make_uint4(hv[c][0], hv[c][1], hv[c][2], hv[c][3]);
                    *reinterpret_cast<uint4*>(brow + ((j1 ^ (r & 7)) << 4)) =
                        make_uint4(hv[c][4], hv[c][5], hv[c][6], hv[c][7]);
                }
                fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
            }
            // The raw stage is released only after the converted values have been stored: those
            // stores consume the registers loaded from it, so the loads have completed. Arriving
            // right after issuing the loads let the next copy into the slot overwrite bytes that
            // a load had not read yet. Every writing thread arrives after its own proxy fence, so
            // the MMA issued after the phase completes reads what each of them wrote.
            mbar_arrive(&w_free[sw]);
            mbar_arrive(&b_full[sb]);
          }
        }
    } else if (is_epi(warp)) {
        // ---------------- epilogue warps: TMEM lanes 32q .. 32q+15 hold batch rows 16q .. 16q+15
        const int q = warp & 3;
        const int b = q * 16 + (lane & 15);
        const bool row_ok = lane < 16 && b < batch;
        const int how = (KS > 1 || ep.mode == EPI_ADD) ? 2 : (ep.mode == EPI_RESID ? 1 : 0);
        pdl_wait();  // outputs may be read or written by earlier kernels of the stream
        for (int j = 0, u = blockIdx.x; u < U; j++, u += G) {
            if (!mbar_wait(&acc_full[j & 1], (j >> 1) & 1)) {
                atomicOr(err, 512u);
                s_abort = 1;
                break;
            }
            if (*(volatile int*)&s_abort) break;
            tc_fence_after();
            const uint32_t dq = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)((j & 1) * kPairRows);
            const int pr = u / KS;  // row-tile pair: rows pr*256 .. pr*256+255
            if (u + G < U) {
                // more units follow: the operand rings are busy, write from the TMEM rows
#pragma unroll 1
                for (int c = 0; c < kPairRows; c += 32) {
                    float v[32];
                    tmem_ld32(dq + c, v);
                    if (row_ok) epi_out32(ep.y + (size_t)b * ep.ldy, pr * kPairRows + c, ep.m_out, how, v);
                }
                tc_fence_before();
                mbar_arrive(&acc_free[j & 1]);  // this thread's TMEM loads are done
                continue;
            }
            // The last unit: the operand rings are idle (every MMA of the CTA has completed, and
            // every copy into them landed before its MMA), so the accumulator is staged there as
            // [64 rows][kStageLd floats]; the 16-byte pad per row keeps the lane-per-row stores at
            // most 2-way bank conflicted. Each batch row's outputs then leave in one bulk
            // operation: a bulk store, or a bulk f32 add at L2 when the output accumulates
            // (K splits, residual). Per-thread 16-byte reductions of the same data were bound
            // by the L2's atomic rate when all CTAs reached their epilogue together.
            float* stage = reinterpret_cast<float*>(smem + UmmaSmem::b_off(0));
            const int r = q * 16 + (lane & 15);
#pragma unroll 1
            for (int c = 0; c < kPairRows; c += 32) {
                float v[32];
                tmem_ld32(dq + c, v);
                if (lane < 16)
#pragma unroll
                    for (int e = 0; e < 8; e++)
                        *reinterpret_cast<float4*>(stage + r * kStageLd + c + 4 * e) =
                            make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
            }
            fence_proxy_async_smem();  // the bulk operations read the staged rows through the async proxy
            tc_fence_before();
            asm volatile("bar.sync %0, %1;" ::"n"(kEpiBar), "n"(kEpiWarps * 32) : "memory");
            const int et = threadIdx.x - 11 * 32;  // 0..127
            const int m0 = pr * kPairRows, valid = min(kPairRows, ep.m_out - m0);
            const bool vec = (ep.ldy & 3) == 0;
            if (valid > 0 && (valid & 3) == 0 && vec && (reinterpret_cast<uintptr_t>(ep.y) & 15) == 0) {
                if (et < 32) {
                    for (int rr = et; rr < batch; rr += 32) {
                        float* dst = ep.y + (size_t)rr * ep.ldy + m0;
                        if (how == 0)
                            bulk_s2g(dst, stage + rr * kStageLd, (uint32_t)valid * 4);
                        else
                            bulk_reduce_add_f32(dst, stage + rr * kStageLd, (uint32_t)valid * 4);
                    }
                    bulk_commit();
                    bulk_wait_all();
                }
                continue;
            }
            for (int rr = et >> 6; rr < batch; rr += 2) {  // two rows per pass, 64 float4 each
                const int c4 = et & 63;
                const int m = m0 + c4 * 4;
                if (m >= ep.m_out) continue;
                const float4 v = *reinterpret_cast<const float4*>(stage + rr * kStageLd + c4 * 4);
                float* yp = ep.y + (size_t)rr * ep.ldy + m;
                if (vec && m + 4 <= ep.m_out) {
                    if (how == 2) {
                        red_add_v4(yp, v.x, v.y, v.z, v.w);
                    } else {
                        float4 o = v;
                        if (how == 1) {
                            const float4 a = *reinterpret_cast<const float4*>(yp);
                            o.x += a.x;
                            o.y += a.y;
                            o.z += a.z;
                            o.w += a.w;
                        }
                        *reinterpret_cast<float4*>(yp) = o;
                    }
                } else {
                    const float vv[4] = {v.x, v.y, v.z, v.w};
                    for (int e = 0; e < 4 && m + e < ep.m_out; e++) {
                        if (how == 2)
                            atomicAdd(yp + e, vv[e]);
                        else
                            yp[e] = how == 1 ? yp[e] + vv[e] : vv[e];
                    }
                }
            }
        }
    }

    // reconverge each warp first: in the producer and MMA warps lane 0 alone ran the role loop,
    // and a CTA barrier reached by part of a warp is not a barrier for the rest of it
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == kWarpMma) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
        tmem_relinquish();
    }
}

// ------------------------------------------------------------------------------ launcher
// K splits so the units (row tile, split) cover the SMs about once, each split at least
// kMinKTilesPerSplit K tiles. SwiGLU epilogues are never split.
int umma_nsplit(int MT, int KT, int mode, int num_sms) {
    (void)mode;
    const int pairs = (MT + 1) / 2;
    int s = std::min(num_sms / pairs, KT / kMinKTilesPerSplit);
    if (s <= 1) return 1;
    const int per = (KT + s - 1) / s;
    return (KT + per - 1) / per;
}

int launch_q8_umma(const Q8Weight& w, const uint8_t* x16, int batch, unsigned* err, const GemmEpi& ep, int num_sms,
                   cudaStream_t st) {
    const int smem = UmmaSmem::bytes() + 1024;
    static bool attr_set[64] = {};  // per device, before the first launch
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev & 63]) {
        if (cudaFuncSetAttribute(q8_umma_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess)
            return -1;
        attr_set[dev & 63] = true;
    }
    if (ep.mode == EPI_SWIGLU) return -3;  // SwiGLU runs as EPI_ADD + launch_glu on this path
    const int KS = umma_nsplit(w.MT, w.KT, ep.mode, num_sms);
    const int pairs = (w.MT + 1) / 2;
    const int U = pairs * KS;
    const int G = std::min(U, num_sms);
    if (launch_pdl(q8_umma_gemm_kernel, dim3(G), dim3(kUmmaThreads), smem, st, w.qt, pairs, w.KT, KS, x16, batch, err,
                   ep) != cudaSuccess)
        return -2;
    return 0;
}

}  // namespace ab2
