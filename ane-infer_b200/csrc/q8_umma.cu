// q8_umma.cu -- batched Q8_0 dequant-GEMM on the 5th-generation tensor cores (tcgen05).
//
// Y[b][m] = sum_k X[b][k] W[m][k] for a batch of up to 64 sequences (or the up to 128 tokens
// of a prefill step). The weights are the A side of every MMA, taken from tensor memory, and
// the activations the N = 64 (or 128) side, taken from shared memory: D[128 x N] (+)=
// W[128 x 16] X[N x 16]^T, two 128-row weight tiles per stage. Keeping the converted f16 weights out of shared memory halves its traffic per
// stage (17 KB raw weights in and out, 16 KB of activation reads), which is what bounded
// the shared-memory-operand form of this kernel.
// W is stored in 128-row x 64-column Q8_0 tiles (the "q8u" layout, 8.5 KB each) grouped in
// row-tile pairs: K tile kt of pair p is the contiguous 17 KB block (p*KT + kt)*17408. The
// work units are (pair, K split); a CTA takes units blockIdx.x, blockIdx.x + gridDim.x, ...
// (one unit per CTA for the layer weights, several for the vocabulary projection), and
// streams all of their K tiles through one pipeline:
//   * warp 13 copies one 17 KB pair block per stage into an 8-deep ring (copies of 16 KB or
//     more are needed to reach HBM bandwidth). Weights never depend on the previous kernel,
//     so under programmatic dependent launch the ring fills while the predecessor runs;
//   * warp 14 waits for the predecessor (griddepcontrol.wait) and copies the activations,
//     already the swizzled shared-memory image, four K tiles (32 KB) at a time;
//   * warps 0-7 (one weight row per thread, two warps per TMEM lane quarter) turn the raw
//     tiles into f16 (w = q*d, one correctly rounded f16 multiply of exact f16 values) and
//     store them into a 4-slot operand ring in tensor memory with tcgen05.st;
//   * warp 12 allocates TMEM and one lane issues 8 x tcgen05.mma (M=128, N=64, K=16, A in
//     TMEM) per stage into one of two TMEM accumulators, alternating per unit so the
//     epilogue of one unit overlaps the MMAs of the next;
//   * warps 8-11 drain the accumulators (TMEM lane = weight row, column = batch row). A unit
//     covering all of K writes its outputs (STORE y = Wx, RESID y += Wx); units of a K split,
//     and every unit of an EPI_ADD call, add their partial sums into y (the caller zeroes a
//     STORE output or an EPI_ADD output before the launch).
// SwiGLU FFN: the gate/up projection runs as EPI_ADD into an f32 scratch h2 (gate and up rows
// interleaved per 64), and the down projection takes its activations from h2 itself: warps
// 8-11, idle until the first accumulator is ready, compute x = silu(g) * u per K tile straight
// into the swizzled f16 image in shared memory (the activation ring as 8 one-tile slots), in
// place of warp 14's copies of a prepared image.
// Every mbarrier wait is bounded; on a timeout the CTA records an error code, drains its
// own copies and MMAs (again bounded), frees its TMEM and returns.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "umma.cuh"

namespace ab2 {

constexpr int kRows = kUTileRows;                 // 128 weight rows per tile (the MMA's M)
constexpr int kPairRows = 2 * kRows;              // 256 weight rows per unit
constexpr int kTileK = 64;
constexpr int kMaxBatchRows = 128;                // the MMA's N: activation rows (a step's batch padded to 64, a
                                                  // prefill step's tokens to 128)
constexpr int kStageTiles = 2;                    // weight tiles per pipeline stage: one K tile of a pair
constexpr int kWStageBytes = kStageTiles * kUTileBytes;
constexpr int kWStages = 8;                       // raw weight ring (136 KB)
constexpr int kXStages = 2;                       // activation ring: two stages of 32 KB
constexpr int kXRingBytes = 64 * 1024;
constexpr int kXSlotsMax = 8;                     // barrier slots of the ring as one-tile slots (SwiGLU source)
// The activation side for NB = 64 or 128 rows: a K tile of the image is NB rows of 128 bytes,
// a copy brings a 32 KB group of them, and the TMEM accumulators of a unit (two weight tiles
// x NB f32 columns) are double-buffered at NB = 64; at NB = 128 one accumulator fills the 256
// columns beside the operand ring, so a unit's MMAs wait for the previous unit's epilogue.
template <int NB>
struct XShape {
    static_assert(NB == 64 || NB == 128, "64 or 128 activation rows");
    static constexpr int kTileBytes = NB * kTileK * 2;  // 8 or 16 KB
    static constexpr int kGroup = kXRingBytes / kXStages / kTileBytes;  // K tiles per copy: 4 or 2
    static constexpr int kSlots = kXStages * kGroup;
    static constexpr int kAccBufs = NB == 64 ? 2 : 1;
    static constexpr int kAccCols = 2 * NB;  // one accumulator: kStageTiles tiles of NB columns
};
constexpr int kOpStages = 4;                      // f16 weight operand ring in TMEM
// TMEM columns: the operand ring in [0, 256) (stage s, tile t at s*64 + t*32: 32 columns hold
// a row's 64 f16 of K), the two accumulators in [256, 512) (unit buffer j at 256 + j*128,
// tile t at + t*64: one f32 column per batch row)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kOpCol0 = 0, kAccCol0 = 256;
// Warp roles: converter warp w < 8 takes tile w / 4 and the TMEM lane quarter w % 4 (a warp
// reaches the lanes 32 * (w % 4) .. + 31 only); epilogue warp 8 + q reads quarter q.
constexpr int kConvWarps = 8, kWarpEpi0 = 8, kEpiWarps = 4, kWarpMma = 12, kWarpW = 13, kWarpX = 14;
constexpr int kUmmaThreads = 15 * 32;
constexpr int kEpiBar = 1;                        // named barrier of the epilogue warps
constexpr int kStageLd = kPairRows + 4;           // floats per staged accumulator row (16-byte pad)
constexpr int kMinKTilesPerSplit = 4;
static_assert(kConvWarps * 32 == kStageTiles * kRows, "one converter thread per weight row of a stage");
static_assert(kOpStages * kStageTiles * 32 <= (int)kAccCol0 &&
                  kAccCol0 + XShape<64>::kAccBufs * XShape<64>::kAccCols <= kTmemCols &&
                  kAccCol0 + XShape<128>::kAccBufs * XShape<128>::kAccCols <= kTmemCols,
              "TMEM column budget");

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
    static constexpr int x_base() { return (kWStages * kWStageBytes + 1023) / 1024 * 1024; }
    // activation stage s of xg K tiles of tb bytes (xg = the copy group for copied images, 1 for
    // the SwiGLU source)
    static constexpr int x_off(int s, int xg, int tb) { return x_base() + s * xg * tb; }
    static constexpr int bar_off() { return x_base() + kXRingBytes; }
    // w_full/w_free[W], op_full/op_free[Op], x_full/x_free[kXSlotsMax], acc_full/acc_free[2], mma_done, tmem slot
    static constexpr int n_bars() { return 2 * kWStages + 2 * kOpStages + 2 * kXSlotsMax + 4 + 1; }
    static constexpr int bytes() { return bar_off() + n_bars() * 8 + 16; }
};
static_assert(XShape<64>::kTileBytes % 1024 == 0 && UmmaSmem::x_base() % 1024 == 0 &&
                  XShape<64>::kSlots <= kXSlotsMax && XShape<128>::kSlots <= kXSlotsMax,
              "operand tiles must stay 1024-aligned");
// the last unit's accumulator is staged over the raw weight ring, idle by then
static_assert(kMaxBatchRows * kStageLd * 4 <= UmmaSmem::x_base(), "the staged accumulator fits in the weight ring");

// Unit u covers the len K tiles from k0 of row-tile pair mt: a main unit (pair u / ks, K split
// u % ks) or, from main_units on, a K piece of one of the tail pairs. A CTA takes units
// blockIdx.x, blockIdx.x + G, ...; every role walks them with plain nested loops (pipeline
// stages and activation groups never span two units), because per-tile bookkeeping in the
// issuing threads sits directly on the pipeline's critical path. `split`: other units cover
// the same pair, so this one adds its partial sums into the output.
struct UnitPlan {
    int KT, ks, kper, main_units, first_tail, ks_tail, kper_tail, units;
};
__device__ __forceinline__ void unit_range(int u, const UnitPlan& P, int& mt, int& k0, int& len, bool& split) {
    if (u < P.main_units) {
        mt = u / P.ks;
        k0 = (u % P.ks) * P.kper;
        len = min(P.KT, k0 + P.kper) - k0;
        split = P.ks > 1;
    } else {
        const int t = u - P.main_units;
        mt = P.first_tail + t / P.ks_tail;
        k0 = (t % P.ks_tail) * P.kper_tail;
        len = min(P.KT, k0 + P.kper_tail) - k0;
        split = true;
    }
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

// 32 lanes x 64 columns of f32 from TMEM (this warp's lane quarter): one weight row per lane,
// one batch row per column
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float v[64]) {
    tmem_ld32(taddr, v);
    tmem_ld32(taddr + 32, v + 32);
}

// 32 lanes x 32 columns of 32-bit values into TMEM (this warp's lane quarter), then wait until
// the writes are done
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t r[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// named barrier of the four epilogue warps that also returns the OR of `v` over them
__device__ __forceinline__ bool epi_bar_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.or.pred p, %2, %3, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(kEpiBar), "n"(kEpiWarps * 32)
        : "memory");
    return r != 0;
}

// silu(g) * u of 8 consecutive K (two float4 of gate, two of up) as 4 packed f16 pairs, for
// the swizzled activation image (vec_silu_mul_inplace, crates/engine/src/scratch.rs:181-186)
__device__ __forceinline__ uint4 glu8(float4 g0, float4 g1, float4 u0, float4 u1) {
    const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    const float uv[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
    uint32_t pk[4];
#pragma unroll
    for (int e = 0; e < 4; e++) {
        const float a = __fdividef(gv[2 * e], 1.0f + __expf(-gv[2 * e])) * uv[2 * e];
        const float b = __fdividef(gv[2 * e + 1], 1.0f + __expf(-gv[2 * e + 1])) * uv[2 * e + 1];
        __half2 t = __floats2half2_rn(a, b);
        pk[e] = *reinterpret_cast<uint32_t*>(&t);
    }
    return make_uint4(pk[0], pk[1], pk[2], pk[3]);
}

// the gate and up halves (8 K each) of activation chunk j of batch row n in K tile kt of h2;
// zeros for rows past the batch
struct GluLoad {
    float4 g[2][2], u[2][2];  // two chunks (rows n and n + 16)
};
__device__ __forceinline__ void glu_load(const float* __restrict__ h2, int ld, int batch, int kt, int n, int j,
                                         GluLoad& r) {
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const int nn = n + 16 * i;
        if (nn < batch) {
            const float4* g = reinterpret_cast<const float4*>(h2 + (size_t)nn * ld + (size_t)kt * 128 + 8 * j);
            r.g[i][0] = g[0];
            r.g[i][1] = g[1];
            r.u[i][0] = g[16];  // the matching up rows: 64 floats further
            r.u[i][1] = g[17];
        } else {
            r.g[i][0] = r.g[i][1] = r.u[i][0] = r.u[i][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
}
__device__ __forceinline__ void glu_store(uint8_t* tile, int n, int j, const GluLoad& r) {
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const int nn = n + 16 * i;
        *reinterpret_cast<uint4*>(tile + nn * 128 + ((j ^ (nn & 7)) << 4)) =
            glu8(r.g[i][0], r.g[i][1], r.u[i][0], r.u[i][1]);
    }
}

template <int NB>
__global__ void __launch_bounds__(kUmmaThreads, 1)
    q8_umma_gemm_kernel(const uint8_t* __restrict__ wt, UnitPlan P, const uint8_t* __restrict__ x16,
                        const float* __restrict__ h2, int h2_ld, int batch, unsigned* __restrict__ err, GemmEpi ep) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* w_full = reinterpret_cast<uint64_t*>(smem + UmmaSmem::bar_off());
    uint64_t* w_free = w_full + kWStages;
    uint64_t* op_full = w_free + kWStages;
    uint64_t* op_free = op_full + kOpStages;
    uint64_t* x_full = op_free + kOpStages;
    uint64_t* x_free = x_full + kXSlotsMax;
    uint64_t* acc_full = x_free + kXSlotsMax;
    uint64_t* acc_free = acc_full + 2;
    uint64_t* mma_done = acc_free + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
    __shared__ int s_abort;

    using X = XShape<NB>;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, U = P.units, KT = P.KT;
    const uint32_t WL = ep.wt.wait_ns;  // the limit of every wait below

    if (threadIdx.x == 0) {
        s_abort = 0;
        for (int s = 0; s < kWStages; s++) {
            mbar_init(&w_full[s], 1);
            mbar_init(&w_free[s], kConvWarps * 32);
        }
        for (int s = 0; s < kOpStages; s++) {
            mbar_init(&op_full[s], kConvWarps * 32);
            mbar_init(&op_free[s], 1);
        }
        for (int s = 0; s < X::kSlots; s++) {
            // a copied stage completes on its bytes; a SwiGLU tile on all epilogue threads' stores
            mbar_init(&x_full[s], h2 ? kEpiWarps * 32 : 1);
            mbar_init(&x_free[s], 1);
        }
        for (int j = 0; j < X::kAccBufs; j++) {
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
                bool split;
                unit_range(u, P, mt, k0, len, split);
                const uint8_t* src = wt + ((size_t)mt * KT + k0) * kWStageBytes;  // the unit's blocks are contiguous
                for (int q = 0; q < len; q++, st++) {
                    const int s = st % kWStages;
                    // once the ring is full, pull this CTA's share of the next GEMM's weights
                    // into L2 (this launch is latency-bound, so the extra HBM reads are free)
                    if (st == kWStages) prefetch_share_l2(ep.pf, ep.pf_bytes, blockIdx.x, G);
                    if (st >= kWStages && !mbar_wait(&w_free[s], ((st / kWStages) - 1) & 1, WL)) {
                        atomicOr(err, 1u);
                        s_abort = 1;
                        ok = false;
                        break;
                    }
                    if (st == ep.wt.withhold) continue;  // test hook: this copy is never issued
                    mbar_arrive_expect_tx(&w_full[s], kWStageBytes);
                    bulk_g2s(smem + UmmaSmem::w_off(s), src + (size_t)q * kWStageBytes, kWStageBytes, &w_full[s]);
                }
            }
            if (st <= kWStages) prefetch_share_l2(ep.pf, ep.pf_bytes, blockIdx.x, G);
            for (int j = max(0, st - kWStages); j < st; j++)  // issued copies land before exit
                if (j != ep.wt.withhold && !mbar_wait(&w_full[j % kWStages], (j / kWStages) & 1, WL))
                    atomicOr(err, 2u);
        }
    } else if (warp == kWarpX) {
        // ---------------- activation producer (after the predecessor has completed); with a
        // SwiGLU source the epilogue warps produce the activations instead
        if (lane == 0 && !h2) {
            pdl_wait();
            int g = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < U && ok; u += G) {
                int mt, k0, len;
                bool split;
                unit_range(u, P, mt, k0, len, split);
                for (int q = 0; q < len; q += X::kGroup, g++) {
                    const int s = g % kXStages;
                    if (g >= kXStages && !mbar_wait(&x_free[s], ((g / kXStages) - 1) & 1, WL)) {
                        atomicOr(err, 4u);
                        s_abort = 1;
                        ok = false;
                        break;
                    }
                    const uint32_t bytes = (uint32_t)min(X::kGroup, len - q) * X::kTileBytes;
                    mbar_arrive_expect_tx(&x_full[s], bytes);
                    bulk_g2s(smem + UmmaSmem::x_off(s, X::kGroup, X::kTileBytes),
                             x16 + (size_t)(k0 + q) * X::kTileBytes, bytes, &x_full[s]);
                }
            }
            for (int j = max(0, g - kXStages); j < g; j++)
                if (!mbar_wait(&x_full[j % kXStages], (j / kXStages) & 1, WL)) atomicOr(err, 8u);
        }
    } else if (warp == kWarpMma) {
        // ---------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(kRows, NB);
            const int xg = h2 ? 1 : X::kGroup, xs = h2 ? X::kSlots : kXStages;  // tiles per stage, stages
            int st = 0, sx = 0, xph = 0, j = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < U && ok; u += G, j++) {
                int mt, k0, len;
                bool split;
                unit_range(u, P, mt, k0, len, split);
                if (j >= X::kAccBufs) {
                    if (!mbar_wait(&acc_free[j % X::kAccBufs], ((j / X::kAccBufs) - 1) & 1, WL)) {
                        atomicOr(err, 16u);
                        ok = false;
                        break;
                    }
                    tc_fence_after();  // the epilogue's TMEM loads of this accumulator are done
                }
                const uint32_t d = tmem + kAccCol0 + (uint32_t)((j % X::kAccBufs) * X::kAccCols);
                int ux = 0;  // K tile within the activation stage sx
                for (int q = 0; q < len; q++, st++) {
                    const int so = st % kOpStages;
                    if (!mbar_wait(&op_full[so], (st / kOpStages) & 1, WL) ||
                        (ux == 0 && !mbar_wait(&x_full[sx], xph, WL))) {
                        atomicOr(err, 32u);
                        ok = false;
                        break;
                    }
                    tc_fence_after();  // the converters' TMEM stores of this stage are complete
                    // one descriptor per stage: a K16 step advances its start address by 32 bytes,
                    // i.e. 2 in the descriptor's 16-byte units
                    const uint64_t xd =
                        umma_desc_sw128(smem_u32(smem + UmmaSmem::x_off(sx, xg, X::kTileBytes) + ux * X::kTileBytes));
                    const uint32_t a0 = tmem + kOpCol0 + (uint32_t)(so * kStageTiles * 32);
                    const uint32_t acc0 = q > 0 ? 1u : 0u;
#pragma unroll
                    for (int k = 0; k < kTileK / 16; k++)
#pragma unroll
                        for (int t = 0; t < kStageTiles; t++)
                            umma_ts_f16(d + t * NB, a0 + t * 32 + k * 8, xd + (uint64_t)(2 * k), idesc,
                                        k > 0 ? 1u : acc0);
                    if (++ux == xg || q == len - 1) {
                        umma_commit(&x_free[sx]);
                        ux = 0;
                        if (++sx == xs) {
                            sx = 0;
                            xph ^= 1;
                        }
                    }
                    umma_commit(&op_free[so]);
                }
                umma_commit(&acc_full[j % X::kAccBufs]);
            }
            if (!ok) s_abort = 1;
            umma_commit(mma_done);  // every MMA issued above has completed before TMEM is freed
            if (!mbar_wait(mma_done, 0, WL)) atomicOr(err, 64u);
        }
    } else if (warp < kConvWarps) {
        // ---------------- converters: weight row r of tile t -> 32 TMEM columns of f16 pairs
        const int t = warp >> 2, quarter = warp & 3;
        const int r = quarter * 32 + lane;
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        int st = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < U && ok; u += G) {
          int mt, k0, len;
          bool split;
          unit_range(u, P, mt, k0, len, split);
          for (int q = 0; q < len; q++, st++) {
            const int sw = st % kWStages, so = st % kOpStages;
            // warp-uniform outcome: tcgen05.st below is a whole-warp instruction
            if (!__all_sync(0xffffffffu, mbar_wait(&w_full[sw], (st / kWStages) & 1, WL))) {
                if (lane == 0) atomicOr(err, 128u);
                s_abort = 1;
                ok = false;
                break;
            }
            const uint8_t* wb = smem + UmmaSmem::w_off(sw) + t * kUTileBytes;
            uint4 qv[4];
#pragma unroll
            for (int c = 0; c < 4; c++) qv[c] = *reinterpret_cast<const uint4*>(wb + ((size_t)c * kRows + r) * 16);
            const uint32_t dd = *reinterpret_cast<const uint32_t*>(wb + 4 * kRows * 16 + r * 4);
            uint32_t hv[32];  // k pairs (2j, 2j+1), j = 0..31, in K order
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const unsigned short dbits = (unsigned short)(c >= 2 ? (dd >> 16) : (dd & 0xffffu));
                const __half2 dh = __halves2half2(__ushort_as_half(dbits), __ushort_as_half(dbits));
                q8_unpack(qv[c], hv + 8 * c);
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    __half2 x = *reinterpret_cast<__half2*>(&hv[8 * c + e]);
                    x = __hmul2(x, dh);
                    hv[8 * c + e] = *reinterpret_cast<uint32_t*>(&x);
                }
            }
            if (st >= kOpStages &&
                !__all_sync(0xffffffffu, mbar_wait(&op_free[so], ((st / kOpStages) - 1) & 1, WL))) {
                if (lane == 0) atomicOr(err, 256u);
                s_abort = 1;
                ok = false;
                break;
            }
            tc_fence_after();  // the MMAs that read this operand slot have completed
            tmem_st32(tmem + lane_base + kOpCol0 + (uint32_t)(so * kStageTiles * 32 + t * 32), hv);
            tc_fence_before();
            // The raw stage is released only after the converted values are stored: the stores
            // consume the registers loaded from it, so those loads have completed. Every thread
            // arrives after its own stores, so the MMA issued after the phase completes reads
            // what each of them wrote.
            mbar_arrive(&w_free[sw]);
            mbar_arrive(&op_full[so]);
          }
        }
    } else if (warp >= kWarpEpi0 && warp < kWarpEpi0 + kEpiWarps) {
        // ---------------- epilogue warps: TMEM lanes 32q .. 32q+31 = weight rows of each tile
        const int q = warp & 3;
        const int et = threadIdx.x - kWarpEpi0 * 32;  // 0..127
        pdl_wait();  // outputs may be read or written by earlier kernels of the stream
        int gx = 0;  // SwiGLU source: activation tiles produced so far
        for (int j = 0, u = blockIdx.x; u < U; j++, u += G) {
            bool fail = false;
            int mt, k0, len;
            bool split;
            unit_range(u, P, mt, k0, len, split);
            // 2: add into y (split units, EPI_ADD), 1: y += Wx (RESID), 0: y = Wx
            const int how = (split || ep.mode == EPI_ADD) ? 2 : (ep.mode == EPI_RESID ? 1 : 0);
            if (h2) {
                // this unit's activation tiles from the gate/up sums: thread et takes the
                // 16-byte chunk jn = et % 8 (8 K) of rows et / 8 + 16 i, i = 0 .. NB / 16 - 1,
                // as loads of two rows (64 rows per pass), each issued half a pass ahead of its use
                const int jn = et & 7, n0 = et >> 3;
                GluLoad ra, rb;
                glu_load(h2, h2_ld, batch, k0, n0, jn, ra);
                for (int kq = 0; kq < len && !fail; kq++, gx++) {
                    const int s = gx % X::kSlots;
                    uint8_t* tile = smem + UmmaSmem::x_off(s, 1, X::kTileBytes);
#pragma unroll
                    for (int ps = 0; ps < NB / 64; ps++) {
                        const int nb = n0 + 64 * ps;
                        glu_load(h2, h2_ld, batch, k0 + kq, nb + 32, jn, rb);
                        if (ps == 0 && gx >= X::kSlots && !mbar_wait(&x_free[s], ((gx / X::kSlots) - 1) & 1, WL)) {
                            atomicOr(err, 2048u);
                            s_abort = 1;
                            fail = true;
                            break;
                        }
                        glu_store(tile, nb, jn, ra);
                        if (ps + 1 < NB / 64)
                            glu_load(h2, h2_ld, batch, k0 + kq, nb + 64, jn, ra);
                        else if (kq + 1 < len)
                            glu_load(h2, h2_ld, batch, k0 + kq + 1, n0, jn, ra);
                        glu_store(tile, nb + 32, jn, rb);
                    }
                    if (fail) break;
                    fence_proxy_async_smem();  // the MMAs read the tile through the async proxy
                    mbar_arrive(&x_full[s]);
                }
            }
            if (!fail && !mbar_wait(&acc_full[j % X::kAccBufs], (j / X::kAccBufs) & 1, WL)) {
                fail = true;
                atomicOr(err, 512u);
                s_abort = 1;
            }
            // one outcome for all epilogue threads, which meet at a named barrier below
            if (epi_bar_or(fail || *(volatile int*)&s_abort)) break;
            tc_fence_after();
            const uint32_t dq =
                tmem + ((uint32_t)(q * 32) << 16) + kAccCol0 + (uint32_t)((j % X::kAccBufs) * X::kAccCols);
            const int pr = mt;  // row-tile pair: rows pr*256 .. pr*256+255
            if (u + G < U) {
                // more units follow: write straight from TMEM, lanes on consecutive rows m
#pragma unroll 1
                for (int tb = 0; tb < kStageTiles * NB / 64; tb++) {
                    // 64 batch rows b0 .. b0 + 63 of weight tile t
                    const int t = tb / (NB / 64), b0 = (tb % (NB / 64)) * 64;
                    float v[64];
                    tmem_ld64(dq + t * NB + b0, v);
                    const int m = pr * kPairRows + t * kRows + q * 32 + lane;
                    if (m < ep.m_out) {
#pragma unroll
                        for (int b = 0; b < 64; b++) {
                            if (b0 + b >= batch) break;
                            float* yp = ep.y + (size_t)(b0 + b) * ep.ldy + m;
                            if (how == 2)
                                atomicAdd(yp, v[b]);  // result unused: compiles to a reduction
                            else
                                *yp = how == 1 ? *yp + v[b] : v[b];
                        }
                    }
                }
                tc_fence_before();
                mbar_arrive(&acc_free[j % X::kAccBufs]);  // this thread's TMEM loads are done
                continue;
            }
            // The last unit: the raw weight ring is idle (every stage was converted before the
            // last MMA), so the accumulator is staged over it as [NB batch rows][kStageLd
            // floats], each lane writing its weight row's column of it (consecutive lanes,
            // consecutive words). Each batch row's outputs then leave in one bulk operation: a
            // bulk store, or a bulk f32 add at L2 when the output accumulates (K splits,
            // residual). Per-thread reductions of the same data were bound by the L2's atomic
            // rate when all CTAs reached their epilogue together.
            float* stage = reinterpret_cast<float*>(smem);
#pragma unroll 1
            for (int tb = 0; tb < kStageTiles * NB / 64; tb++) {
                const int t = tb / (NB / 64), b0 = (tb % (NB / 64)) * 64;
                float v[64];
                tmem_ld64(dq + t * NB + b0, v);
                const int ml = t * kRows + q * 32 + lane;
#pragma unroll
                for (int b = 0; b < 64; b++) stage[(b0 + b) * kStageLd + ml] = v[b];
            }
            fence_proxy_async_smem();  // the bulk operations read the staged rows through the async proxy
            tc_fence_before();
            asm volatile("bar.sync %0, %1;" ::"n"(kEpiBar), "n"(kEpiWarps * 32) : "memory");
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
                    // the CTA may leave once the staged rows have been read out; the writes
                    // themselves complete with the grid, before any dependent grid reads them
                    bulk_wait_read();
                }
                continue;
            }
            for (int rr = et >> 6; rr < batch; rr += 2) {  // two rows per pass, 64 groups of 4 each
                const int c4 = et & 63;
                const int m = m0 + c4 * 4;
                const float4 v = *reinterpret_cast<const float4*>(stage + rr * kStageLd + c4 * 4);
                float* yp = ep.y + (size_t)rr * ep.ldy + m;
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

// The unit plan of a weight with MT row tiles and KT K tiles on num_sms SMs. Layer weights
// (fewer pairs than SMs) are K-split so the units cover the SMs about once. A weight with more
// pairs than SMs runs whole pairs, several rounds per CTA; when the last round would hold only
// a few pairs (at most a quarter of the SMs), those pairs are cut into K pieces of at least
// two tiles spread over as many CTAs, so no CTA runs a whole extra pair at the end.
UmmaPlan umma_plan(int MT, int KT, int64_t M, int num_sms) {
    UmmaPlan p;
    p.pairs = (MT + 1) / 2;
    p.ks = umma_nsplit(MT, KT, EPI_STORE, num_sms);
    p.kper = (KT + p.ks - 1) / p.ks;
    const int rem = p.ks == 1 && p.pairs > num_sms ? p.pairs % num_sms : 0;
    if (rem > 0 && rem * 4 <= num_sms && KT >= 4) {
        p.tail_pairs = rem;
        const int want = std::min(num_sms / rem, KT / 2);
        p.kper_tail = (KT + want - 1) / want;
        p.ks_tail = (KT + p.kper_tail - 1) / p.kper_tail;
    }
    p.main_units = (p.pairs - p.tail_pairs) * p.ks;
    p.units = p.main_units + p.tail_pairs * p.ks_tail;
    p.zero_row0 = p.ks > 1 ? 0 : (p.tail_pairs ? (int64_t)(p.pairs - p.tail_pairs) * kPairRows : M);
    if (p.zero_row0 > M) p.zero_row0 = M;
    return p;
}

template <int NB>
static int launch_umma_t(const Q8Weight& w, const uint8_t* x16, int batch, unsigned* err, const GemmEpi& ep,
                         int num_sms, cudaStream_t st, const float* h2, int h2_ld) {
    const int smem = UmmaSmem::bytes() + 1024;
    static bool attr_set[64] = {};  // per device, before the first launch
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev & 63]) {
        if (cudaFuncSetAttribute(q8_umma_gemm_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess)
            return -1;
        attr_set[dev & 63] = true;
    }
    const UmmaPlan pl = umma_plan(w.MT, w.KT, w.M, num_sms);
    UnitPlan P;
    P.KT = w.KT;
    P.ks = pl.ks;
    P.kper = pl.kper;
    P.main_units = pl.main_units;
    P.first_tail = pl.pairs - pl.tail_pairs;
    P.ks_tail = pl.ks_tail;
    P.kper_tail = pl.kper_tail;
    P.units = pl.units;
    const int G = std::min(pl.units, num_sms);
    GemmEpi e = ep;
    e.wt = take_wait_test(kWaitTestGemm, st);
    if (launch_pdl(q8_umma_gemm_kernel<NB>, dim3(G), dim3(kUmmaThreads), smem, st, w.qt, P, x16, h2, h2_ld, batch,
                   err, e) != cudaSuccess)
        return -2;
    return 0;
}

// batch <= 64 runs the N = 64 form (the activation image x16 holds 64 rows), 65..128 the
// N = 128 form (128 rows: a prefill step)
int launch_q8_umma(const Q8Weight& w, const uint8_t* x16, int batch, unsigned* err, const GemmEpi& ep, int num_sms,
                   cudaStream_t st, const float* h2, int h2_ld) {
    if (batch < 1 || batch > kMaxBatchRows) return -1;
    if (ep.mode == EPI_SWIGLU) return -3;  // SwiGLU: EPI_ADD into h2, then a launch with the h2 source
    // the SwiGLU source reads whole 64-column gate/up groups of h2 (K = ffn a multiple of 64)
    if (h2 && (w.KB % 2 != 0 || h2_ld < 2 * 32 * w.KB || (h2_ld & 3) != 0)) return -1;
    return batch > 64 ? launch_umma_t<128>(w, x16, batch, err, ep, num_sms, st, h2, h2_ld)
                      : launch_umma_t<64>(w, x16, batch, err, ep, num_sms, st, h2, h2_ld);
}

}  // namespace ab2
