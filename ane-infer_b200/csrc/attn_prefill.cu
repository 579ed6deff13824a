// attn_prefill.cu -- causal GQA attention of a prefill step on the tensor cores, bf16 KV cache.
//
// The rows of a prefill step are consecutive prompt tokens of one sequence (positions
// p0 .. p0 + rows - 1) that all read one cache slot, after attn_prep_kernel appended their
// keys and values. Row b attends over cache positions 0 .. pos[b] (full_attn_decode_step per
// token, crates/engine/src/deltanet.rs:565-669, as the reference's prompt loop runs it,
// crates/cli/src/main.rs:358-362). The decode kernel would stream the prefix once per row;
// here a CTA takes a query block of 8 tokens x the 4 query heads of one kv head (32 query
// rows) and one split of the prefix, and streams each 64-token K/V tile once for the block:
//   * a producer warp copies the tiles with TMA (the decode kernel's boxes of 64 tokens x 64
//     dims, 128-byte swizzle) into a 2-stage mbarrier ring;
//   * eight compute warps form S = Q K^T (warp w: query rows 16 (w % 2) .. + 15, keys
//     16 (w / 2) .. + 15 of the tile) and O += P V (warp w: all 32 rows, dims w HD/8 .. + HD/8)
//     with mma.m16n8k16, the queries and the probabilities as bf16 hi/lo pairs against exact
//     bf16 K and V (two products each), so scores and outputs keep about f32 accuracy;
//   * the online softmax runs per tile, 8 threads per row, through shared memory;
//   * a row whose prefix lies in one split writes its gated output; otherwise each split
//     writes the row's partial (m, l, unnormalised O) in the decode kernel's layout, and
//     attn_merge_kernel merges them in split order.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>

#include "attn_tiles.cuh"
#include "common.cuh"
#include "kernels.h"
#include "umma.cuh"

namespace ab2 {
namespace {

constexpr int kQTok = 8;                 // prompt tokens per query block
constexpr int kQRows = kGQ * kQTok;      // query rows: row r = head r / kQTok, token r % kQTok
constexpr int kPfWarps = 8;              // compute warps
constexpr int kPfCT = kPfWarps * 32;
constexpr int kPfThreads = kPfCT + 32;   // + one TMA producer warp
constexpr int kPfStages = 2;
constexpr int kPfPStride = kT + 8;       // bf16 per P row (padding against ldmatrix bank conflicts)
static_assert(kQRows == 32 && kPfCT == kQRows * 8, "eight softmax threads per query row");

template <int HD>
struct PfAttnSmem {
    static constexpr int kTileBytes = kT * HD * 2;  // one K (or V) tile
    static constexpr int kQStride = HD + 8;         // bf16 per query row
    static constexpr int k_off(int s) { return s * kTileBytes; }
    static constexpr int v_off(int s) { return (kPfStages + s) * kTileBytes; }
    static constexpr int qh_off() { return 2 * kPfStages * kTileBytes; }          // q hi [32][kQStride] bf16
    static constexpr int ql_off() { return qh_off() + kQRows * kQStride * 2; }    // q lo
    static constexpr int s_off() { return ql_off() + kQRows * kQStride * 2; }     // scores [32][kT] f32
    static constexpr int ph_off() { return s_off() + kQRows * kT * 4; }           // p hi [32][kPfPStride] bf16
    static constexpr int pl_off() { return ph_off() + kQRows * kPfPStride * 2; }  // p lo
    static constexpr int misc_off() { return pl_off() + kQRows * kPfPStride * 2; }  // corr, m, l [32] each
    static constexpr int bar_off() { return misc_off() + 3 * kQRows * 4; }          // full[S], empty[S]
    static constexpr int bytes() { return bar_off() + 2 * kPfStages * 8; }
};

__device__ __forceinline__ void pf_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kPfCT) : "memory"); }
// pf_bar that also returns the OR of `v` over the compute threads
__device__ __forceinline__ bool pf_bar_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.or.pred p, 1, %2, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(kPfCT)
        : "memory");
    return r != 0;
}

// CTA (blockIdx.x = query block * Hkv + kv head, blockIdx.y = split of the prefix)
template <int HD>
__global__ void __launch_bounds__(kPfThreads, 1)
    attn_prefill_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv, AttnParams p,
                        int64_t row_base, int rows) {
    using L = PfAttnSmem<HD>;
    constexpr int NDB = HD / 64;
    constexpr int QS = L::kQStride;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    __nv_bfloat16* Qh = reinterpret_cast<__nv_bfloat16*>(smem + L::qh_off());
    __nv_bfloat16* Ql = reinterpret_cast<__nv_bfloat16*>(smem + L::ql_off());
    float* S_s = reinterpret_cast<float*>(smem + L::s_off());
    float* corr_s = reinterpret_cast<float*>(smem + L::misc_off());
    float* m_s = corr_s + kQRows;
    float* l_s = corr_s + 2 * kQRows;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::bar_off());
    uint64_t* empty = full + kPfStages;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int blk = blockIdx.x / p.Hkv, kvh = blockIdx.x % p.Hkv, split = blockIdx.y;
    const int b0 = blk * kQTok, nrow = min(kQTok, rows - b0);
    const uint32_t WL = p.wt.wait_ns;  // the limit of every wait below

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPfStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kPfCT);
        }
        mbar_fence_init();
    }
    __syncthreads();
    asm volatile("griddepcontrol.wait;" ::: "memory");  // prepared queries and appended K/V

    // the block's keys: positions below the largest valid position + 1 of its rows; this
    // split covers [t0, t1) of them (a CTA whose split starts past them has nothing to do)
    int Lb = 0;
    for (int j = 0; j < nrow; j++) {
        const int ps = p.pos[b0 + j];
        if (attn_pos_ok(p, ps)) Lb = max(Lb, ps + 1);
    }
    const int t0 = split * p.chunk;
    if (t0 >= Lb) return;
    const int t1 = min(Lb, t0 + p.chunk);
    const int ntiles = (t1 - t0 + kT - 1) / kT;

    if (warp == kPfWarps) {
        // ---------------- producer: the K and V tiles of [t0, t1) of this kv head
        if (lane == 0) {
            // every row of the block reads the one slot at row_base (seq_rows 0)
            const int rows0 = (int)(row_base + (int64_t)kvh * p.cap + t0);
            bool ok = true;
            int i = 0;
            for (; i < ntiles; i++) {
                const int s = i % kPfStages;
                if (i >= kPfStages && !mbar_wait(&empty[s], ((i / kPfStages) - 1) & 1, WL)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&full[s], 2u * L::kTileBytes);
#pragma unroll
                for (int d = 0; d < NDB; d++) {
                    tma_load_2d(smem + L::k_off(s) + d * 8192, &tmk, d * 64, rows0 + i * kT, &full[s]);
                    tma_load_2d(smem + L::v_off(s) + d * 8192, &tmv, d * 64, rows0 + i * kT, &full[s]);
                }
            }
            if (!ok && p.err) atomicOr(p.err, 4096u);
            // every issued copy lands before the CTA can exit
            for (int j = max(0, i - kPfStages); j < i; j++) mbar_wait(&full[j % kPfStages], (j / kPfStages) & 1, WL);
        }
        __syncwarp();
        return;
    }

    // ---------------- compute warps
    const int ct = threadIdx.x;
    const int g = lane >> 2, t = lane & 3;
    // the token of every row this thread touches in the products is token g of the block
    // (rows 16 m + g and 16 m + g + 8 are heads 2m and 2m + 1 of it); -1 when absent
    int pos_g = -1;
    if (g < nrow) {
        const int ps = p.pos[b0 + g];
        if (attn_pos_ok(p, ps)) pos_g = ps;
    }
    // queries as bf16 hi/lo pairs: row r = (head hh, token j), zero for absent tokens
    for (int e4 = ct; e4 < kQRows * HD / 4; e4 += kPfCT) {
        const int r = e4 / (HD / 4), d = (e4 % (HD / 4)) * 4, hh = r / kQTok, j = r % kQTok;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j < nrow) v = *reinterpret_cast<const float4*>(p.qprep + (((size_t)(b0 + j) * p.Hkv + kvh) * kGQ + hh) * HD + d);
        const float vv[4] = {v.x, v.y, v.z, v.w};
        float hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; e++) split_bf16(vv[e], hi[e], lo[e]);
        *reinterpret_cast<uint2*>(Qh + r * QS + d) = make_uint2(pack_bf16(hi[0], hi[1]), pack_bf16(hi[2], hi[3]));
        *reinterpret_cast<uint2*>(Ql + r * QS + d) = make_uint2(pack_bf16(lo[0], lo[1]), pack_bf16(lo[2], lo[3]));
    }
    pf_bar();

    const uint32_t qh_b = smem_u32(Qh), ql_b = smem_u32(Ql);
    const uint32_t ph_b = smem_u32(smem + L::ph_off()), pl_b = smem_u32(smem + L::pl_off());
    const int mq = warp & 1, nq = warp >> 1;  // S: rows 16 mq .. + 15, tile keys 16 nq .. + 15
    const float sq = sqrtf((float)HD);
    constexpr int DW = HD / kPfWarps;  // output dims of this warp
    constexpr int NPV = DW / 8;        // their 8-dim n-tiles
    float o[2][NPV][4];
#pragma unroll
    for (int mt = 0; mt < 2; mt++)
#pragma unroll
        for (int n = 0; n < NPV; n++) o[mt][n][0] = o[mt][n][1] = o[mt][n][2] = o[mt][n][3] = 0.0f;
    const int sr = ct >> 3, sc8 = (ct & 7) * 8;  // softmax: row sr, tile columns sc8 .. + 7
    float m_run = -INFINITY, l_run = 0.0f;       // of row sr (the same in its 8 threads)
    bool ok = true;
    for (int i = 0; i < ntiles; i++) {
        const int s = i % kPfStages;
        const bool w_ok = mbar_wait(&full[s], (i / kPfStages) & 1, WL);
        const uint32_t kb = smem_u32(smem + L::k_off(s)), vb = smem_u32(smem + L::v_off(s));
        const int tbase = t0 + i * kT;
        // S = Q K^T: k-steps 2 kk and 2 kk + 1 per round; A (queries) hi and lo, B (keys) exact
        float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll 4
        for (int kk = 0; kk < HD / 32; kk++) {
            uint32_t ah[2][4], al[2][4];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int m = lane >> 3;
                const int row = 16 * mq + (m & 1) * 8 + (lane & 7), col = (2 * kk + h) * 16 + (m >> 1) * 8;
                ldsm_x4(qh_b + (row * QS + col) * 2, ah[h][0], ah[h][1], ah[h][2], ah[h][3]);
                ldsm_x4(ql_b + (row * QS + col) * 2, al[h][0], al[h][1], al[h][2], al[h][3]);
            }
#pragma unroll
            for (int jn = 0; jn < 2; jn++) {
                const int row = 16 * nq + 8 * jn + (lane & 7), chunk = kk * 4 + (lane >> 3);
                uint32_t r0, r1, r2, r3;
                ldsm_x4(kv_tile_addr(kb, row, chunk), r0, r1, r2, r3);
                mma_bf16(acc[jn], ah[0][0], ah[0][1], ah[0][2], ah[0][3], r0, r1);
                mma_bf16(acc[jn], al[0][0], al[0][1], al[0][2], al[0][3], r0, r1);
                mma_bf16(acc[jn], ah[1][0], ah[1][1], ah[1][2], ah[1][3], r2, r3);
                mma_bf16(acc[jn], al[1][0], al[1][1], al[1][2], al[1][3], r2, r3);
            }
        }
        // causal mask: key position kidx is visible to token g when kidx <= pos[g] (and < t1)
#pragma unroll
        for (int jn = 0; jn < 2; jn++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int col = 16 * nq + 8 * jn + 2 * t + (e & 1), r = 16 * mq + g + (e >> 1) * 8;
                const int kidx = tbase + col;
                S_s[r * kT + col] = (kidx <= pos_g && kidx < t1) ? acc[jn][e] / sq : -INFINITY;
            }
        if (pf_bar_or(!w_ok)) {
            ok = false;
            break;
        }
        // online softmax of row sr over the tile: 8 threads, 8 columns each
        {
            float v[8];
            float mx = -INFINITY;
#pragma unroll
            for (int e = 0; e < 8; e++) {
                v[e] = S_s[sr * kT + sc8 + e];
                mx = fmaxf(mx, v[e]);
            }
            mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 2));
            mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 4));
            const float m_new = fmaxf(m_run, mx);
            float pv[8], sum = 0.0f, corr = 1.0f;
#pragma unroll
            for (int e = 0; e < 8; e++) pv[e] = 0.0f;
            if (m_new != -INFINITY) {
#pragma unroll
                for (int e = 0; e < 8; e++) pv[e] = v[e] == -INFINITY ? 0.0f : expf(v[e] - m_new);
                corr = m_run == -INFINITY ? 0.0f : expf(m_run - m_new);
            }
#pragma unroll
            for (int e = 0; e < 8; e++) sum += pv[e];
            sum += __shfl_xor_sync(kFull, sum, 1);
            sum += __shfl_xor_sync(kFull, sum, 2);
            sum += __shfl_xor_sync(kFull, sum, 4);
            l_run = l_run * corr + sum;
            m_run = m_new;
            uint32_t ph[4], pl[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                float h0, l0, h1, l1;
                split_bf16(pv[2 * e], h0, l0);
                split_bf16(pv[2 * e + 1], h1, l1);
                ph[e] = pack_bf16(h0, h1);
                pl[e] = pack_bf16(l0, l1);
            }
            const int po = (sr * kPfPStride + sc8) * 2;
            *reinterpret_cast<uint4*>(smem + L::ph_off() + po) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
            *reinterpret_cast<uint4*>(smem + L::pl_off() + po) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
            if ((ct & 7) == 0) corr_s[sr] = corr;
        }
        pf_bar();
        // O = O * corr + P V: rows 0..31 (two m-tiles), dims warp * DW .. + DW
#pragma unroll
        for (int mt = 0; mt < 2; mt++) {
            const float c0 = corr_s[16 * mt + g], c1 = corr_s[16 * mt + g + 8];
#pragma unroll
            for (int n = 0; n < NPV; n++) {
                o[mt][n][0] *= c0;
                o[mt][n][1] *= c0;
                o[mt][n][2] *= c1;
                o[mt][n][3] *= c1;
            }
        }
#pragma unroll
        for (int kk = 0; kk < kT / 16; kk++) {
            uint32_t ah[2][4], al[2][4];
            const int m = lane >> 3;
#pragma unroll
            for (int mt = 0; mt < 2; mt++) {
                const int prow = 16 * mt + (m & 1) * 8 + (lane & 7), pcol = kk * 16 + (m >> 1) * 8;
                ldsm_x4(ph_b + (prow * kPfPStride + pcol) * 2, ah[mt][0], ah[mt][1], ah[mt][2], ah[mt][3]);
                ldsm_x4(pl_b + (prow * kPfPStride + pcol) * 2, al[mt][0], al[mt][1], al[mt][2], al[mt][3]);
            }
#pragma unroll
            for (int np = 0; np < NPV / 2; np++) {
                const int d0 = warp * DW + np * 16;
                const int tok = kk * 16 + (lane & 7) + (m & 1) * 8, chunk = (d0 >> 3) + (m >> 1);
                uint32_t r0, r1, r2, r3;
                ldsm_x4_t(kv_tile_addr(vb, tok, chunk), r0, r1, r2, r3);
#pragma unroll
                for (int mt = 0; mt < 2; mt++) {
                    mma_bf16(o[mt][2 * np], ah[mt][0], ah[mt][1], ah[mt][2], ah[mt][3], r0, r1);
                    mma_bf16(o[mt][2 * np], al[mt][0], al[mt][1], al[mt][2], al[mt][3], r0, r1);
                    mma_bf16(o[mt][2 * np + 1], ah[mt][0], ah[mt][1], ah[mt][2], ah[mt][3], r2, r3);
                    mma_bf16(o[mt][2 * np + 1], al[mt][0], al[mt][1], al[mt][2], al[mt][3], r2, r3);
                }
            }
        }
        mbar_arrive(&empty[s]);
    }
    if (!ok) {
        // a timed-out wait: report it and stop; the results of this launch are invalid
        if (ct == 0 && p.err) atomicOr(p.err, 4096u);
        return;
    }
    if ((ct & 7) == 0) {
        m_s[sr] = m_run;
        l_s[sr] = l_run;
    }
    pf_bar();
    // token g's rows of this thread: a prefix in one split gives the gated output, else this
    // split's partial for attn_merge_kernel (only splits that hold some of the token's keys)
    if (pos_g < 0) return;
    const int b = b0 + g, nsplit = (pos_g + 1 + p.chunk - 1) / p.chunk;
    if (split >= nsplit) return;
    const float* proj = p.proj + (size_t)b * p.ldp;
    const size_t part_floats = attn_part_floats(HD);
    float* part = p.ws + (((size_t)b * p.Hkv + kvh) * kMaxSplits + split) * part_floats;
#pragma unroll
    for (int mt = 0; mt < 2; mt++)
#pragma unroll
        for (int e2 = 0; e2 < 2; e2++) {
            const int r = 16 * mt + g + 8 * e2, hh = r / kQTok, h = (p.kvh0 + kvh) * kGQ + hh;
#pragma unroll
            for (int n = 0; n < NPV; n++)
#pragma unroll
                for (int e1 = 0; e1 < 2; e1++) {
                    const int d = warp * DW + 8 * n + 2 * t + e1;
                    const float ov = o[mt][n][2 * e2 + e1];
                    if (nsplit == 1) {
                        float y = ov / l_s[r];
                        y *= ref_sigmoid(proj[(size_t)h * 2 * HD + HD + d]);
                        act_store(p.out, b, h * HD + d, y);
                        if (p.o_out) p.o_out[(size_t)b * p.Hq * HD + h * HD + d] = y;
                    } else {
                        __stcg(part + 2 * kGQ + hh * HD + d, ov);
                    }
                }
            if (nsplit > 1 && warp == 0 && t == 0) {
                __stcg(part + hh, m_s[r]);
                __stcg(part + kGQ + hh, l_s[r]);
            }
        }
}

}  // namespace

// Tokens per split: the decode kernel's cost model over (query block, kv head) pairs instead
// of (sequence, kv head) pairs, since a block streams the prefix once for its 8 tokens.
int attn_prefill_chunk(int rows, int hkv, int max_len, int num_sms) {
    return attn_mma_chunk((rows + kQTok - 1) / kQTok, hkv, max_len, num_sms);
}

template <int HD>
static int launch_prefill_t(const void* tmk, const void* tmv, const AttnParams& p, int64_t row_base, int rows,
                            int max_len, cudaStream_t st, cudaEvent_t core_begin, cudaEvent_t core_end) {
    const int smem = PfAttnSmem<HD>::bytes() + 1024;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev & 63]) {
        if (cudaFuncSetAttribute(attn_prefill_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess)
            return -1;
        attr_set[dev & 63] = true;
    }
    const int splits = attn_nsplit(max_len, p.chunk);
    const int nblk = (rows + kQTok - 1) / kQTok;
    if (launch_attn_prep(p, rows, HD, st)) return -2;
    if (core_begin) cudaEventRecord(core_begin, st);
    AttnParams pm = p;
    pm.wt = WaitTest{};  // the production wait limit (the test hook arms the decode kernel)
    if (launch_pdl(attn_prefill_kernel<HD>, dim3(nblk * p.Hkv, splits), dim3(kPfThreads), smem, st,
                   *reinterpret_cast<const CUtensorMap*>(tmk), *reinterpret_cast<const CUtensorMap*>(tmv), pm,
                   row_base, rows) != cudaSuccess)
        return -2;
    if (core_end) cudaEventRecord(core_end, st);
    if (splits > 1 && launch_attn_merge(p, rows, HD, st)) return -2;
    return 0;
}

int launch_attention_prefill(const void* tmk, const void* tmv, const AttnParams& p, int64_t row_base, int rows,
                             int hd, int max_len, int num_sms, cudaStream_t st, cudaEvent_t core_begin,
                             cudaEvent_t core_end) {
    (void)num_sms;
    if (p.Hq != kGQ * (p.Hkv_all ? p.Hkv_all : p.Hkv) || p.seq_rows != 0 || !p.qprep) return -1;
    if (attn_nsplit(max_len, p.chunk) > kMaxSplits) return -1;
    if (hd == 256) return launch_prefill_t<256>(tmk, tmv, p, row_base, rows, max_len, st, core_begin, core_end);
    if (hd == 128) return launch_prefill_t<128>(tmk, tmv, p, row_base, rows, max_len, st, core_begin, core_end);
    return -1;
}

}  // namespace ab2
