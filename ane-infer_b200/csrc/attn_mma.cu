// attn_mma.cu -- GQA split-KV flash-decode on the tensor cores, bf16 KV cache.
//
// Same contract as attn_decode_kernel (attention.cu: full_attn_decode_step without its
// projections, crates/engine/src/deltanet.rs:565-669), restructured for B200:
//   * a producer warp streams 64-token K and V tiles with TMA (cp.async.bulk.tensor, boxes of
//     64 tokens x 64 dims, 128-byte swizzle) into a 3-stage mbarrier ring, so the HBM stream
//     never waits on the math;
//   * four compute warps form S = Q K^T and O += P V with mma.m16n8k16 (bf16 inputs, f32
//     accumulate). The query and the probabilities enter as bf16 hi/lo pairs (rows 0-3 hi,
//     4-7 lo of the M=16 operand), K and V are exact bf16, so scores and outputs keep ~f32
//     accuracy;
//   * the online softmax runs per 64-token tile across the warps through shared memory;
//   * the CTA holding the new position first writes the new (normed, rotated) key and value
//     into the cache and fences them to the async proxy before TMA reads that tile;
//   * split partials are merged by the last CTA of a (sequence, kv head) in split order.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"
#include "umma.cuh"

namespace ab2 {

constexpr int kT = 64;  // tokens per tile
constexpr int kAttnStages = 3;
constexpr int kCompWarps = 4;
constexpr int kAttnMmaThreads = (kCompWarps + 1) * 32;  // + one TMA producer warp
constexpr int kGQ = 4;
constexpr int kPStride = kT + 8;  // bf16 elements per P row (padding avoids ldmatrix bank conflicts)

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

template <int HD>
struct AttnSmem {
    static constexpr int kNDB = HD / 64;                   // 64-dim TMA boxes per row
    static constexpr int kTileBytes = kT * HD * 2;         // one K (or V) tile
    static constexpr int k_off(int s) { return s * kTileBytes; }
    static constexpr int v_off(int s) { return (kAttnStages + s) * kTileBytes; }
    static constexpr int s_off() { return 2 * kAttnStages * kTileBytes; }     // scores [4][kT] f32
    static constexpr int p_off() { return s_off() + kGQ * kT * 4; }           // P [16][kPStride] bf16
    static constexpr int q_off() { return p_off() + 16 * kPStride * 2; }      // q [4][HD] f32
    static constexpr int kn_off() { return q_off() + kGQ * HD * 4; }          // new k [HD], new v [HD]
    static constexpr int misc_off() { return kn_off() + 2 * HD * 4; }         // corr[4], m[4], l[4], sc[8]
    static constexpr int bar_off() { return misc_off() + 32 * 4; }            // full[S], empty[S]
    static constexpr int bytes() { return bar_off() + 2 * kAttnStages * 8; }
};

template <int HD>
__global__ void __launch_bounds__(kAttnMmaThreads, 1)
    attn_mma_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv, AttnParams p,
                    int64_t row_base) {
    using L = AttnSmem<HD>;
    constexpr int NDB = L::kNDB;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    float* S_s = reinterpret_cast<float*>(smem + L::s_off());
    __nv_bfloat16* P_s = reinterpret_cast<__nv_bfloat16*>(smem + L::p_off());
    float* q_s = reinterpret_cast<float*>(smem + L::q_off());
    float* kn_s = reinterpret_cast<float*>(smem + L::kn_off());
    float* vn_s = kn_s + HD;
    float* corr_s = reinterpret_cast<float*>(smem + L::misc_off());
    float* m_s = corr_s + 4;
    float* l_s = corr_s + 8;
    float* sc = corr_s + 12;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::bar_off());
    uint64_t* empty = full + kAttnStages;
    __shared__ unsigned s_last;
    __shared__ int s_abort;

    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z, nsplit = gridDim.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = p.pos[b], Ltok = pos + 1;
    const int t0 = split * p.chunk, t1 = min(Ltok, t0 + p.chunk);
    const int ntiles = t1 > t0 ? (t1 - t0 + kT - 1) / kT : 0;
    const bool has_new = t0 <= pos && pos < t0 + p.chunk;
    const int rows0 = (int)(row_base + ((int64_t)b * p.Hkv + kvh) * p.cap + t0);
    const float* proj = p.proj + (size_t)b * p.ldp;
    const int half_rot = p.rot / 2;
    const float2* rope = p.rope + (size_t)pos * half_rot;
    constexpr uint32_t kStageTx = 2u * L::kTileBytes;

    if (threadIdx.x == 0) {
        s_abort = 0;
        for (int s = 0; s < kAttnStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kCompWarps * 32);
        }
        mbar_fence_init();
    }
    __syncthreads();

    // tiles that cannot hold the new position are independent of the prologue: start them now
    const int n_pre = min(kAttnStages, has_new ? ntiles - 1 : ntiles);
    const bool producer = warp == kCompWarps && lane == 0;
    if (producer) {
        for (int i = 0; i < n_pre; i++) {
            mbar_arrive_expect_tx(&full[i], kStageTx);
#pragma unroll
            for (int d = 0; d < NDB; d++) {
                tma_load_2d(smem + L::k_off(i) + d * 8192, &tmk, d * 64, rows0 + i * kT, &full[i]);
                tma_load_2d(smem + L::v_off(i) + d * 8192, &tmv, d * 64, rows0 + i * kT, &full[i]);
            }
        }
    }

    // ---- prologue: queries of the kGQ heads, new key / value (deltanet.rs:565-625)
    const int koff = p.Hq * 2 * HD, voff = koff + p.Hkv * HD;
    for (int i = threadIdx.x; i < kGQ * HD; i += kAttnMmaThreads) {
        const int hh = i / HD, d = i % HD, h = kvh * kGQ + hh;
        q_s[i] = proj[(size_t)h * 2 * HD + d];
    }
    if (has_new)
        for (int d = threadIdx.x; d < HD; d += kAttnMmaThreads) {
            kn_s[d] = proj[koff + kvh * HD + d];
            vn_s[d] = proj[voff + kvh * HD + d];
        }
    for (int i = threadIdx.x; i < 16 * kPStride; i += kAttnMmaThreads) P_s[i] = __float2bfloat16_rn(0.0f);
    __syncthreads();
    if (warp < kGQ && p.q_norm) {
        float ss = 0.0f;
        for (int d = lane; d < HD; d += 32) ss += q_s[warp * HD + d] * q_s[warp * HD + d];
        ss = warp_sum(ss);
        if (lane == 0) sc[warp] = 1.0f / sqrtf(ss / (float)HD + 1e-6f);
    }
    if (warp == kGQ && has_new && p.k_norm) {
        float ss = 0.0f;
        for (int d = lane; d < HD; d += 32) ss += kn_s[d] * kn_s[d];
        ss = warp_sum(ss);
        if (lane == 0) sc[kGQ] = 1.0f / sqrtf(ss / (float)HD + 1e-6f);
    }
    __syncthreads();
    if (p.q_norm)
        for (int i = threadIdx.x; i < kGQ * HD; i += kAttnMmaThreads) q_s[i] = q_s[i] * sc[i / HD] * p.q_norm[i % HD];
    if (has_new && p.k_norm)
        for (int d = threadIdx.x; d < HD; d += kAttnMmaThreads) kn_s[d] = kn_s[d] * sc[kGQ] * p.k_norm[d];
    __syncthreads();
    for (int i = threadIdx.x; i < (kGQ + 1) * half_rot; i += kAttnMmaThreads) {
        const int hh = i / half_rot, j = i % half_rot;
        if (hh == kGQ && !has_new) continue;
        float* t = hh < kGQ ? q_s + hh * HD : kn_s;
        const float2 cs = rope[j];
        const float a0 = t[2 * j], a1 = t[2 * j + 1];
        t[2 * j] = a0 * cs.x - a1 * cs.y;
        t[2 * j + 1] = a0 * cs.y + a1 * cs.x;
    }
    __syncthreads();
    if (has_new) {
        __nv_bfloat16* kc = reinterpret_cast<__nv_bfloat16*>(p.kc) + (size_t)b * p.kv_slot_stride +
                            (size_t)kvh * p.cap * HD + (size_t)pos * HD;
        __nv_bfloat16* vc = reinterpret_cast<__nv_bfloat16*>(p.vc) + (size_t)b * p.kv_slot_stride +
                            (size_t)kvh * p.cap * HD + (size_t)pos * HD;
        for (int d = threadIdx.x; d < HD; d += kAttnMmaThreads) {
            kc[d] = __float2bfloat16_rn(kn_s[d]);
            vc[d] = __float2bfloat16_rn(vn_s[d]);
        }
        asm volatile("fence.proxy.async.global;" ::: "memory");  // visible to the TMA reads below
    }
    __syncthreads();

    if (warp == kCompWarps) {
        // ---------------- producer: the remaining tiles
        if (lane == 0) {
            int issued = n_pre;
            for (int i = n_pre; i < ntiles; i++) {
                const int s = i % kAttnStages;
                if (i >= kAttnStages && !mbar_wait(&empty[s], ((i / kAttnStages) - 1) & 1)) {
                    s_abort = 1;
                    break;
                }
                if (*(volatile int*)&s_abort) break;
                mbar_arrive_expect_tx(&full[s], kStageTx);
#pragma unroll
                for (int d = 0; d < NDB; d++) {
                    tma_load_2d(smem + L::k_off(s) + d * 8192, &tmk, d * 64, rows0 + i * kT, &full[s]);
                    tma_load_2d(smem + L::v_off(s) + d * 8192, &tmv, d * 64, rows0 + i * kT, &full[s]);
                }
                issued = i + 1;
            }
            // every issued tile lands before the CTA can exit
            for (int j = max(0, issued - kAttnStages); j < issued; j++)
                if (!mbar_wait(&full[j % kAttnStages], (j / kAttnStages) & 1)) s_abort = 1;
        }
        __syncwarp();  // lanes 1-31 wait for the producer lane before the CTA barrier below
    } else {
        // ---------------- compute warps
        const int g = lane >> 2, t = lane & 3;
        const int hq = g & 3;             // head of this lane's operand row (rows 0-3 hi, 4-7 lo)
        const bool lo_row = g >= 4;
        // Q A-fragments for every k16 step: a0 = (row g, k 2t..2t+1), a2 = (row g, k 2t+8..+9)
        uint32_t qa0[HD / 16], qa2[HD / 16];
#pragma unroll
        for (int ks = 0; ks < HD / 16; ks++) {
            const float* qr = q_s + hq * HD + ks * 16;
            float x0 = qr[2 * t], x1 = qr[2 * t + 1], x2 = qr[2 * t + 8], x3 = qr[2 * t + 9];
            float h0, l0, h1, l1, h2, l2, h3, l3;
            split_bf16(x0, h0, l0);
            split_bf16(x1, h1, l1);
            split_bf16(x2, h2, l2);
            split_bf16(x3, h3, l3);
            qa0[ks] = lo_row ? pack_bf16(l0, l1) : pack_bf16(h0, h1);
            qa2[ks] = lo_row ? pack_bf16(l2, l3) : pack_bf16(h2, h3);
        }
        constexpr int NPV = HD / 32;  // 8-dim n-tiles of this warp's HD/4 output dims
        float o[NPV][4];
#pragma unroll
        for (int n = 0; n < NPV; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
        float m_run = -INFINITY, l_run = 0.0f;  // head `warp` (warps 0..3 own heads 0..3)
        const float sq = sqrtf((float)HD);
        const uint32_t pbase = smem_u32(P_s);

        for (int i = 0; i < ntiles; i++) {
            const int s = i % kAttnStages;
            if (!mbar_wait(&full[s], (i / kAttnStages) & 1)) {
                s_abort = 1;
                break;
            }
            const uint32_t kb = smem_u32(smem + L::k_off(s)), vb = smem_u32(smem + L::v_off(s));
            const int tbase = t0 + i * kT;
            // S = Q K^T for tokens [16w, 16w+16) of the tile
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const int n0 = 16 * warp + 8 * j;
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
                const int row = n0 + (lane & 7);
#pragma unroll
                for (int kk = 0; kk < HD / 32; kk++) {
                    const int chunk = kk * 4 + (lane >> 3);
                    const uint32_t addr = kb + (chunk >> 3) * 8192 + row * 128 + (((chunk & 7) ^ (row & 7)) << 4);
                    uint32_t r0, r1, r2, r3;
                    ldsm_x4(addr, r0, r1, r2, r3);
                    mma_bf16(acc, qa0[2 * kk], 0u, qa2[2 * kk], 0u, r0, r1);
                    mma_bf16(acc, qa0[2 * kk + 1], 0u, qa2[2 * kk + 1], 0u, r2, r3);
                }
                const float s0 = acc[0] + __shfl_xor_sync(kFull, acc[0], 16);
                const float s1 = acc[1] + __shfl_xor_sync(kFull, acc[1], 16);
                if (g < 4) {
                    const int tt = n0 + 2 * t;
                    S_s[g * kT + tt] = (tbase + tt < t1) ? s0 / sq : -INFINITY;
                    S_s[g * kT + tt + 1] = (tbase + tt + 1 < t1) ? s1 / sq : -INFINITY;
                }
            }
            asm volatile("bar.sync 1, %0;" ::"n"(kCompWarps * 32) : "memory");
            // online softmax for head `warp` over the tile's 64 tokens
            {
                const float v0 = S_s[warp * kT + lane], v1 = S_s[warp * kT + lane + 32];
                const float mx = warp_max(fmaxf(v0, v1));
                const float m_new = fmaxf(m_run, mx);
                float p0 = 0.0f, p1 = 0.0f, corr = 1.0f;
                if (m_new != -INFINITY) {
                    p0 = v0 == -INFINITY ? 0.0f : expf(v0 - m_new);
                    p1 = v1 == -INFINITY ? 0.0f : expf(v1 - m_new);
                    corr = m_run == -INFINITY ? 0.0f : expf(m_run - m_new);
                }
                l_run = l_run * corr + warp_sum(p0 + p1);
                m_run = m_new;
                float ph, pl;
                split_bf16(p0, ph, pl);
                P_s[warp * kPStride + lane] = __float2bfloat16_rn(ph);
                P_s[(warp + 4) * kPStride + lane] = __float2bfloat16_rn(pl);
                split_bf16(p1, ph, pl);
                P_s[warp * kPStride + lane + 32] = __float2bfloat16_rn(ph);
                P_s[(warp + 4) * kPStride + lane + 32] = __float2bfloat16_rn(pl);
                if (lane == 0) corr_s[warp] = corr;
            }
            asm volatile("bar.sync 1, %0;" ::"n"(kCompWarps * 32) : "memory");
            // O = O * corr + P V for dims [warp*HD/4, (warp+1)*HD/4)
            const float cr = corr_s[hq];
#pragma unroll
            for (int n = 0; n < NPV; n++) {
                o[n][0] *= cr;
                o[n][1] *= cr;
            }
#pragma unroll
            for (int kk = 0; kk < kT / 16; kk++) {
                uint32_t a0, a1, a2, a3;
                {
                    const int m = lane >> 3;
                    const int prow = (m & 1) * 8 + (lane & 7), pcol = kk * 16 + (m >> 1) * 8;
                    ldsm_x4(pbase + (prow * kPStride + pcol) * 2, a0, a1, a2, a3);
                }
#pragma unroll
                for (int np = 0; np < NPV / 2; np++) {
                    const int d0 = warp * (HD / 4) + np * 16;
                    const int m = lane >> 3;
                    const int tok = kk * 16 + (lane & 7) + (m & 1) * 8;
                    const int chunk = (d0 >> 3) + (m >> 1);
                    const uint32_t addr = vb + (chunk >> 3) * 8192 + tok * 128 + (((chunk & 7) ^ (tok & 7)) << 4);
                    uint32_t r0, r1, r2, r3;
                    ldsm_x4_t(addr, r0, r1, r2, r3);
                    mma_bf16(o[2 * np], a0, a1, a2, a3, r0, r1);
                    mma_bf16(o[2 * np + 1], a0, a1, a2, a3, r2, r3);
                }
            }
            mbar_arrive(&empty[s]);
        }
        // merge hi/lo rows: lanes g < 4 hold head g for dims d0 + 8n + 2t, +1
#pragma unroll
        for (int n = 0; n < NPV; n++) {
            o[n][0] += __shfl_xor_sync(kFull, o[n][0], 16);
            o[n][1] += __shfl_xor_sync(kFull, o[n][1], 16);
        }
        if (lane == 0) {
            m_s[warp] = m_run;
            l_s[warp] = l_run;
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kCompWarps * 32) : "memory");
        // unnormalised O of this CTA into q_s (reused as [4][HD])
        if (g < 4) {
#pragma unroll
            for (int n = 0; n < NPV; n++) {
                const int d = warp * (HD / 4) + 8 * n + 2 * t;
                q_s[g * HD + d] = o[n][0];
                q_s[g * HD + d + 1] = o[n][1];
            }
        }
    }
    __syncthreads();
    // a timed-out wait leaves this CTA's numbers invalid: report it, but keep taking part in
    // the split ticket below so the per-(sequence, head) counters stay consistent
    if (s_abort && threadIdx.x == 0 && p.err) atomicOr(p.err, 256u);

    // ---- finish: one split writes its partial; the last CTA merges in split order
    const size_t part_floats = (size_t)kGQ * 2 + (size_t)kGQ * HD;
    if (nsplit == 1) {
        for (int i = threadIdx.x; i < kGQ * HD; i += kAttnMmaThreads) {
            const int hh = i / HD, d = i % HD, h = kvh * kGQ + hh;
            float o = q_s[i] / l_s[hh];
            o *= ref_sigmoid(proj[(size_t)h * 2 * HD + HD + d]);
            act_store(p.out, b, h * HD + d, o);
            if (p.o_out) p.o_out[(size_t)b * p.Hq * HD + h * HD + d] = o;
        }
        return;
    }
    float* mypart = p.ws + (((size_t)b * p.Hkv + kvh) * nsplit + split) * part_floats;
    for (int i = threadIdx.x; i < kGQ * HD; i += kAttnMmaThreads) __stcg(mypart + 2 * kGQ + i, q_s[i]);
    if (threadIdx.x < kGQ) {
        __stcg(mypart + threadIdx.x, m_s[threadIdx.x]);
        __stcg(mypart + kGQ + threadIdx.x, l_s[threadIdx.x]);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(&p.tickets[b * p.Hkv + kvh], 1u);
        s_last = (prev == (unsigned)nsplit - 1u) ? 1u : 0u;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // merge: per-(split, head) weights e = exp(m_s - M) once into shared memory (the K/V ring
    // is idle now), then every output element sums its splits in split order
    const float* parts = p.ws + (((size_t)b * p.Hkv + kvh) * nsplit) * part_floats;
    float* e_s = reinterpret_cast<float*>(smem);  // [nsplit][kGQ]
    float* lsum_s = e_s + nsplit * kGQ;           // [kGQ]
    if (warp < kGQ) {
        float M = -INFINITY;
        for (int s = lane; s < nsplit; s += 32) M = fmaxf(M, __ldcg(parts + s * part_floats + warp));
        M = warp_max(M);
        for (int s = lane; s < nsplit; s += 32) {
            const float ms = __ldcg(parts + s * part_floats + warp);
            e_s[s * kGQ + warp] = (ms == -INFINITY) ? 0.0f : expf(ms - M);
        }
        __syncwarp();
        if (lane == 0) {
            float Lsum = 0.0f;
            for (int s = 0; s < nsplit; s++) Lsum += __ldcg(parts + s * part_floats + kGQ + warp) * e_s[s * kGQ + warp];
            lsum_s[warp] = Lsum;
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kGQ * HD; i += kAttnMmaThreads) {
        const int hh = i / HD, d = i % HD, h = kvh * kGQ + hh;
        float A = 0.0f;
#pragma unroll 8
        for (int s = 0; s < nsplit; s++) A += __ldcg(parts + s * part_floats + 2 * kGQ + i) * e_s[s * kGQ + hh];
        float o = A / lsum_s[hh];
        o *= ref_sigmoid(proj[(size_t)h * 2 * HD + HD + d]);
        act_store(p.out, b, h * HD + d, o);
        if (p.o_out) p.o_out[(size_t)b * p.Hq * HD + h * HD + d] = o;
    }
    if (threadIdx.x == 0) p.tickets[b * p.Hkv + kvh] = 0u;
}

// ------------------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

// 2-D map over a bf16 cache viewed as [rows][hd], boxes of 64 tokens x 64 dims, 128-byte swizzle
int make_kv_tensor_map(void* map_out, void* base, int64_t rows, int hd) {
    auto enc = tensor_map_encoder();
    if (!enc) return -1;
    cuuint64_t dims[2] = {(cuuint64_t)hd, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)hd * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)kT};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(reinterpret_cast<CUtensorMap*>(map_out), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -2;
}

// tokens per split for the tensor-core kernel: about seven CTA waves over the SMs, and at
// least kMinSplitTiles tiles per split so the pipeline fill and the merge stay small
constexpr int kMinSplitTiles = 4;
int attn_mma_chunk(int batch, int hkv, int max_len, int num_sms) {
    int pairs = batch * hkv;
    int want = (7 * num_sms + pairs - 1) / pairs;
    if (want < 1) want = 1;
    int chunk = (max_len + want - 1) / want;
    chunk = (chunk + kT - 1) / kT * kT;
    return chunk < kMinSplitTiles * kT ? kMinSplitTiles * kT : chunk;
}

// the split count is at most min(want, ceil(max_len / (kMinSplitTiles * kT)))
int attn_mma_nsplit_bound(int batch, int hkv, int cap, int num_sms) {
    int want = (7 * num_sms + batch * hkv - 1) / (batch * hkv);
    int by_len = (cap + kMinSplitTiles * kT - 1) / (kMinSplitTiles * kT);
    return want < by_len ? want : by_len;
}

template <int HD>
static int launch_mma_t(const void* tmk, const void* tmv, const AttnParams& p, int64_t row_base, int batch,
                        int max_len, cudaStream_t st) {
    const int smem = AttnSmem<HD>::bytes() + 1024;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev & 63]) {
        if (cudaFuncSetAttribute(attn_mma_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return -1;
        attr_set[dev & 63] = true;
    }
    dim3 grid(attn_nsplit(max_len, p.chunk), p.Hkv, batch);
    attn_mma_kernel<HD><<<grid, kAttnMmaThreads, smem, st>>>(*reinterpret_cast<const CUtensorMap*>(tmk),
                                                             *reinterpret_cast<const CUtensorMap*>(tmv), p, row_base);
    return 0;
}

int launch_attention_mma(const void* tmk, const void* tmv, const AttnParams& p, int64_t row_base, int batch, int hd,
                         int max_len, cudaStream_t st) {
    if (p.Hq != kGQ * p.Hkv) return -1;
    if (hd == 256) return launch_mma_t<256>(tmk, tmv, p, row_base, batch, max_len, st);
    if (hd == 128) return launch_mma_t<128>(tmk, tmv, p, row_base, batch, max_len, st);
    return -1;
}

}  // namespace ab2
