// attention.cu -- fused GQA decode attention (the part of full_attn_decode_step between the
// q/k/v projections and the W_o projection, crates/engine/src/deltanet.rs:565-669).
//
// Grid (split, kv_head, sequence). Every CTA rebuilds the GQ query heads that share its KV
// head: de-interleave [q | gate] per head, RMSNorm with q_norm (eps 1e-6), RoPE on adjacent
// pairs at the sequence position. The CTA whose split holds the new position also normalises
// and rotates the new key and appends k/v to the cache. Each CTA then runs an online-softmax
// pass over its slice of the cache, and the last CTA of a (sequence, kv_head) to finish
// (atomic ticket, no waiting) merges the split partials in split order, divides by the
// softmax sum, applies sigmoid(gate) and writes the W_o GEMM's activation fragments.
#include "common.cuh"
#include "kernels.h"

namespace ab2 {

constexpr int kAttnWarps = 8;

template <typename KV, int DPL>
struct RowLoad;

template <>
struct RowLoad<float, 8> {
    static __device__ __forceinline__ void load(const float* row, int lane, float* out) {
        const float4 a = *reinterpret_cast<const float4*>(row + lane * 8);
        const float4 c = *reinterpret_cast<const float4*>(row + lane * 8 + 4);
        out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
        out[4] = c.x; out[5] = c.y; out[6] = c.z; out[7] = c.w;
    }
};
template <>
struct RowLoad<float, 4> {
    static __device__ __forceinline__ void load(const float* row, int lane, float* out) {
        const float4 a = *reinterpret_cast<const float4*>(row + lane * 4);
        out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
    }
};
template <>
struct RowLoad<__nv_bfloat16, 8> {
    static __device__ __forceinline__ void load(const __nv_bfloat16* row, int lane, float* out) {
        const uint4 a = *reinterpret_cast<const uint4*>(row + lane * 8);
        out[0] = bf16lo(a.x); out[1] = bf16hi(a.x); out[2] = bf16lo(a.y); out[3] = bf16hi(a.y);
        out[4] = bf16lo(a.z); out[5] = bf16hi(a.z); out[6] = bf16lo(a.w); out[7] = bf16hi(a.w);
    }
};
template <>
struct RowLoad<__nv_bfloat16, 4> {
    static __device__ __forceinline__ void load(const __nv_bfloat16* row, int lane, float* out) {
        const uint2 a = *reinterpret_cast<const uint2*>(row + lane * 4);
        out[0] = bf16lo(a.x); out[1] = bf16hi(a.x); out[2] = bf16lo(a.y); out[3] = bf16hi(a.y);
    }
};

__device__ __forceinline__ void kv_store(float* p, float v) { *p = v; }
__device__ __forceinline__ void kv_store(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

// 32 per-lane partial values -> lane l holds the warp-wide sum of value l
__device__ __forceinline__ float transpose_reduce32(float v[32], int lane) {
#pragma unroll
    for (int lvl = 16; lvl >= 1; lvl >>= 1) {
        const bool upper = (lane & lvl) != 0;
#pragma unroll
        for (int i = 0; i < lvl; i++) {
            const float send = upper ? v[i] : v[i + lvl];
            const float keep = upper ? v[i + lvl] : v[i];
            v[i] = keep + __shfl_xor_sync(kFull, send, lvl);
        }
    }
    return v[0];
}

template <typename KV, int HD, int GQ>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_decode_kernel(AttnParams p) {
    static_assert(GQ * (32 / GQ) == 32, "GQ must divide 32");
    constexpr int DPL = HD / 32;
    constexpr int TG = 32 / GQ;  // tokens per warp iteration
    constexpr int NT = kAttnWarps * 32;
    __shared__ __align__(16) float q_s[GQ][HD];
    __shared__ __align__(16) float kn_s[HD];
    __shared__ __align__(16) float vn_s[HD];
    __shared__ float m_s[kAttnWarps][GQ], l_s[kAttnWarps][GQ];
    __shared__ __align__(16) float acc_s[kAttnWarps][GQ][HD];
    __shared__ float sc[GQ + 1];
    __shared__ unsigned s_last;

    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z, nsplit = gridDim.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int pos = p.pos[b], L = pos + 1;
    if (!attn_pos_ok(p, pos)) {  // nothing is appended or read at an out-of-range position
        if (threadIdx.x == 0 && split == 0 && kvh == 0 && p.err) atomicOr(p.err, kAttnErrPos);
        return;
    }
    const int t0 = split * p.chunk, t1 = min(L, t0 + p.chunk);
    const float* proj = p.proj + (size_t)b * p.ldp;
    KV* kc = reinterpret_cast<KV*>(p.kc) + (size_t)b * p.kv_slot_stride + (size_t)kvh * p.cap * HD;
    KV* vc = reinterpret_cast<KV*>(p.vc) + (size_t)b * p.kv_slot_stride + (size_t)kvh * p.cap * HD;
    const int half_rot = p.rot / 2;
    const float2* rope = p.rope + (size_t)pos * half_rot;

    // ---- queries of the GQ heads of this KV head (q/gate split, deltanet.rs:565-573)
    for (int i = threadIdx.x; i < GQ * HD; i += NT) {
        const int hh = i / HD, d = i % HD, h = kvh * GQ + hh;
        q_s[hh][d] = proj[(size_t)h * 2 * HD + d];
    }
    const bool has_new = t0 <= pos && pos < t0 + p.chunk;
    const int koff = p.Hq * 2 * HD, voff = koff + p.Hkv * HD;
    if (has_new) {
        for (int d = threadIdx.x; d < HD; d += NT) {
            kn_s[d] = proj[koff + kvh * HD + d];
            vn_s[d] = proj[voff + kvh * HD + d];
        }
    }
    __syncthreads();
    // q_norm / k_norm: RMSNorm with eps 1e-6 (deltanet.rs:575-598)
    if (warp < GQ && p.q_norm) {
        float ss = 0.0f;
        for (int d = lane; d < HD; d += 32) ss += q_s[warp][d] * q_s[warp][d];
        ss = warp_sum(ss);
        if (lane == 0) sc[warp] = 1.0f / sqrtf(ss / (float)HD + 1e-6f);
    }
    if (warp == GQ && has_new && p.k_norm) {
        float ss = 0.0f;
        for (int d = lane; d < HD; d += 32) ss += kn_s[d] * kn_s[d];
        ss = warp_sum(ss);
        if (lane == 0) sc[GQ] = 1.0f / sqrtf(ss / (float)HD + 1e-6f);
    }
    __syncthreads();
    if (p.q_norm)
        for (int i = threadIdx.x; i < GQ * HD; i += NT) {
            const int hh = i / HD, d = i % HD;
            q_s[hh][d] = q_s[hh][d] * sc[hh] * p.q_norm[d];
        }
    if (has_new && p.k_norm)
        for (int d = threadIdx.x; d < HD; d += NT) kn_s[d] = kn_s[d] * sc[GQ] * p.k_norm[d];
    __syncthreads();
    // RoPE on adjacent pairs (2i, 2i+1) with the host-built (cos, sin) table (deltanet.rs:600-623)
    for (int i = threadIdx.x; i < (GQ + 1) * half_rot; i += NT) {
        const int hh = i / half_rot, j = i % half_rot;
        if (hh == GQ && !has_new) continue;
        float* t = hh < GQ ? q_s[hh] : kn_s;
        const float2 cs = rope[j];
        const float a0 = t[2 * j], a1 = t[2 * j + 1];
        t[2 * j] = a0 * cs.x - a1 * cs.y;
        t[2 * j + 1] = a0 * cs.y + a1 * cs.x;
    }
    __syncthreads();
    // append the new key/value at pos (kv_cache.rs:32-40); visible to this CTA after the barrier
    if (has_new)
        for (int d = threadIdx.x; d < HD; d += NT) {
            kv_store(kc + (size_t)pos * HD + d, kn_s[d]);
            kv_store(vc + (size_t)pos * HD + d, vn_s[d]);
        }
    __syncthreads();

    // ---- online softmax over tokens [t0, t1)
    float qr[GQ][DPL];
#pragma unroll
    for (int hh = 0; hh < GQ; hh++)
#pragma unroll
        for (int d = 0; d < DPL; d++) qr[hh][d] = q_s[hh][lane * DPL + d];
    float acc[GQ][DPL];
#pragma unroll
    for (int hh = 0; hh < GQ; hh++)
#pragma unroll
        for (int d = 0; d < DPL; d++) acc[hh][d] = 0.0f;
    float m_run = -INFINITY, l_run = 0.0f;  // for head (lane % GQ), replicated over its lanes
    const float sq = sqrtf((float)HD);
    const int my_tt = lane / GQ, my_hh = lane % GQ;

    for (int tg0 = t0 + warp * TG; tg0 < t1; tg0 += kAttnWarps * TG) {
        float part[32];
#pragma unroll
        for (int tt = 0; tt < TG; tt++) {
            float kr[DPL];
            const int t = tg0 + tt;
            if (t < t1) {
                RowLoad<KV, DPL>::load(kc + (size_t)t * HD, lane, kr);
            } else {
#pragma unroll
                for (int d = 0; d < DPL; d++) kr[d] = 0.0f;
            }
#pragma unroll
            for (int hh = 0; hh < GQ; hh++) {
                float s = 0.0f;
#pragma unroll
                for (int d = 0; d < DPL; d++) s = fmaf(qr[hh][d], kr[d], s);
                part[tt * GQ + hh] = s;
            }
        }
        const float dot = transpose_reduce32(part, lane);
        const float score = (tg0 + my_tt < t1) ? dot / sq : -INFINITY;
        float gmax = score;
#pragma unroll
        for (int o = GQ; o < 32; o <<= 1) gmax = fmaxf(gmax, __shfl_xor_sync(kFull, gmax, o));
        const float m_new = fmaxf(m_run, gmax);
        const float pr = (score == -INFINITY) ? 0.0f : expf(score - m_new);
        const float corr = (m_run == -INFINITY) ? 0.0f : expf(m_run - m_new);
        float psum = pr;
#pragma unroll
        for (int o = GQ; o < 32; o <<= 1) psum += __shfl_xor_sync(kFull, psum, o);
        l_run = l_run * corr + psum;
        m_run = m_new;
#pragma unroll
        for (int hh = 0; hh < GQ; hh++) {
            const float c = __shfl_sync(kFull, corr, hh);
#pragma unroll
            for (int d = 0; d < DPL; d++) acc[hh][d] *= c;
        }
#pragma unroll
        for (int tt = 0; tt < TG; tt++) {
            const int t = tg0 + tt;
            if (t < t1) {
                float vr[DPL];
                RowLoad<KV, DPL>::load(vc + (size_t)t * HD, lane, vr);
#pragma unroll
                for (int hh = 0; hh < GQ; hh++) {
                    const float pp = __shfl_sync(kFull, pr, tt * GQ + hh);
#pragma unroll
                    for (int d = 0; d < DPL; d++) acc[hh][d] = fmaf(pp, vr[d], acc[hh][d]);
                }
            }
        }
    }
    (void)my_tt;

    // ---- merge the warps of this CTA
    if (lane < GQ) {
        m_s[warp][lane] = m_run;
        l_s[warp][lane] = l_run;
    }
#pragma unroll
    for (int hh = 0; hh < GQ; hh++)
#pragma unroll
        for (int d = 0; d < DPL; d++) acc_s[warp][hh][lane * DPL + d] = acc[hh][d];
    (void)my_hh;
    __syncthreads();

    const size_t part_floats = (size_t)GQ * 2 + (size_t)GQ * HD;
    float* mypart = p.ws + (((size_t)b * p.Hkv + kvh) * nsplit + split) * part_floats;
    for (int i = threadIdx.x; i < GQ * HD; i += NT) {
        const int hh = i / HD, d = i % HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAttnWarps; w++) M = fmaxf(M, m_s[w][hh]);
        float Lsum = 0.0f, A = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kAttnWarps; w++) {
                const float e = (m_s[w][hh] == -INFINITY) ? 0.0f : expf(m_s[w][hh] - M);
                Lsum += l_s[w][hh] * e;
                A += acc_s[w][hh][d] * e;
            }
        }
        if (nsplit == 1) {
            const int h = kvh * GQ + hh;
            float o = A / Lsum;
            o *= ref_sigmoid(proj[(size_t)h * 2 * HD + HD + d]);
            act_store(p.out, b, h * HD + d, o);
            if (p.o_out) p.o_out[(size_t)b * p.Hq * HD + h * HD + d] = o;
        } else {
            if (d == 0) {
                __stcg(mypart + hh, M);
                __stcg(mypart + GQ + hh, Lsum);
            }
            __stcg(mypart + 2 * GQ + i, A);
        }
    }
    if (nsplit == 1) return;

    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(&p.tickets[b * p.Hkv + kvh], 1u);
        s_last = (prev == (unsigned)nsplit - 1u) ? 1u : 0u;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float* parts = p.ws + (((size_t)b * p.Hkv + kvh) * nsplit) * part_floats;
    for (int i = threadIdx.x; i < GQ * HD; i += NT) {
        const int hh = i / HD, d = i % HD, h = kvh * GQ + hh;
        float M = -INFINITY;
        for (int s = 0; s < nsplit; s++) M = fmaxf(M, __ldcg(parts + s * part_floats + hh));
        float Lsum = 0.0f, A = 0.0f;
        for (int s = 0; s < nsplit; s++) {
            const float ms = __ldcg(parts + s * part_floats + hh);
            const float e = (ms == -INFINITY) ? 0.0f : expf(ms - M);
            Lsum += __ldcg(parts + s * part_floats + GQ + hh) * e;
            A += __ldcg(parts + s * part_floats + 2 * GQ + i) * e;
        }
        float o = A / Lsum;
        o *= ref_sigmoid(proj[(size_t)h * 2 * HD + HD + d]);
        act_store(p.out, b, h * HD + d, o);
        if (p.o_out) p.o_out[(size_t)b * p.Hq * HD + h * HD + d] = o;
    }
    if (threadIdx.x == 0) p.tickets[b * p.Hkv + kvh] = 0u;
}

int attn_nsplit(int max_len, int chunk) { return (max_len + chunk - 1) / chunk; }

static int attn_want(int batch, int hkv, int num_sms) {
    int want = (4 * num_sms + batch * hkv - 1) / (batch * hkv);
    return want < 1 ? 1 : want;
}

// tokens per split: about four CTAs per SM over the grid, at least 64 tokens per split.
// Since chunk >= max_len / want and chunk >= 64, the split count is at most
// min(want, ceil(max_len / 64)) (attn_nsplit_bound).
int attn_chunk(int batch, int hkv, int max_len, int num_sms) {
    int want = attn_want(batch, hkv, num_sms);
    int chunk = (max_len + want - 1) / want;
    chunk = (chunk + 63) / 64 * 64;
    return chunk < 64 ? 64 : chunk;
}

int attn_nsplit_bound(int batch, int hkv, int cap, int num_sms) {
    int want = attn_want(batch, hkv, num_sms);
    int by_len = (cap + 63) / 64;
    return want < by_len ? want : by_len;
}

size_t attn_ws_floats(int batch, int hkv, int nsplit, int hd, int gq) {
    return (size_t)batch * hkv * nsplit * ((size_t)gq * 2 + (size_t)gq * hd);
}

int launch_attention(const AttnParams& p, int batch, int hd, bool kv_bf16, int max_len, cudaStream_t st) {
    const int gq = p.Hq / p.Hkv;
    if (gq != 4) return -1;
    if (p.kvh0 != 0 || (p.Hkv_all && p.Hkv_all != p.Hkv)) return -1;  // the split runs the bf16 (tensor-core) path
    dim3 grid(attn_nsplit(max_len, p.chunk), p.Hkv, batch);
    const int nt = kAttnWarps * 32;
    if (hd == 256) {
        if (kv_bf16)
            attn_decode_kernel<__nv_bfloat16, 256, 4><<<grid, nt, 0, st>>>(p);
        else
            attn_decode_kernel<float, 256, 4><<<grid, nt, 0, st>>>(p);
    } else if (hd == 128) {
        if (kv_bf16)
            attn_decode_kernel<__nv_bfloat16, 128, 4><<<grid, nt, 0, st>>>(p);
        else
            attn_decode_kernel<float, 128, 4><<<grid, nt, 0, st>>>(p);
    } else {
        return -1;
    }
    return 0;
}

}  // namespace ab2
