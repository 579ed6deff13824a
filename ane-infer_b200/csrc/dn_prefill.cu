// dn_prefill.cu -- chunked Gated DeltaNet prefill: the mixer of up to kPrefillChunk prompt
// tokens of one sequence per launch, between the input projection GEMM and the ssm_out GEMM.
//
// Per token the reference runs the recurrence of deltanet_decode_step
// (crates/engine/src/deltanet.rs:485-512) one step at a time:
//   S_t = d_t S_{t-1};  delta_t = beta_t (v_t - S_t^T k_t);  S_t += k_t delta_t^T;  o_t = S_t^T q_t.
// Over a chunk of T tokens with the state S0 before it and g_t = sum_{s<=t} log d_s, the same
// recurrence unrolls to (the chunkwise form of the delta rule, Yang et al., "Gated Delta
// Networks"; the algorithm the reference plans for its prefill, HANDOVER.md:67-72):
//   A[t][s] = beta_t e^{g_t - g_s} (k_t . k_s)    (s < t),     P[t][s] = e^{g_t - g_s} (q_t . k_s)  (s <= t)
//   (I + A) Delta = beta (V - e^g K S0)          (forward substitution over the chunk)
//   O = e^g Q S0 + P Delta,                      S_T = e^{g_{T-1}} S0 + K^T diag(e^{g_{T-1} - g}) Delta
// so the state is read and written once per chunk instead of once per token. The conv1d +
// SiLU over the chunk, the q/k L2 norms, beta, the decay and the gated RMSNorm times
// SiLU(gate) are the decode mixer's, token by token, fused around it.
//
// One CTA per head holds the head's 128 x 128 state and the chunk's q, k, v in shared
// memory (198 KB); the products run on the CUDA cores in f32, like the reference's.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace ab2 {
namespace {

constexpr int DK = 128;             // key_dim = value_dim
constexpr int kT = kPrefillChunk;   // tokens per launch
constexpr int kPfThreads = 512;
constexpr int kLd = DK + 4;         // padded row stride of q and k (conflict-free float4 rows)
constexpr int kLv = DK + 8;         // padded row stride of v / R / Delta (conflict-free substitution)

struct PfSmem {
    static constexpr int S = 0;                     // [DK][DK] state before the chunk
    static constexpr int K = S + DK * DK;           // [kT][kLd] normed keys
    static constexpr int Q = K + kT * kLd;          // [kT][kLd] normed, scaled queries; later O
    static constexpr int V = Q + kT * kLd;          // [kT][kLv] values; later R, then Delta
    static constexpr int A = V + kT * kLv;          // [kT][kT]
    static constexpr int P = A + kT * kT;           // [kT][kT]
    static constexpr int G = P + kT * kT;           // [kT] cumulative log-decay
    static constexpr int BETA = G + kT;             // [kT]
    static constexpr int EG = BETA + kT;            // [kT] e^{g_t}
    static constexpr int W = EG + kT;               // [kT] e^{g_{T-1} - g_t}
    static constexpr int floats = W + kT;
    static constexpr int bytes = floats * 4;
};
static_assert(PfSmem::bytes <= 227 * 1024, "prefill shared memory");

__device__ __forceinline__ float dot4(float4 a, float4 b, float acc) {
    acc += a.x * b.x;
    acc += a.y * b.y;
    acc += a.z * b.z;
    acc += a.w * b.w;
    return acc;
}

__global__ void __launch_bounds__(kPfThreads, 1) dn_prefill_kernel(DnParams p, int T) {
    extern __shared__ float4 pf_smem4[];
    float* sm = reinterpret_cast<float*>(pf_smem4);
    float* S = sm + PfSmem::S;
    float* Kb = sm + PfSmem::K;
    float* Qb = sm + PfSmem::Q;
    float* Vb = sm + PfSmem::V;
    float* A = sm + PfSmem::A;
    float* P = sm + PfSmem::P;
    float* g = sm + PfSmem::G;
    float* beta = sm + PfSmem::BETA;
    float* eg = sm + PfSmem::EG;
    float* w = sm + PfSmem::W;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int h = blockIdx.x, hg = p.h0 + h, H_all = p.H_all ? p.H_all : p.H;
    float* Sg = p.S + (size_t)h * DK * DK;

    // constants, before the grid dependency wait: this thread's conv channel weights, ssm_a, dt_bias
    const int ch_i = tid / DK, ch_c = tid % DK;                // q / k / v channel group and index
    const int ch = tid < 3 * DK ? ch_i * p.D + hg * DK + ch_c : -1;
    float4 cw = make_float4(0.f, 0.f, 0.f, 0.f);
    if (ch >= 0) cw = *reinterpret_cast<const float4*>(p.conv_w + (size_t)ch * 4);
    const float sa = p.ssm_a[hg], dtb = p.dt_bias[hg];
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    for (int e = tid; e < DK * DK / 4; e += kPfThreads)
        reinterpret_cast<float4*>(S)[e] = reinterpret_cast<const float4*>(Sg)[e];
    if (ch >= 0) {
        // conv_shift_and_append + conv_apply + SiLU per token (deltanet_cache.rs:34-54,
        // deltanet.rs:444-450), the window carried in registers across the chunk
        float* cs_g = p.conv + (size_t)ch * 4;
        float4 cs = *reinterpret_cast<const float4*>(cs_g);
        float* dst = ch_i == 0 ? Qb : ch_i == 1 ? Kb : Vb;
        const int ld = ch_i == 2 ? kLv : kLd;
        // the chunk's inputs of this channel are loaded 16 at a time ahead of the window's
        // serial dependency, so their latencies overlap
        for (int t0 = 0; t0 < T; t0 += 16) {
            float xin[16];
#pragma unroll
            for (int u = 0; u < 16; u++) xin[u] = t0 + u < T ? p.proj[(size_t)(t0 + u) * p.ldp + ch] : 0.0f;
#pragma unroll
            for (int u = 0; u < 16; u++) {
                if (t0 + u >= T) break;
                cs = make_float4(cs.y, cs.z, cs.w, xin[u]);
                float sum = cs.x * cw.x;
                sum += cs.y * cw.y;
                sum += cs.z * cw.z;
                sum += cs.w * cw.w;
                dst[(t0 + u) * ld + ch_c] = ref_silu(sum);
            }
        }
        *reinterpret_cast<float4*>(cs_g) = cs;
    } else if (tid - 3 * DK < T) {
        // beta = sigmoid(W_beta x) and log d = ssm_a * softplus(W_alpha x + dt_bias) (deltanet.rs:469-480)
        const int t = tid - 3 * DK;
        const float* pr = p.proj + (size_t)t * p.ldp;
        beta[t] = ref_sigmoid(pr[4 * p.D + hg]);
        g[t] = sa * ref_softplus(pr[4 * p.D + H_all + hg] + dtb);
    }
    __syncthreads();
    if (tid == 0) {
        float acc = 0.0f;
        for (int t = 0; t < T; t++) {
            acc += g[t];
            g[t] = acc;
        }
    }
    // per-token L2 norm of q (then * 1/sqrt(dk)) and k (deltanet.rs:459-467), a warp per row
    for (int r = warp; r < 2 * T; r += kPfThreads / 32) {
        float* v = r < T ? Qb + r * kLd : Kb + (r - T) * kLd;
        float xs[4], ss = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            xs[i] = v[lane + 32 * i];
            ss += xs[i] * xs[i];
        }
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss + 1e-12f);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float t = xs[i] * inv;
            if (r < T) t *= 1.0f / sqrtf((float)DK);
            v[lane + 32 * i] = t;
        }
    }
    __syncthreads();
    if (tid < T) {
        eg[tid] = expf(g[tid]);
        w[tid] = expf(g[T - 1] - g[tid]);
    }

    // A and P: warp w holds rows t = w + 16a, lane holds columns s = lane + 32b
    {
        float kk[4][2], qk[4][2];
#pragma unroll
        for (int a = 0; a < 4; a++)
#pragma unroll
            for (int b = 0; b < 2; b++) kk[a][b] = qk[a][b] = 0.0f;
        for (int i = 0; i < DK; i += 4) {
            float4 ks[2];
#pragma unroll
            for (int b = 0; b < 2; b++) ks[b] = *reinterpret_cast<const float4*>(Kb + (lane + 32 * b) * kLd + i);
#pragma unroll
            for (int a = 0; a < 4; a++) {
                const int t = warp + 16 * a;
                const float4 kt = *reinterpret_cast<const float4*>(Kb + t * kLd + i);
                const float4 qt = *reinterpret_cast<const float4*>(Qb + t * kLd + i);
#pragma unroll
                for (int b = 0; b < 2; b++) {
                    kk[a][b] = dot4(kt, ks[b], kk[a][b]);
                    qk[a][b] = dot4(qt, ks[b], qk[a][b]);
                }
            }
        }
#pragma unroll
        for (int a = 0; a < 4; a++)
#pragma unroll
            for (int b = 0; b < 2; b++) {
                const int t = warp + 16 * a, s = lane + 32 * b;
                const bool in = t < T && s <= t;  // rows and columns past T were never written
                const float e = in ? expf(g[t] - g[s]) : 0.0f;
                A[t * kT + s] = in && s < t ? beta[t] * e * kk[a][b] : 0.0f;
                P[t * kT + s] = in ? e * qk[a][b] : 0.0f;
            }
    }

    // R = beta (V - e^g K S0) and e^g Q S0; thread: column j, tokens [16 tg, 16 tg + 16)
    const int j = tid & (DK - 1), tg = tid >> 7;
    {
        float ks0[16], qs0[16];
#pragma unroll
        for (int u = 0; u < 16; u++) ks0[u] = qs0[u] = 0.0f;
        for (int i = 0; i < DK; i += 4) {
            const float4 s4 = make_float4(S[i * DK + j], S[(i + 1) * DK + j], S[(i + 2) * DK + j], S[(i + 3) * DK + j]);
#pragma unroll
            for (int u = 0; u < 16; u++) {
                const int t = tg * 16 + u;
                ks0[u] = dot4(*reinterpret_cast<const float4*>(Kb + t * kLd + i), s4, ks0[u]);
                qs0[u] = dot4(*reinterpret_cast<const float4*>(Qb + t * kLd + i), s4, qs0[u]);
            }
        }
        __syncthreads();  // every read of Q is done: it now holds O
#pragma unroll
        for (int u = 0; u < 16; u++) {
            const int t = tg * 16 + u;
            if (t < T) {
                Vb[t * kLv + j] = beta[t] * (Vb[t * kLv + j] - eg[t] * ks0[u]);
                Qb[t * kLd + j] = eg[t] * qs0[u];
            }
        }
    }
    __syncthreads();
    // (I + A) Delta = R by forward substitution. A column is four lanes of one warp (column
    // tid / 4, part tid % 4 over s = part, part + 4, ...), so a row's result needs only the warp.
    {
        const int col = tid >> 2, part = tid & 3;
        float* vc = Vb + col;
        for (int t = 1; t < T; t++) {
            const float* at = A + t * kT;
            float a = 0.0f;
            for (int s = part; s < t; s += 4) a += at[s] * vc[s * kLv];
            a += __shfl_xor_sync(0xffffffffu, a, 1);
            a += __shfl_xor_sync(0xffffffffu, a, 2);
            if (part == 0) vc[t * kLv] -= a;
            __syncwarp();
        }
    }
    __syncthreads();
    // O += P Delta (column j, tokens of group tg)
#pragma unroll 1
    for (int u = 0; u < 16; u++) {
        const int t = tg * 16 + u;
        if (t >= T) break;
        const float* pt = P + t * kT;
        float o0 = Qb[t * kLd + j], o1 = 0.0f;
        int s = 0;
        for (; s + 2 <= t + 1; s += 2) {
            o0 += pt[s] * Vb[s * kLv + j];
            o1 += pt[s + 1] * Vb[(s + 1) * kLv + j];
        }
        if (s <= t) o0 += pt[s] * Vb[s * kLv + j];
        Qb[t * kLd + j] = o0 + o1;
    }
    // S_T = e^{g_{T-1}} S0 + K^T diag(w) Delta (column j, rows [32 tg, 32 tg + 32)), to HBM
    {
        const float eT = eg[T - 1];
        float acc[32];
#pragma unroll
        for (int r = 0; r < 32; r++) acc[r] = eT * S[(tg * 32 + r) * DK + j];
        for (int t = 0; t < T; t++) {
            const float dw = w[t] * Vb[t * kLv + j];
            const float* kr = Kb + t * kLd + tg * 32;
#pragma unroll
            for (int r = 0; r < 32; r += 4) {
                const float4 k4 = *reinterpret_cast<const float4*>(kr + r);
                acc[r] += k4.x * dw;
                acc[r + 1] += k4.y * dw;
                acc[r + 2] += k4.z * dw;
                acc[r + 3] += k4.w * dw;
            }
        }
#pragma unroll
        for (int r = 0; r < 32; r++) Sg[(size_t)(tg * 32 + r) * DK + j] = acc[r];
    }
    __syncthreads();
    // gated RMSNorm with ssm_norm, times SiLU(gate) (deltanet.rs:514-533), a warp per token;
    // the sum of squares adds the four 32-column partials in the decode mixer's order
    for (int t = warp; t < T; t += kPfThreads / 32) {
        float ov[4], ss[4];
#pragma unroll
        for (int c = 0; c < 4; c++) {
            ov[c] = Qb[t * kLd + lane + 32 * c];
            ss[c] = warp_sum(ov[c] * ov[c]);
        }
        const float rms = 1.0f / sqrtf((ss[0] + ss[1] + ss[2] + ss[3]) / (float)DK + p.eps);
        const float* gate = p.proj + (size_t)t * p.ldp + 3 * p.D + hg * DK;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const int col = lane + 32 * c;
            const float gt = gate[col];
            float nv = ov[c] * rms * p.ssm_norm[col];
            nv *= gt / (1.0f + expf(-gt));
            act_store(p.out, t, hg * DK + col, nv);
            if (p.o_out) p.o_out[(size_t)t * p.D + hg * DK + col] = nv;
        }
    }
}

}  // namespace

int launch_dn_prefill(const DnParams& p, int tokens, cudaStream_t st) {
    if (tokens < 1 || tokens > kT || p.K != 4) return -1;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev & 63]) {
        if (cudaFuncSetAttribute(dn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PfSmem::bytes) !=
            cudaSuccess)
            return -2;
        attr_set[dev & 63] = true;
    }
    return launch_pdl(dn_prefill_kernel, dim3(p.H), dim3(kPfThreads), PfSmem::bytes, st, p, tokens) == cudaSuccess
               ? 0
               : -2;
}

}  // namespace ab2
