// deltanet.cu -- fused Gated DeltaNet decode mixer (everything between the input projection
// GEMM and the ssm_out GEMM of deltanet_decode_step, crates/engine/src/deltanet.rs:429-538).
//
// One CTA per (sequence, head). The head's 128x128 f32 state is read from HBM once with
// coalesced 16-byte loads into registers (8 warps x 16 rows, each lane 4 columns), decayed,
// used for S^T k, updated with the delta rule and used for S^T q, then written back once.
// conv1d + SiLU, the q/k L2 norms, beta = sigmoid, decay = exp(a * softplus(alpha + dt_bias)),
// the gated RMSNorm and the SiLU(gate) product are fused around it, and the result is
// written straight into the activation fragments of the ssm_out GEMM.
#include "common.cuh"
#include "kernels.h"

namespace ab2 {

constexpr int DK = 128;       // key_dim = value_dim = per-head channel count
constexpr int kDnThreads = 256;

// Gated delta rule on one head with the state in registers (deltanet.rs:485-512):
//   S *= decay; sk = S^T k; delta = beta (v - sk); S += k delta^T; o = S^T q
// q_s/k_s/v_s are shared [128] vectors; o_s receives the output.
// this thread's 16 rows x 4 columns of the head state (rows warp*16.., columns lane*4..)
__device__ __forceinline__ void load_state(const float* __restrict__ S, float4 s[16]) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int i = 0; i < 16; i++)
        s[i] = __ldcs(reinterpret_cast<const float4*>(S + (size_t)(warp * 16 + i) * DK + lane * 4));
}

// s[] holds the state loaded by load_state (issued early so HBM latency overlaps other work)
__device__ __forceinline__ void delta_rule_head(float4 s[16], float* __restrict__ S, const float* q_s, const float* k_s,
                                                const float* v_s, float beta, float decay, float* red /*[8][128]*/,
                                                float* delta_s, float* o_s) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r0 = warp * 16, c0 = lane * 4;
    float4 sk = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 16; i++) {
        s[i].x *= decay;
        s[i].y *= decay;
        s[i].z *= decay;
        s[i].w *= decay;
        const float kr = k_s[r0 + i];
        sk.x += s[i].x * kr;
        sk.y += s[i].y * kr;
        sk.z += s[i].z * kr;
        sk.w += s[i].w * kr;
    }
    *reinterpret_cast<float4*>(red + warp * DK + c0) = sk;
    __syncthreads();
    if (threadIdx.x < DK) {
        float a = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; w++) a += red[w * DK + threadIdx.x];
        delta_s[threadIdx.x] = beta * (v_s[threadIdx.x] - a);
    }
    __syncthreads();
    const float4 dl = *reinterpret_cast<const float4*>(delta_s + c0);
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 16; i++) {
        const float kr = k_s[r0 + i], qr = q_s[r0 + i];
        s[i].x += kr * dl.x;
        s[i].y += kr * dl.y;
        s[i].z += kr * dl.z;
        s[i].w += kr * dl.w;
        __stcs(reinterpret_cast<float4*>(S + (size_t)(r0 + i) * DK + c0), s[i]);
        o.x += s[i].x * qr;
        o.y += s[i].y * qr;
        o.z += s[i].z * qr;
        o.w += s[i].w * qr;
    }
    *reinterpret_cast<float4*>(red + warp * DK + c0) = o;
    __syncthreads();
    if (threadIdx.x < DK) {
        float a = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; w++) a += red[w * DK + threadIdx.x];
        o_s[threadIdx.x] = a;
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kDnThreads) deltanet_fused_kernel(DnParams p) {
    __shared__ __align__(16) float qkv_s[3][DK];
    __shared__ __align__(16) float red[8 * DK];
    __shared__ __align__(16) float delta_s[DK];
    __shared__ __align__(16) float o_s[DK];
    __shared__ float sc[4];
    const int h = blockIdx.x, b = blockIdx.y;
    const int D = p.D, H = p.H, K = p.K;
    const float* proj = p.proj + (size_t)b * p.ldp;
    float* S = p.S + (size_t)b * p.s_stride + (size_t)h * DK * DK;
    // launched with programmatic dependent launch: wait for the input projection, then let
    // the output projection start its weight prefetch
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    float4 st_regs[16];
    load_state(S, st_regs);  // 64 KB per CTA in flight while the prologue below runs

    // conv_shift_and_append + conv_apply + SiLU (deltanet_cache.rs:34-54, deltanet.rs:444-450)
    for (int c = threadIdx.x; c < 3 * DK; c += kDnThreads) {
        const int which = c / DK, j = c % DK;
        const int ch = which * D + h * DK + j;
        float* cs = p.conv + (size_t)b * p.conv_stride + (size_t)ch * K;
        const float* cw = p.conv_w + (size_t)ch * K;
        const float in = proj[ch];
        float sum = 0.0f;
        if (K == 4) {
            float4 st = *reinterpret_cast<float4*>(cs);
            const float4 w4 = *reinterpret_cast<const float4*>(cw);
            st = make_float4(st.y, st.z, st.w, in);
            *reinterpret_cast<float4*>(cs) = st;
            sum = st.x * w4.x;
            sum += st.y * w4.y;
            sum += st.z * w4.z;
            sum += st.w * w4.w;
        } else {
            for (int k = 0; k + 1 < K; k++) cs[k] = cs[k + 1];
            cs[K - 1] = in;
            for (int k = 0; k < K; k++) sum += cs[k] * cw[k];
        }
        qkv_s[which][j] = ref_silu(sum);
    }
    __syncthreads();

    // per-head L2 norm of q (then * 1/sqrt(dk)) and k (deltanet.rs:459-467)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp < 2) {
        float* v = qkv_s[warp];
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; i++) ss += v[lane + 32 * i] * v[lane + 32 * i];
        ss = warp_sum(ss);
        if (lane == 0) sc[warp] = 1.0f / sqrtf(ss + 1e-12f);
    } else if (warp == 2 && lane == 0) {
        // beta = sigmoid(W_beta x), decay = exp(ssm_a * softplus(W_alpha x + dt_bias)) (deltanet.rs:469-480)
        const float br = proj[4 * D + h], ar = proj[4 * D + H + h];
        sc[2] = ref_sigmoid(br);
        sc[3] = expf(p.ssm_a[h] * ref_softplus(ar + p.dt_bias[h]));
    }
    __syncthreads();
    if (threadIdx.x < 2 * DK) {
        const int which = threadIdx.x / DK, j = threadIdx.x % DK;
        float v = qkv_s[which][j] * sc[which];
        if (which == 0) v *= 1.0f / sqrtf((float)DK);
        qkv_s[which][j] = v;
    }
    __syncthreads();

    delta_rule_head(st_regs, S, qkv_s[0], qkv_s[1], qkv_s[2], sc[2], sc[3], red, delta_s, o_s);

    // gated RMSNorm with ssm_norm, times SiLU(gate) (deltanet.rs:514-533)
    if (warp == 0) {
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; i++) ss += o_s[lane + 32 * i] * o_s[lane + 32 * i];
        ss = warp_sum(ss);
        if (lane == 0) sc[0] = 1.0f / sqrtf(ss / (float)DK + p.eps);
    }
    __syncthreads();
    if (threadIdx.x < DK) {
        const int c = threadIdx.x;
        const float g = proj[3 * D + h * DK + c];
        float nv = o_s[c] * sc[0] * p.ssm_norm[c];
        nv *= g / (1.0f + expf(-g));
        act_store(p.out, b, h * DK + c, nv);
        if (p.o_out) p.o_out[(size_t)b * D + h * DK + c] = nv;
    }
}

// Recurrence-only op: q/k/v in bf16 (already normalised by the caller), beta and decay given.
__global__ void __launch_bounds__(kDnThreads) gated_delta_kernel(float* S, const uint16_t* __restrict__ q,
                                                                 const uint16_t* __restrict__ k,
                                                                 const uint16_t* __restrict__ v,
                                                                 const float* __restrict__ beta,
                                                                 const float* __restrict__ decay, int H, float* o) {
    __shared__ __align__(16) float qkv_s[3][DK];
    __shared__ __align__(16) float red[8 * DK];
    __shared__ __align__(16) float delta_s[DK];
    __shared__ __align__(16) float o_s[DK];
    const int bh = blockIdx.y * H + blockIdx.x;
    float4 st_regs[16];
    load_state(S + (size_t)bh * DK * DK, st_regs);
    for (int c = threadIdx.x; c < 3 * DK; c += kDnThreads) {
        const int which = c / DK, j = c % DK;
        const uint16_t* src = which == 0 ? q : (which == 1 ? k : v);
        qkv_s[which][j] = __uint_as_float((uint32_t)src[(size_t)bh * DK + j] << 16);
    }
    __syncthreads();
    delta_rule_head(st_regs, S + (size_t)bh * DK * DK, qkv_s[0], qkv_s[1], qkv_s[2], beta[bh], decay[bh], red, delta_s,
                    o_s);
    if (threadIdx.x < DK) o[(size_t)bh * DK + threadIdx.x] = o_s[threadIdx.x];
}

void launch_deltanet(const DnParams& p, int batch, cudaStream_t st) {
    dim3 grid(p.H, batch);
    launch_pdl(deltanet_fused_kernel, grid, dim3(kDnThreads), 0, st, p);
}

void launch_gated_delta(float* S, const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* beta,
                        const float* decay, int B, int H, float* o, cudaStream_t st) {
    dim3 grid(H, B);
    gated_delta_kernel<<<grid, kDnThreads, 0, st>>>(S, q, k, v, beta, decay, H, o);
}

}  // namespace ab2
