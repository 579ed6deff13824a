// deltanet.cu -- fused Gated DeltaNet decode mixer (everything between the input projection
// GEMM and the ssm_out GEMM of deltanet_decode_step, crates/engine/src/deltanet.rs:429-538).
//
// Each head's 128x128 f32 state is read from HBM once into registers (8 warps x 16 rows, each
// lane 4 columns), decayed, used for S^T k, updated with the delta rule and used for S^T q,
// then written back once with coalesced 16-byte stores. conv1d + SiLU, the q/k L2 norms,
// beta = sigmoid, decay = exp(a * softplus(alpha + dt_bias)), the gated RMSNorm and the
// SiLU(gate) product are fused around it, and the result is written straight into the
// activation fragments of the ssm_out GEMM.
//
// deltanet_persist_kernel (the decode path) runs one CTA per SM over the (sequence, head)
// items and stages the states through a ring of shared-memory slots filled by bulk copies;
// gated_delta_kernel (the recurrence-only op) runs the same delta rule with one CTA per item.
#include "common.cuh"
#include "kernels.h"
#include "umma.cuh"

#include <algorithm>

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

// ------------------------------------------------------------------------------------------
// Persistent form of the fused mixer: CTA c takes the (sequence, head) items c, c + grid, ...
// Each head's 64 KB state is copied into one of kDnSlots shared-memory slots with bulk copies
// (four 16 KB pieces) issued kDnSlots heads ahead, read into registers (the same 16-row x
// 4-column split as delta_rule_head), updated there and written back to global memory
// with coalesced 16-byte stores, so the slot is refilled as soon as the registers hold it.
// The per-head inputs (conv1d + SiLU of q/k/v, their L2 norms, beta, decay and SiLU(gate))
// are prepared for kDnGroup heads at a time with every global load of the group in flight
// at once, so their latency is paid once per group rather than once per head.
constexpr int kDnSlots = 3;
constexpr int kDnGroup = 8;
constexpr int kStateBytes = DK * DK * 4;
constexpr int kConvPerThread = kDnGroup * 3 * DK / kDnThreads;  // 12
constexpr int kGatePerThread = kDnGroup * DK / kDnThreads;      // 4

struct DnItem {
    int b, h;
};
__device__ __forceinline__ DnItem dn_item(int j, int H) {
    const int item = blockIdx.x + j * gridDim.x;
    return {item / H, item % H};
}

// The inputs of a group that do not come from the input projection: the conv states and
// conv weights of this thread's channels (conv_k = 4), and ssm_a / dt_bias of item jg + tid.
struct DnGroupIn {
    float4 st[kConvPerThread], w4[kConvPerThread];
    float sa, dtb;
};

__device__ __forceinline__ void dn_group_load(const DnParams& p, int jg, int ng, DnGroupIn& g) {
    const int tid = threadIdx.x;
    const int D = p.D, H = p.H;
    const int nconv = ng * 3 * DK;
    g.sa = 0.0f;
    g.dtb = 0.0f;
    if (tid < ng) {
        const DnItem it = dn_item(jg + tid, H);
        g.sa = p.ssm_a[it.h];
        g.dtb = p.dt_bias[it.h];
    }
    if (p.K != 4) return;
#pragma unroll
    for (int u = 0; u < kConvPerThread; u++) {
        const int e = tid + u * kDnThreads;
        if (e < nconv) {
            const int i = e / (3 * DK), rem = e % (3 * DK);
            const DnItem it = dn_item(jg + i, H);
            const int ch = (rem / DK) * D + it.h * DK + rem % DK;
            g.st[u] = *reinterpret_cast<const float4*>(p.conv + (size_t)it.b * p.conv_stride + (size_t)ch * 4);
            g.w4[u] = *reinterpret_cast<const float4*>(p.conv_w + (size_t)ch * 4);
        }
    }
}

// conv_shift_and_append + conv_apply + SiLU (deltanet_cache.rs:34-54, deltanet.rs:444-450),
// SiLU(gate) (deltanet.rs:527-533), beta = sigmoid(W_beta x) and
// decay = exp(ssm_a * softplus(W_alpha x + dt_bias)) (deltanet.rs:469-480) for items jg..jg+ng-1,
// then the per-head L2 norms of q (times 1/sqrt(dk)) and k (deltanet.rs:459-467)
__device__ __forceinline__ void dn_prepare_group(const DnParams& p, int jg, int ng, const DnGroupIn& g,
                                                 float (*qkv)[3][DK], float (*gs)[DK], float (*bd)[2]) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int D = p.D, H = p.H, K = p.K;
    const int nconv = ng * 3 * DK;
    // gate, beta and decay inputs: loads issued first, consumed after the conv loop
    float graw[kGatePerThread];
#pragma unroll
    for (int u = 0; u < kGatePerThread; u++) {
        const int e = tid + u * kDnThreads;
        graw[u] = 0.0f;
        if (e < ng * DK) {
            const DnItem it = dn_item(jg + e / DK, H);
            graw[u] = p.proj[(size_t)it.b * p.ldp + 3 * D + it.h * DK + e % DK];
        }
    }
    float br = 0.0f, ar = 0.0f;
    if (tid < ng) {
        const DnItem it = dn_item(jg + tid, H);
        const float* proj = p.proj + (size_t)it.b * p.ldp;
        br = proj[4 * D + it.h];
        ar = proj[4 * D + H + it.h];
    }
    if (K == 4) {
        float in[kConvPerThread];
#pragma unroll
        for (int u = 0; u < kConvPerThread; u++) {
            const int e = tid + u * kDnThreads;
            if (e < nconv) {
                const int i = e / (3 * DK), rem = e % (3 * DK);
                const DnItem it = dn_item(jg + i, H);
                in[u] = p.proj[(size_t)it.b * p.ldp + (rem / DK) * D + it.h * DK + rem % DK];
            }
        }
#pragma unroll
        for (int u = 0; u < kConvPerThread; u++) {
            const int e = tid + u * kDnThreads;
            if (e < nconv) {
                const int i = e / (3 * DK), rem = e % (3 * DK);
                const DnItem it = dn_item(jg + i, H);
                const int ch = (rem / DK) * D + it.h * DK + rem % DK;
                const float4 s4 = make_float4(g.st[u].y, g.st[u].z, g.st[u].w, in[u]);
                *reinterpret_cast<float4*>(p.conv + (size_t)it.b * p.conv_stride + (size_t)ch * 4) = s4;
                float sum = s4.x * g.w4[u].x;
                sum += s4.y * g.w4[u].y;
                sum += s4.z * g.w4[u].z;
                sum += s4.w * g.w4[u].w;
                qkv[i][rem / DK][rem % DK] = ref_silu(sum);
            }
        }
    } else {
        for (int e = tid; e < nconv; e += kDnThreads) {
            const int i = e / (3 * DK), rem = e % (3 * DK);
            const DnItem it = dn_item(jg + i, H);
            const int ch = (rem / DK) * D + it.h * DK + rem % DK;
            float* cs = p.conv + (size_t)it.b * p.conv_stride + (size_t)ch * K;
            const float* cw = p.conv_w + (size_t)ch * K;
            for (int k = 0; k + 1 < K; k++) cs[k] = cs[k + 1];
            cs[K - 1] = p.proj[(size_t)it.b * p.ldp + ch];
            float sum = 0.0f;
            for (int k = 0; k < K; k++) sum += cs[k] * cw[k];
            qkv[i][rem / DK][rem % DK] = ref_silu(sum);
        }
    }
#pragma unroll
    for (int u = 0; u < kGatePerThread; u++) {
        const int e = tid + u * kDnThreads;
        if (e < ng * DK) gs[e / DK][e % DK] = graw[u] / (1.0f + expf(-graw[u]));
    }
    if (tid < ng) {
        bd[tid][0] = ref_sigmoid(br);
        bd[tid][1] = expf(g.sa * ref_softplus(ar + g.dtb));
    }
    __syncthreads();
    for (int v = warp; v < 2 * ng; v += kDnThreads / 32) {
        float* x = qkv[v >> 1][v & 1];
        float xs[4], ss = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            xs[i] = x[lane + 32 * i];
            ss += xs[i] * xs[i];
        }
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss + 1e-12f);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float t = xs[i] * inv;
            if ((v & 1) == 0) t *= 1.0f / sqrtf((float)DK);
            x[lane + 32 * i] = t;
        }
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kDnThreads, 1) deltanet_persist_kernel(DnParams p, int n_items) {
    extern __shared__ uint8_t dn_smem_raw[];
    float* slots = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(dn_smem_raw) + 127) & ~(uintptr_t)127);
    __shared__ __align__(16) float qkv[kDnGroup][3][DK];
    __shared__ __align__(16) float gs[kDnGroup][DK];
    __shared__ float bd[kDnGroup][2];
    __shared__ __align__(16) float red[8 * DK];
    __shared__ __align__(16) float delta_s[DK];
    __shared__ float ssp[4];
    __shared__ uint64_t full[kDnSlots];
    __shared__ int s_abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int H = p.H;
    const int G = gridDim.x;
    const int nmy = n_items > (int)blockIdx.x ? (n_items - (int)blockIdx.x + G - 1) / G : 0;

    if (tid == 0) {
        s_abort = 0;
        for (int s = 0; s < kDnSlots; s++) mbar_init(&full[s], 1);
        mbar_fence_init();
    }
    __syncthreads();
    auto state_of = [&](int j) {
        const DnItem it = dn_item(j, H);
        return p.S + (size_t)it.b * p.s_stride + (size_t)it.h * DK * DK;
    };
    auto load = [&](int j) {  // thread 0
        const int s = j % kDnSlots;
        float* dst = slots + (size_t)s * DK * DK;
        const float* src = state_of(j);
        mbar_arrive_expect_tx(&full[s], kStateBytes);
#pragma unroll
        for (int c = 0; c < 4; c++)
            bulk_g2s(dst + c * (DK * DK / 4), src + c * (DK * DK / 4), kStateBytes / 4, &full[s]);
    };
    // Launched with programmatic dependent launch behind the input projection GEMM, which lets
    // this grid start once the GEMM has set up. The GEMM itself started only after the kernel
    // before it (the RMSNorm, which waits for its own predecessor before it lets the next
    // kernel start) had waited, so every kernel before that RMSNorm has completed, among them
    // this layer's mixer of the previous step: the head states, conv states and weights can be
    // read now. Only the projection output needs the wait.
    int issued = 0;  // thread 0: items whose state load has been issued
    if (tid == 0) {
        for (; issued < min(kDnSlots, nmy); issued++) load(issued);
        if (issued == nmy) prefetch_share_l2(p.pf, p.pf_bytes, blockIdx.x, G);
    }
    DnGroupIn gin;
    dn_group_load(p, 0, min(kDnGroup, nmy), gin);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    const int r0 = warp * 16, c0 = lane * 4;  // this thread's 16 rows x 4 columns of a head state
    for (int jg = 0; jg < nmy; jg += kDnGroup) {
        const int ng = min(kDnGroup, nmy - jg);
        if (jg > 0) {
            __syncthreads();  // the previous group's inputs are no longer read
            dn_group_load(p, jg, ng, gin);
        }
        dn_prepare_group(p, jg, ng, gin, qkv, gs, bd);
        for (int i = 0; i < ng; i++) {
            const int j = jg + i;
            const DnItem it = dn_item(j, H);
            const float* Ss = slots + (size_t)(j % kDnSlots) * DK * DK;
            // every thread observes the copy's completion itself, so the bytes it reads from
            // the slot are ones the bulk copy wrote
            if (!mbar_wait(&full[j % kDnSlots], (j / kDnSlots) & 1)) s_abort = 1 + j;
            __syncthreads();
            if (s_abort) break;

            // gated delta rule (deltanet.rs:485-512):
            //   S *= decay; sk = S^T k; delta = beta (v - sk); S += k delta^T; o = S^T q
            const float beta = bd[i][0], decay = bd[i][1];
            const float* qv = qkv[i][0];
            const float* kv = qkv[i][1];
            float4 s[16];
            float4 sk = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int r = 0; r < 16; r++) {
                s[r] = *reinterpret_cast<const float4*>(Ss + (r0 + r) * DK + c0);
                s[r].x *= decay;
                s[r].y *= decay;
                s[r].z *= decay;
                s[r].w *= decay;
                const float kr = kv[r0 + r];
                sk.x += s[r].x * kr;
                sk.y += s[r].y * kr;
                sk.z += s[r].z * kr;
                sk.w += s[r].w * kr;
            }
            *reinterpret_cast<float4*>(red + warp * DK + c0) = sk;
            __syncthreads();  // the slot has been read into registers
            if (tid == 0 && issued < nmy) {
                load(issued++);
                // the last head-state copy of this CTA is on its way: pull this CTA's share of
                // the output projection's weights into L2 for the GEMM that follows
                if (issued == nmy) prefetch_share_l2(p.pf, p.pf_bytes, blockIdx.x, G);
            }
            if (tid < DK) {
                float a = 0.0f;
#pragma unroll
                for (int w = 0; w < 8; w++) a += red[w * DK + tid];
                delta_s[tid] = beta * (qkv[i][2][tid] - a);
            }
            __syncthreads();
            float* Sg = const_cast<float*>(state_of(j));
            const float4 dl = *reinterpret_cast<const float4*>(delta_s + c0);
            float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int r = 0; r < 16; r++) {
                const float kr = kv[r0 + r], qr = qv[r0 + r];
                s[r].x += kr * dl.x;
                s[r].y += kr * dl.y;
                s[r].z += kr * dl.z;
                s[r].w += kr * dl.w;
                __stcs(reinterpret_cast<float4*>(Sg + (size_t)(r0 + r) * DK + c0), s[r]);
                o.x += s[r].x * qr;
                o.y += s[r].y * qr;
                o.z += s[r].z * qr;
                o.w += s[r].w * qr;
            }
            *reinterpret_cast<float4*>(red + warp * DK + c0) = o;
            __syncthreads();
            // gated RMSNorm with ssm_norm, times SiLU(gate) (deltanet.rs:514-533)
            float ov = 0.0f;
            if (tid < DK) {
#pragma unroll
                for (int w = 0; w < 8; w++) ov += red[w * DK + tid];
                const float ss = warp_sum(ov * ov);
                if (lane == 0) ssp[warp] = ss;
            }
            __syncthreads();
            if (tid < DK) {
                const float rms = 1.0f / sqrtf((ssp[0] + ssp[1] + ssp[2] + ssp[3]) / (float)DK + p.eps);
                float nv = ov * rms * p.ssm_norm[tid];
                nv *= gs[i][tid];
                act_store(p.out, it.b, it.h * DK + tid, nv);
                if (p.o_out) p.o_out[(size_t)it.b * p.D + it.h * DK + tid] = nv;
            }
        }
        if (s_abort) break;
    }
    if (tid == 0 && s_abort) {
        // a state copy timed out: report it, then give the copies still in flight into the
        // slots a bounded time to land before the CTA's shared memory is released
        if (p.err) atomicOr(p.err, 1024u);
        for (int k = s_abort - 1; k < issued; k++) mbar_wait(&full[k % kDnSlots], (k / kDnSlots) & 1);
    }
}

void launch_deltanet(const DnParams& p, int batch, cudaStream_t st) {
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const int smem = kDnSlots * kStateBytes + 128;
    if (!attr_set[dev & 63]) {
        cudaFuncSetAttribute(deltanet_persist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        attr_set[dev & 63] = true;
    }
    int nsm = 148;
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    const int n_items = p.H * batch;
    launch_pdl(deltanet_persist_kernel, dim3(std::min(n_items, nsm)), dim3(kDnThreads), smem, st, p, n_items);
}

void launch_gated_delta(float* S, const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* beta,
                        const float* decay, int B, int H, float* o, cudaStream_t st) {
    dim3 grid(H, B);
    gated_delta_kernel<<<grid, kDnThreads, 0, st>>>(S, q, k, v, beta, decay, H, o);
}

}  // namespace ab2
