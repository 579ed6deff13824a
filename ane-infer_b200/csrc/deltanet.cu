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
// Two warp groups share the work:
//   * eight update warps run the delta rule: each head's 64 KB state is copied into one of
//     kDnSlots shared-memory slots with bulk copies (four 16 KB pieces) issued kDnSlots heads
//     ahead, read into registers (the same 16-row x 4-column split as delta_rule_head),
//     updated there and written back to global memory with coalesced 16-byte stores, so the
//     slot is refilled as soon as the registers hold it;
//   * four prep warps prepare the per-head inputs one or more heads ahead into a ring of
//     kPrepSlots shared-memory slots: conv1d shift/append + SiLU of q/k/v, their L2 norms,
//     beta, decay and SiLU(gate), with the global loads of the next head issued while the
//     current one is computed.
// The groups hand slots to each other through mbarriers and synchronise internally on their
// own named barriers, so neither waits for the other's internal steps.
constexpr int kDnSlots = 3;
constexpr int kPrepSlots = 3;
constexpr int kStateBytes = DK * DK * 4;
constexpr int kUpdThreads = 256, kPrepThreads = 128;
constexpr int kDnPersistThreads = kUpdThreads + kPrepThreads;
constexpr int kUpdBar = 1, kPrepBar = 2;  // named barriers (0 is __syncthreads)

struct DnItem {
    int b, h;
};
__device__ __forceinline__ DnItem dn_item(int j, int H) {
    const int item = blockIdx.x + j * gridDim.x;
    return {item / H, item % H};
}

struct PrepSlot {
    float qkv[3][DK];  // q, k (normalised; q also scaled by 1/sqrt(dk)), v
    float g[DK];       // SiLU(gate)
    float beta, decay;
};

// Global inputs of one head for one prep thread (channel `tid` of each of q, k, v).
struct PrepIn {
    float4 st[3], w4[3];  // conv states and conv weights (conv_k = 4)
    float in[3], g;       // projection outputs: q/k/v channel and gate
    float br, ar, sa, dtb;  // thread 0: beta/alpha inputs, ssm_a, dt_bias
};

// loads that do not depend on the input projection: conv states and weights, ssm_a, dt_bias
__device__ __forceinline__ void prep_load_const(const DnParams& p, int j, int tid, PrepIn& in) {
    const DnItem it = dn_item(j, p.H);
    const int hg = p.h0 + it.h;  // the head's index in the model
    if (p.K == 4) {
#pragma unroll
        for (int i = 0; i < 3; i++) {
            const int ch = i * p.D + hg * DK + tid;
            in.st[i] = *reinterpret_cast<const float4*>(p.conv + (size_t)it.b * p.conv_stride + (size_t)ch * 4);
            in.w4[i] = *reinterpret_cast<const float4*>(p.conv_w + (size_t)ch * 4);
        }
    }
    if (tid == 0) {
        in.sa = p.ssm_a[hg];
        in.dtb = p.dt_bias[hg];
    }
}
// loads of the projection outputs (after the grid dependency wait)
__device__ __forceinline__ void prep_load_proj(const DnParams& p, int j, int tid, PrepIn& in) {
    const DnItem it = dn_item(j, p.H);
    const int hg = p.h0 + it.h, H_all = p.H_all ? p.H_all : p.H;
    const float* proj = p.proj + (size_t)it.b * p.ldp;
#pragma unroll
    for (int i = 0; i < 3; i++) in.in[i] = proj[i * p.D + hg * DK + tid];
    in.g = proj[3 * p.D + hg * DK + tid];
    if (tid == 0) {
        in.br = proj[4 * p.D + hg];
        in.ar = proj[4 * p.D + H_all + hg];
    }
}

// conv_shift_and_append + conv_apply + SiLU (deltanet_cache.rs:34-54, deltanet.rs:444-450),
// SiLU(gate) (deltanet.rs:527-533), beta = sigmoid(W_beta x) and
// decay = exp(ssm_a * softplus(W_alpha x + dt_bias)) (deltanet.rs:469-480) for head j
__device__ __forceinline__ void prep_compute(const DnParams& p, int j, int tid, const PrepIn& in, PrepSlot& ps) {
    const DnItem it = dn_item(j, p.H);
    const int hg = p.h0 + it.h;
#pragma unroll
    for (int i = 0; i < 3; i++) {
        const int ch = i * p.D + hg * DK + tid;
        float* cs = p.conv + (size_t)it.b * p.conv_stride + (size_t)ch * p.K;
        float sum = 0.0f;
        if (p.K == 4) {
            const float4 s4 = make_float4(in.st[i].y, in.st[i].z, in.st[i].w, in.in[i]);
            *reinterpret_cast<float4*>(cs) = s4;
            sum = s4.x * in.w4[i].x;
            sum += s4.y * in.w4[i].y;
            sum += s4.z * in.w4[i].z;
            sum += s4.w * in.w4[i].w;
        } else {
            const float* cw = p.conv_w + (size_t)ch * p.K;
            for (int k = 0; k + 1 < p.K; k++) cs[k] = cs[k + 1];
            cs[p.K - 1] = in.in[i];
            for (int k = 0; k < p.K; k++) sum += cs[k] * cw[k];
        }
        ps.qkv[i][tid] = ref_silu(sum);
    }
    ps.g[tid] = in.g / (1.0f + expf(-in.g));
    if (tid == 0) {
        ps.beta = ref_sigmoid(in.br);
        ps.decay = expf(in.sa * ref_softplus(in.ar + in.dtb));
    }
}

__global__ void __launch_bounds__(kDnPersistThreads, 1) deltanet_persist_kernel(DnParams p, int n_items) {
    extern __shared__ uint8_t dn_smem_raw[];
    float* slots = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(dn_smem_raw) + 127) & ~(uintptr_t)127);
    __shared__ __align__(16) PrepSlot prep[kPrepSlots];
    __shared__ __align__(16) float red[8 * DK];
    __shared__ __align__(16) float delta_s[DK];
    __shared__ float ssp[4];
    __shared__ uint64_t full[kDnSlots], prep_full[kPrepSlots], prep_free[kPrepSlots];
    __shared__ int s_abort, s_prep_abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int H = p.H;
    const int G = gridDim.x;
    const int nmy = n_items > (int)blockIdx.x ? (n_items - (int)blockIdx.x + G - 1) / G : 0;

    if (tid == 0) {
        s_abort = 0;
        s_prep_abort = 0;
        for (int s = 0; s < kDnSlots; s++) mbar_init(&full[s], 1);
        for (int s = 0; s < kPrepSlots; s++) {
            mbar_init(&prep_full[s], kPrepThreads);
            mbar_init(&prep_free[s], kUpdThreads);
        }
        mbar_fence_init();
    }
    __syncthreads();
    auto state_of = [&](int j) {
        const DnItem it = dn_item(j, H);
        return p.S + (size_t)it.b * p.s_stride + (size_t)it.h * DK * DK;
    };
    // Launched with programmatic dependent launch behind the input projection GEMM, which lets
    // this grid start once the GEMM has set up. The GEMM itself started only after the kernel
    // before it (the RMSNorm, which waits for its own predecessor before it lets the next
    // kernel start) had waited, so every kernel before that RMSNorm has completed, among them
    // this layer's mixer of the previous step: the head states, conv states and weights can be
    // read now. Only the projection output needs the wait.

    if (tid >= kUpdThreads) {
        // ---------------- prep warps: per-head inputs, one head ahead of the update warps
        const int pt = tid - kUpdThreads;
        PrepIn cur, nxt;
        if (nmy > 0) prep_load_const(p, 0, pt, cur);
        asm volatile("griddepcontrol.wait;" ::: "memory");
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        if (nmy > 0) prep_load_proj(p, 0, pt, cur);
        for (int j = 0; j < nmy; j++) {
            const int s = j % kPrepSlots;
            if (j + 1 < nmy) {  // the next head's loads overlap this head's math
                prep_load_const(p, j + 1, pt, nxt);
                prep_load_proj(p, j + 1, pt, nxt);
            }
            if (j >= kPrepSlots && !mbar_wait(&prep_free[s], ((j / kPrepSlots) - 1) & 1, p.wt.wait_ns))
                s_prep_abort = 1;
            asm volatile("bar.sync %0, %1;" ::"n"(kPrepBar), "n"(kPrepThreads) : "memory");
            if (s_prep_abort) break;
            prep_compute(p, j, pt, cur, prep[s]);
            asm volatile("bar.sync %0, %1;" ::"n"(kPrepBar), "n"(kPrepThreads) : "memory");
            // per-head L2 norm of q (then * 1/sqrt(dk)) and k (deltanet.rs:459-467)
            const int pw = pt >> 5;
            if (pw < 2) {
                float* v = prep[s].qkv[pw];
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
                    if (pw == 0) t *= 1.0f / sqrtf((float)DK);
                    v[lane + 32 * i] = t;
                }
            }
            mbar_arrive(&prep_full[s]);
            cur = nxt;
        }
        return;
    }

    // ---------------- update warps
    const uint32_t WL = p.wt.wait_ns;  // the limit of every wait below
    auto load = [&](int j) {  // thread 0
        if (j == p.wt.withhold) return;  // test hook: this state copy is never issued
        const int s = j % kDnSlots;
        float* dst = slots + (size_t)s * DK * DK;
        const float* src = state_of(j);
        mbar_arrive_expect_tx(&full[s], kStateBytes);
#pragma unroll
        for (int c = 0; c < 4; c++)
            bulk_g2s(dst + c * (DK * DK / 4), src + c * (DK * DK / 4), kStateBytes / 4, &full[s]);
    };
    int issued = 0;  // thread 0: items whose state load has been issued
    if (tid == 0) {
        for (; issued < min(kDnSlots, nmy); issued++) load(issued);
        if (issued == nmy) prefetch_share_l2(p.pf, p.pf_bytes, blockIdx.x, G);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    const int r0 = warp * 16, c0 = lane * 4;  // this thread's 16 rows x 4 columns of a head state
    for (int j = 0; j < nmy; j++) {
        const DnItem it = dn_item(j, H);
        const int ps = j % kPrepSlots;
        const float* Ss = slots + (size_t)(j % kDnSlots) * DK * DK;
        // every thread observes the copy's and the prep slot's completion itself, so the bytes
        // it reads are the ones the bulk copy and the prep warps wrote
        if (!mbar_wait(&full[j % kDnSlots], (j / kDnSlots) & 1, WL)) s_abort = 1 + j;
        if (!mbar_wait(&prep_full[ps], (j / kPrepSlots) & 1, WL)) s_abort = 1 + j;
        asm volatile("bar.sync %0, %1;" ::"n"(kUpdBar), "n"(kUpdThreads) : "memory");
        if (s_abort) break;
        const PrepSlot& in = prep[ps];

        // gated delta rule (deltanet.rs:485-512):
        //   S *= decay; sk = S^T k; delta = beta (v - sk); S += k delta^T; o = S^T q
        const float beta = in.beta, decay = in.decay;
        const float* qv = in.qkv[0];
        const float* kv = in.qkv[1];
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
        asm volatile("bar.sync %0, %1;" ::"n"(kUpdBar), "n"(kUpdThreads) : "memory");  // the slot is in registers
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
            delta_s[tid] = beta * (in.qkv[2][tid] - a);
        }
        asm volatile("bar.sync %0, %1;" ::"n"(kUpdBar), "n"(kUpdThreads) : "memory");
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
        asm volatile("bar.sync %0, %1;" ::"n"(kUpdBar), "n"(kUpdThreads) : "memory");
        // gated RMSNorm with ssm_norm, times SiLU(gate) (deltanet.rs:514-533)
        float ov = 0.0f;
        if (tid < DK) {
#pragma unroll
            for (int w = 0; w < 8; w++) ov += red[w * DK + tid];
            const float ss = warp_sum(ov * ov);
            if (lane == 0) ssp[warp] = ss;
        }
        asm volatile("bar.sync %0, %1;" ::"n"(kUpdBar), "n"(kUpdThreads) : "memory");
        if (tid < DK) {
            const float rms = 1.0f / sqrtf((ssp[0] + ssp[1] + ssp[2] + ssp[3]) / (float)DK + p.eps);
            float nv = ov * rms * p.ssm_norm[tid];
            nv *= in.g[tid];
            act_store(p.out, it.b, (p.h0 + it.h) * DK + tid, nv);  // the head's columns in the model
            if (p.o_out) p.o_out[(size_t)it.b * p.D + (p.h0 + it.h) * DK + tid] = nv;
        }
        mbar_arrive(&prep_free[ps]);  // this thread's reads of the prep slot are done
    }
    if (tid == 0 && s_abort) {
        // a copy or a prep slot did not arrive in time: report it, then give the copies still in
        // flight into the state slots a bounded time to land before shared memory is released
        if (p.err) atomicOr(p.err, 1024u);
        for (int k = s_abort - 1; k < issued; k++)
            if (k != p.wt.withhold) mbar_wait(&full[k % kDnSlots], (k / kDnSlots) & 1, WL);
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
    DnParams q = p;
    q.wt = take_wait_test(kWaitTestDeltaNet, st);
    launch_pdl(deltanet_persist_kernel, dim3(std::min(n_items, nsm)), dim3(kDnPersistThreads), smem, st, q, n_items);
}

void launch_gated_delta(float* S, const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* beta,
                        const float* decay, int B, int H, float* o, cudaStream_t st) {
    dim3 grid(H, B);
    gated_delta_kernel<<<grid, kDnThreads, 0, st>>>(S, q, k, v, beta, decay, H, o);
}

}  // namespace ab2
