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
// Each head runs on a thread-block cluster of kPfCluster CTAs. Every CTA of the cluster
// holds the chunk's normed q and k, computes kT / kPfCluster rows of A and P and stores them
// into every CTA's shared memory (distributed shared memory), and owns 128 / kPfCluster of
// the head's value columns: their slice of the state, of V, Delta and O. The gated RMSNorm's
// sum of squares over the 128 columns is exchanged the same way. The products run on the
// CUDA cores in f32, like the reference's.
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"

namespace ab2 {
namespace {

namespace cg = cooperative_groups;

constexpr int DK = 128;                   // key_dim = value_dim
constexpr int kT = kPrefillChunk;         // tokens per launch
constexpr int kPfThreads = 512;
constexpr int kPfCluster = 4;             // CTAs per head (16 clusters of 8 do not fit at once)
constexpr int kCols = DK / kPfCluster;    // value columns per CTA (32)
constexpr int kRows = kT / kPfCluster;    // rows of A and P each CTA computes (16)
constexpr int kTg = kPfThreads / kCols;   // thread groups of one column (16)
constexpr int kLd = DK + 4;               // padded row stride of q and k (conflict-free float4 rows)
constexpr int kLv = kCols + 1;            // padded row stride of the per-CTA column buffers
constexpr int kSb = 16;                   // rows per block of the forward substitution
constexpr int kConvCh = 2 * DK + kCols;   // conv channels of a CTA: q, k and its v columns
constexpr int kConvTok = 16;              // tokens per conv work item

struct PfSmem {
    static constexpr int K = 0;                      // [kT][kLd] normed keys
    static constexpr int Q = K + kT * kLd;           // [kT][kLd] normed, scaled queries
    static constexpr int S = Q + kT * kLd;           // [DK][kCols] this CTA's columns of the state
    static constexpr int V = S + DK * kCols;         // [kT][kLv] values; later R, then Delta
    static constexpr int O = V + kT * kLv;           // [kT][kLv] outputs
    static constexpr int A = O + kT * kLv;           // [kT][kT]
    static constexpr int P = A + kT * kT;            // [kT][kT]
    static constexpr int G = P + kT * kT;            // [kT] cumulative log-decay
    static constexpr int BETA = G + kT;              // [kT]
    static constexpr int EG = BETA + kT;             // [kT] e^{g_t}
    static constexpr int W = EG + kT;                // [kT] e^{g_{T-1} - g_t}
    static constexpr int SS = W + kT;                // [kPfCluster][kT] partial sums of squares of O
    static constexpr int floats = SS + kPfCluster * kT;
    static constexpr int bytes = floats * 4;
};
static_assert(PfSmem::bytes <= 227 * 1024, "prefill shared memory");
static_assert(kCols == 32 && kTg == 16 && kRows * kT == 2 * kPfThreads, "prefill thread mapping");

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
    float* Kb = sm + PfSmem::K;
    float* Qb = sm + PfSmem::Q;
    float* S = sm + PfSmem::S;
    float* Vb = sm + PfSmem::V;
    float* Ob = sm + PfSmem::O;
    float* A = sm + PfSmem::A;
    float* P = sm + PfSmem::P;
    float* g = sm + PfSmem::G;
    float* beta = sm + PfSmem::BETA;
    float* eg = sm + PfSmem::EG;
    float* w = sm + PfSmem::W;
    float* ssp = sm + PfSmem::SS;
    cg::cluster_group cluster = cg::this_cluster();
    const int c = (int)cluster.block_rank();                  // this CTA's column block
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int h = blockIdx.x / kPfCluster, hg = p.h0 + h, H_all = p.H_all ? p.H_all : p.H;
    const int c0 = c * kCols;                                  // first value column of this CTA
    float* Sg = p.S + (size_t)h * DK * DK;

    // conv channels of this CTA: q and k (every CTA: all 256), v (its kCols columns); channel
    // cc of kConvCh maps to the model's channel conv_channel(cc)
    auto conv_channel = [&](int cc) {
        return cc < 2 * DK ? (cc / DK) * p.D + hg * DK + cc % DK : 2 * p.D + hg * DK + c0 + (cc - 2 * DK);
    };
    const float sa = p.ssm_a[hg], dtb = p.dt_bias[hg];
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    // this CTA's columns of the head's state: [DK rows][kCols], 8 float4 per row, copied
    // asynchronously (cp.async: the thread goes on to the conv while they travel; waited
    // for before the first barrier)
    for (int e = tid; e < DK * kCols / 4; e += kPfThreads) {
        const uint32_t dsm = (uint32_t)__cvta_generic_to_shared(reinterpret_cast<float4*>(S) + e);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dsm),
                     "l"(reinterpret_cast<const float4*>(Sg + (size_t)(e >> 3) * DK + c0) + (e & 7))
                     : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    // the gate values of this thread's outputs (token e / kCols, column e % kCols), loaded now
    float gate[kT * kCols / kPfThreads];
#pragma unroll
    for (int u = 0; u < kT * kCols / kPfThreads; u++) {
        const int e = tid + u * kPfThreads, t = e / kCols;
        gate[u] = t < T ? p.proj[(size_t)t * p.ldp + 3 * p.D + hg * DK + c0 + e % kCols] : 0.0f;
    }
    // conv_shift_and_append + conv_apply + SiLU per token (deltanet_cache.rs:34-54,
    // deltanet.rs:444-450). A token's window is the channel's last 4 inputs, so the work splits
    // into items of (channel, 16 tokens) with no order between them: an item loads the 3 inputs
    // before its tokens (from the conv state for the first block) with its own 16 in one round.
    // The item holding the chunk's last token keeps the final window, the new conv state.
    const int nblk = (T + kConvTok - 1) / kConvTok, nitems = kConvCh * nblk;
    float4 fin_cs = make_float4(0.f, 0.f, 0.f, 0.f);
    int fin_ch = -1;
#pragma unroll 1
    for (int e = tid; e < nitems; e += kPfThreads) {
        const int cc = e % kConvCh, t0 = (e / kConvCh) * kConvTok, ch = conv_channel(cc);
        const float4 cw = *reinterpret_cast<const float4*>(p.conv_w + (size_t)ch * 4);
        float4 cs;
        if (t0 == 0) {
            cs = *reinterpret_cast<const float4*>(p.conv + (size_t)ch * 4);
        } else {
            const float* pr = p.proj + (size_t)(t0 - 3) * p.ldp + ch;
            cs = make_float4(0.0f, pr[0], pr[p.ldp], pr[2 * (size_t)p.ldp]);
        }
        float xin[kConvTok];
#pragma unroll
        for (int u = 0; u < kConvTok; u++) xin[u] = t0 + u < T ? p.proj[(size_t)(t0 + u) * p.ldp + ch] : 0.0f;
        float* dst = cc < DK ? Qb + cc : cc < 2 * DK ? Kb + (cc - DK) : Vb + (cc - 2 * DK);
        const int ld = cc < 2 * DK ? kLd : kLv;
#pragma unroll
        for (int u = 0; u < kConvTok; u++) {
            if (t0 + u >= T) break;
            cs = make_float4(cs.y, cs.z, cs.w, xin[u]);
            float sum = cs.x * cw.x;
            sum += cs.y * cw.y;
            sum += cs.z * cw.z;
            sum += cs.w * cw.w;
            dst[(t0 + u) * ld] = ref_silu(sum);
        }
        if (t0 + kConvTok >= T) {
            fin_cs = cs;
            fin_ch = ch;
            if (cc < 2 * DK && c != 0) fin_ch = -1;  // q and k channels: one CTA of the cluster writes
        }
    }
    if (tid < T) {
        // beta = sigmoid(W_beta x) and log d = ssm_a * softplus(W_alpha x + dt_bias) (deltanet.rs:469-480)
        const float* pr = p.proj + (size_t)tid * p.ldp;
        beta[tid] = ref_sigmoid(pr[4 * p.D + hg]);
        g[tid] = sa * ref_softplus(pr[4 * p.D + H_all + hg] + dtb);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        // inclusive prefix sum of the log-decays: lane l holds tokens 2l, 2l + 1
        const float a0 = 2 * lane < T ? g[2 * lane] : 0.0f;
        const float a1 = 2 * lane + 1 < T ? g[2 * lane + 1] : 0.0f;
        float pre = a0 + a1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float n = __shfl_up_sync(0xffffffffu, pre, o);
            if (lane >= o) pre += n;
        }
        const float base = pre - (a0 + a1);
        if (2 * lane < T) g[2 * lane] = base + a0;
        if (2 * lane + 1 < T) g[2 * lane + 1] = pre;
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
            float x = xs[i] * inv;
            if (r < T) x *= 1.0f / sqrtf((float)DK);
            v[lane + 32 * i] = x;
        }
    }
    __syncthreads();
    if (tid < T) {
        eg[tid] = expf(g[tid]);
        w[tid] = expf(g[T - 1] - g[tid]);
    }
    // every CTA of the cluster has started (its shared memory may now be written) and has
    // read the conv windows before they are replaced
    cluster.sync();
    // the windows after the chunk: the q and k channels' by one CTA of the cluster, the v
    // channels' by the CTA that owns them
    if (fin_ch >= 0) *reinterpret_cast<float4*>(p.conv + (size_t)fin_ch * 4) = fin_cs;

    // rows [kRows c, kRows (c+1)) of A and P, one entry of each per thread, stored into every
    // CTA of the cluster
#pragma unroll 1
    for (int u = 0; u < 2; u++) {
        const int e = tid + u * kPfThreads, t = c * kRows + (e >> 6), s = e & (kT - 1);
        float kk = 0.0f, qk = 0.0f;
        if (t < T && s <= t) {
            const float* kt = Kb + t * kLd;
            const float* qt = Qb + t * kLd;
            const float* ks = Kb + s * kLd;
#pragma unroll 8
            for (int i = 0; i < DK; i += 4) {
                const float4 k4 = *reinterpret_cast<const float4*>(ks + i);
                kk = dot4(*reinterpret_cast<const float4*>(kt + i), k4, kk);
                qk = dot4(*reinterpret_cast<const float4*>(qt + i), k4, qk);
            }
        }
        const bool in = t < T && s <= t;  // rows and columns past T were never written
        const float dec = in ? expf(g[t] - g[s]) : 0.0f;
        const float a_ts = in && s < t ? beta[t] * dec * kk : 0.0f;
        const float p_ts = in ? dec * qk : 0.0f;
#pragma unroll
        for (int r = 0; r < kPfCluster; r++) {
            cluster.map_shared_rank(A, r)[t * kT + s] = a_ts;
            cluster.map_shared_rank(P, r)[t * kT + s] = p_ts;
        }
    }

    // R = beta (V - e^g K S0) and e^g Q S0 for this CTA's columns; thread: column j,
    // tokens tg + kTg u
    const int j = tid & (kCols - 1), tg = tid / kCols;
    {
        float ks0[4] = {0.f, 0.f, 0.f, 0.f}, qs0[4] = {0.f, 0.f, 0.f, 0.f};
        for (int i = 0; i < DK; i += 4) {
            const float4 s4 = make_float4(S[i * kCols + j], S[(i + 1) * kCols + j], S[(i + 2) * kCols + j],
                                          S[(i + 3) * kCols + j]);
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int t = tg + kTg * u;
                ks0[u] = dot4(*reinterpret_cast<const float4*>(Kb + t * kLd + i), s4, ks0[u]);
                qs0[u] = dot4(*reinterpret_cast<const float4*>(Qb + t * kLd + i), s4, qs0[u]);
            }
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int t = tg + kTg * u;
            if (t < T) {
                Vb[t * kLv + j] = beta[t] * (Vb[t * kLv + j] - eg[t] * ks0[u]);
                Ob[t * kLv + j] = eg[t] * qs0[u];
            }
        }
    }
    cluster.sync();  // all of A and P has arrived; R is complete
    // (I + A) Delta = R by forward substitution in blocks of kSb rows: warp 0 solves a block
    // (lane = column, the block's values in registers), then every thread subtracts the
    // block's contribution from the rows below it
    for (int jb = 0; jb < T; jb += kSb) {
        const int nb = min(kSb, T - jb);
        if (warp == 0) {
            float dl[kSb];
#pragma unroll
            for (int r = 0; r < kSb; r++) {
                dl[r] = 0.0f;
                if (r < nb) {
                    const float* at = A + (jb + r) * kT + jb;
                    float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
                    for (int s2 = 0; s2 < r; s2++) {
                        if (s2 & 1) a1 += at[s2] * dl[s2];
                        else a0 += at[s2] * dl[s2];
                    }
                    dl[r] = Vb[(jb + r) * kLv + lane] - (a0 + a1);
                }
            }
#pragma unroll
            for (int r = 0; r < kSb; r++)
                if (r < nb) Vb[(jb + r) * kLv + lane] = dl[r];
        }
        __syncthreads();
        for (int e = tid; e < (T - jb - nb) * kCols; e += kPfThreads) {
            const int t = jb + nb + e / kCols, col = e % kCols;
            const float* at = A + t * kT + jb;
            float a = 0.0f;
            for (int s2 = 0; s2 < nb; s2++) a += at[s2] * Vb[(jb + s2) * kLv + col];
            Vb[t * kLv + col] -= a;
        }
        __syncthreads();
    }
    // O += P Delta (column j, tokens tg + kTg u)
#pragma unroll
    for (int u = 0; u < 4; u++) {
        const int t = tg + kTg * u;
        if (t < T) {
            const float* pt = P + t * kT;
            float o0 = Ob[t * kLv + j], o1 = 0.0f;
            int s = 0;
            for (; s + 2 <= t + 1; s += 2) {
                o0 += pt[s] * Vb[s * kLv + j];
                o1 += pt[s + 1] * Vb[(s + 1) * kLv + j];
            }
            if (s <= t) o0 += pt[s] * Vb[s * kLv + j];
            Ob[t * kLv + j] = o0 + o1;
        }
    }
    // S_T = e^{g_{T-1}} S0 + K^T diag(w) Delta for this CTA's columns (column j, rows
    // tg * 8 .. tg * 8 + 7), to HBM
    {
        const float eT = eg[T - 1];
        float acc[8];
#pragma unroll
        for (int r = 0; r < 8; r++) acc[r] = eT * S[(tg * 8 + r) * kCols + j];
        for (int t = 0; t < T; t++) {
            const float dw = w[t] * Vb[t * kLv + j];
            const float4 ka = *reinterpret_cast<const float4*>(Kb + t * kLd + tg * 8);
            const float4 kb = *reinterpret_cast<const float4*>(Kb + t * kLd + tg * 8 + 4);
            acc[0] += ka.x * dw;
            acc[1] += ka.y * dw;
            acc[2] += ka.z * dw;
            acc[3] += ka.w * dw;
            acc[4] += kb.x * dw;
            acc[5] += kb.y * dw;
            acc[6] += kb.z * dw;
            acc[7] += kb.w * dw;
        }
#pragma unroll
        for (int r = 0; r < 8; r++) Sg[(size_t)(tg * 8 + r) * DK + c0 + j] = acc[r];
    }
    __syncthreads();
    // gated RMSNorm with ssm_norm, times SiLU(gate) (deltanet.rs:514-533): each CTA's sum of
    // squares over its 32 columns (a warp sum, as the decode mixer's per-warp partials) goes
    // to every CTA, which adds the four in rank order, as the decode mixer does
    for (int t = warp; t < T; t += kPfThreads / 32) {
        const float o = Ob[t * kLv + lane];
        const float ss = warp_sum(o * o);
        if (lane < kPfCluster) cluster.map_shared_rank(ssp, lane)[c * kT + t] = ss;
    }
    cluster.sync();
#pragma unroll
    for (int u = 0; u < kT * kCols / kPfThreads; u++) {
        const int e = tid + u * kPfThreads, t = e / kCols, col = e % kCols;
        if (t >= T) break;
        float tot = 0.0f;
#pragma unroll
        for (int r = 0; r < kPfCluster; r++) tot += ssp[r * kT + t];
        const float rms = 1.0f / sqrtf(tot / (float)DK + p.eps);
        const int hc = c0 + col;  // the column in the head
        const float gt = gate[u];
        float nv = Ob[t * kLv + col] * rms * p.ssm_norm[hc];
        nv *= gt / (1.0f + expf(-gt));
        act_store(p.out, t, hg * DK + hc, nv);
        if (p.o_out) p.o_out[(size_t)t * p.D + hg * DK + hc] = nv;
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
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.H * kPfCluster);
    cfg.blockDim = dim3(kPfThreads);
    cfg.dynamicSmemBytes = PfSmem::bytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kPfCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, dn_prefill_kernel, p, tokens) == cudaSuccess ? 0 : -2;
}

}  // namespace ab2
