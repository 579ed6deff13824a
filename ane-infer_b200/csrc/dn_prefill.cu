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
// sum of squares over the 128 columns is exchanged the same way. The matrix products run on
// the tensor cores in 3xTF32 (about f32 accuracy, below); the rest is f32 on the CUDA cores.
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
constexpr int kLd = DK + 4;               // padded row stride of q and k (conflict-free float4 rows)
constexpr int kLv = kCols + 8;            // padded row stride of V / Delta and O (conflict-free fragments)
constexpr int kLs = kCols + 8;            // padded row stride of the state slice
constexpr int kLp = kT + 4;               // padded row stride of A and P
constexpr int kSb = 16;                   // rows per block of the forward substitution
constexpr int kConvCh = 2 * DK + kCols;   // conv channels of a CTA: q, k and its v columns
constexpr int kConvTok = 16;              // tokens per conv work item

struct PfSmem {
    static constexpr int K = 0;                      // [kT][kLd] normed keys
    static constexpr int Q = K + kT * kLd;           // [kT][kLd] normed, scaled queries
    static constexpr int S = Q + kT * kLd;           // [DK][kLs] this CTA's columns of the state
    static constexpr int V = S + DK * kLs;           // [kT][kLv] values; later R, then Delta
    static constexpr int O = V + kT * kLv;           // [kT][kLv] outputs
    static constexpr int A = O + kT * kLv;           // [kT][kLp]
    static constexpr int P = A + kT * kLp;           // [kT][kLp]
    static constexpr int G = P + kT * kLp;           // [kT] cumulative log-decay
    static constexpr int BETA = G + kT;              // [kT]
    static constexpr int EG = BETA + kT;             // [kT] e^{g_t}
    static constexpr int W = EG + kT;                // [kT] e^{g_{T-1} - g_t}
    static constexpr int SS = W + kT;                // [kPfCluster][kT] partial sums of squares of O
    static constexpr int floats = SS + kPfCluster * kT;
    static constexpr int bytes = floats * 4;
};
static_assert(PfSmem::bytes <= 227 * 1024, "prefill shared memory");
// the warp tilings below: 16 warps; A/P rows are one m16 tile per CTA; 4 x 4 tiles of 16
// tokens x 8 columns; 8 x 4 tiles of 16 state rows x 8 columns
static_assert(kPfThreads == 512 && kCols == 32 && kRows == 16 && kT == 64, "prefill warp tiling");

// The chunk's matrix products run on the tensor cores at about f32 accuracy (3xTF32): each
// f32 operand is split into a tf32 high part and a tf32 remainder, and the three products
// that matter (lo*hi, hi*lo, hi*hi) are accumulated in f32 by mma.sync m16n8k8. Fragments
// (g = lane / 4, q = lane % 4): A[16 x 8] a0 (g, q), a1 (g + 8, q), a2 (g, q + 4),
// a3 (g + 8, q + 4); B[8 x 8] b0 (q, g), b1 (q + 4, g); C[16 x 8] c0 (g, 2q), c1 (g, 2q + 1),
// c2 (g + 8, 2q), c3 (g + 8, 2q + 1).
__device__ __forceinline__ uint32_t to_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
    hi = to_tf32(x);
    lo = to_tf32(x - __uint_as_float(hi));
}
__device__ __forceinline__ void mma_tf32(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
struct SplitB {
    uint32_t h0, l0, h1, l1;
};
__device__ __forceinline__ SplitB split_b(float b0, float b1) {
    SplitB r;
    split_tf32(b0, r.h0, r.l0);
    split_tf32(b1, r.h1, r.l1);
    return r;
}
// c += A B (A as four f32 fragment values, B pre-split)
__device__ __forceinline__ void mma3(float c[4], const float a[4], const SplitB& b) {
    uint32_t ah[4], al[4];
#pragma unroll
    for (int i = 0; i < 4; i++) split_tf32(a[i], ah[i], al[i]);
    mma_tf32(c, al, b.h0, b.h1);
    mma_tf32(c, ah, b.l0, b.l1);
    mma_tf32(c, ah, b.h0, b.h1);
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
        const uint32_t dsm = (uint32_t)__cvta_generic_to_shared(reinterpret_cast<float4*>(S + (e >> 3) * kLs) + (e & 7));
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
    // the inputs of item e: conv weights, the window before its tokens, its tokens' inputs
    struct ConvIn {
        float4 cw, cs;
        float x[kConvTok];
    };
    auto conv_load = [&](int e, ConvIn& in) {
        const int cc = e % kConvCh, t0 = (e / kConvCh) * kConvTok, ch = conv_channel(cc);
        in.cw = *reinterpret_cast<const float4*>(p.conv_w + (size_t)ch * 4);
        if (t0 == 0) {
            in.cs = *reinterpret_cast<const float4*>(p.conv + (size_t)ch * 4);
        } else {
            const float* pr = p.proj + (size_t)(t0 - 3) * p.ldp + ch;
            in.cs = make_float4(0.0f, pr[0], pr[p.ldp], pr[2 * (size_t)p.ldp]);
        }
#pragma unroll
        for (int u = 0; u < kConvTok; u++) in.x[u] = t0 + u < T ? p.proj[(size_t)(t0 + u) * p.ldp + ch] : 0.0f;
    };
    // software-pipelined: the next item's loads are in flight while this item is computed
    ConvIn cur, nxt;
    if (tid < nitems) conv_load(tid, cur);
#pragma unroll 1
    for (int e = tid; e < nitems; e += kPfThreads) {
        if (e + kPfThreads < nitems) conv_load(e + kPfThreads, nxt);
        const int cc = e % kConvCh, t0 = (e / kConvCh) * kConvTok, ch = conv_channel(cc);
        float4 cs = cur.cs;
        const float4 cw = cur.cw;
        float* dst = cc < DK ? Qb + cc : cc < 2 * DK ? Kb + (cc - DK) : Vb + (cc - 2 * DK);
        const int ld = cc < 2 * DK ? kLd : kLv;
#pragma unroll
        for (int u = 0; u < kConvTok; u++) {
            if (t0 + u >= T) break;
            cs = make_float4(cs.y, cs.z, cs.w, cur.x[u]);
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
        cur = nxt;
    }
    if (tid < T) {
        // beta = sigmoid(W_beta x) and log d = ssm_a * softplus(W_alpha x + dt_bias) (deltanet.rs:469-480)
        const float* pr = p.proj + (size_t)tid * p.ldp;
        beta[tid] = ref_sigmoid(pr[4 * p.D + hg]);
        g[tid] = sa * ref_softplus(pr[4 * p.D + H_all + hg] + dtb);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    // rows past the chunk's last token enter the products as zeros (a shorter last chunk)
    for (int e = tid; e < (kT - T) * kLd; e += kPfThreads) {
        Kb[T * kLd + e] = 0.0f;
        Qb[T * kLd + e] = 0.0f;
    }
    for (int e = tid; e < (kT - T) * kLv; e += kPfThreads) Vb[T * kLv + e] = 0.0f;
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
    if (tid < kT) {
        eg[tid] = tid < T ? expf(g[tid]) : 0.0f;
        w[tid] = tid < T ? expf(g[T - 1] - g[tid]) : 0.0f;
    }
    // every CTA of the cluster has started (its shared memory may now be written) and has
    // read the conv windows before they are replaced
    cluster.sync();
    // the windows after the chunk: the q and k channels' by one CTA of the cluster, the v
    // channels' by the CTA that owns them
    if (fin_ch >= 0) *reinterpret_cast<float4*>(p.conv + (size_t)fin_ch * 4) = fin_cs;

    const int gq = lane >> 2, tq = lane & 3;  // fragment row group and column pair
    // rows [kRows c, kRows (c+1)) of A (warps 0-7, from k) and P (warps 8-15, from q): warp w
    // computes columns s of tile w % 8, and stores its entries into every CTA of the cluster
    {
        const bool is_a = warp < 8;
        const float* src = (is_a ? Kb : Qb) + c * kRows * kLd;
        const float* kr = Kb + ((warp & 7) * 8 + gq) * kLd;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
        for (int kk = 0; kk < DK; kk += 8) {
            const float a[4] = {src[gq * kLd + kk + tq], src[(gq + 8) * kLd + kk + tq], src[gq * kLd + kk + tq + 4],
                                src[(gq + 8) * kLd + kk + tq + 4]};
            mma3(acc, a, split_b(kr[kk + tq], kr[kk + tq + 4]));
        }
        float* dstm = is_a ? A : P;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int t = c * kRows + gq + 8 * (i >> 1), s = (warp & 7) * 8 + 2 * tq + (i & 1);
            const bool in = t < T && s <= t;  // the causal part of the chunk
            const float dec = in ? expf(g[t] - g[s]) : 0.0f;
            const float v = is_a ? (in && s < t ? beta[t] * dec * acc[i] : 0.0f) : (in ? dec * acc[i] : 0.0f);
#pragma unroll
            for (int r = 0; r < kPfCluster; r++) cluster.map_shared_rank(dstm, r)[t * kLp + s] = v;
        }
    }

    // R = beta (V - e^g K S0) into V and e^g Q S0 into O for this CTA's columns: warp w
    // computes tokens of tile w / 4 and columns of tile w % 4
    {
        const int r0 = (warp >> 2) * 16 + gq, n0 = (warp & 3) * 8;
        float ck[4] = {0.f, 0.f, 0.f, 0.f}, cq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
        for (int kk = 0; kk < DK; kk += 8) {
            const SplitB b = split_b(S[(kk + tq) * kLs + n0 + gq], S[(kk + tq + 4) * kLs + n0 + gq]);
            const float ak[4] = {Kb[r0 * kLd + kk + tq], Kb[(r0 + 8) * kLd + kk + tq], Kb[r0 * kLd + kk + tq + 4],
                                 Kb[(r0 + 8) * kLd + kk + tq + 4]};
            const float aq[4] = {Qb[r0 * kLd + kk + tq], Qb[(r0 + 8) * kLd + kk + tq], Qb[r0 * kLd + kk + tq + 4],
                                 Qb[(r0 + 8) * kLd + kk + tq + 4]};
            mma3(ck, ak, b);
            mma3(cq, aq, b);
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int t = r0 + 8 * (i >> 1), jc = n0 + 2 * tq + (i & 1);
            if (t < T) {
                Vb[t * kLv + jc] = beta[t] * (Vb[t * kLv + jc] - eg[t] * ck[i]);
                Ob[t * kLv + jc] = eg[t] * cq[i];
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
                    const float* at = A + (jb + r) * kLp + jb;
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
            const float* at = A + t * kLp + jb;
            float a = 0.0f;
            for (int s2 = 0; s2 < nb; s2++) a += at[s2] * Vb[(jb + s2) * kLv + col];
            Vb[t * kLv + col] -= a;
        }
        __syncthreads();
    }
    // O += P Delta (P is causal: the k range stops at the tile's last token): warp w, token
    // tile w / 4, column tile w % 4
    {
        const int r0 = (warp >> 2) * 16 + gq, n0 = (warp & 3) * 8;
        float co[4];
#pragma unroll
        for (int i = 0; i < 4; i++) co[i] = Ob[(r0 + 8 * (i >> 1)) * kLv + n0 + 2 * tq + (i & 1)];
        const int kend = min(T, (warp >> 2) * 16 + 16);
        for (int kk = 0; kk < kend; kk += 8) {
            const float a[4] = {P[r0 * kLp + kk + tq], P[(r0 + 8) * kLp + kk + tq], P[r0 * kLp + kk + tq + 4],
                                P[(r0 + 8) * kLp + kk + tq + 4]};
            mma3(co, a, split_b(Vb[(kk + tq) * kLv + n0 + gq], Vb[(kk + tq + 4) * kLv + n0 + gq]));
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int t = r0 + 8 * (i >> 1);
            if (t < T) Ob[t * kLv + n0 + 2 * tq + (i & 1)] = co[i];
        }
    }
    // S_T = e^{g_{T-1}} S0 + K^T diag(w) Delta for this CTA's columns, to HBM: tiles of 16
    // state rows x 8 columns, two per warp
    {
        const float eT = eg[T - 1];
#pragma unroll 1
        for (int tile = warp; tile < (DK / 16) * (kCols / 8); tile += kPfThreads / 32) {
            const int i0 = (tile >> 2) * 16 + gq, n0 = (tile & 3) * 8;
            float cs4[4];
#pragma unroll
            for (int i = 0; i < 4; i++) cs4[i] = eT * S[(i0 + 8 * (i >> 1)) * kLs + n0 + 2 * tq + (i & 1)];
            for (int kk = 0; kk < T; kk += 8) {
                const float a[4] = {Kb[(kk + tq) * kLd + i0], Kb[(kk + tq) * kLd + i0 + 8], Kb[(kk + tq + 4) * kLd + i0],
                                    Kb[(kk + tq + 4) * kLd + i0 + 8]};
                mma3(cs4, a,
                     split_b(w[kk + tq] * Vb[(kk + tq) * kLv + n0 + gq], w[kk + tq + 4] * Vb[(kk + tq + 4) * kLv + n0 + gq]));
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
                Sg[(size_t)(i0 + 8 * (i >> 1)) * DK + c0 + n0 + 2 * tq + (i & 1)] = cs4[i];
        }
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
        act_store(p.out, p.row0 + t, hg * DK + hc, nv);
        if (p.o_out) p.o_out[(size_t)(p.row0 + t) * p.D + hg * DK + hc] = nv;
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
