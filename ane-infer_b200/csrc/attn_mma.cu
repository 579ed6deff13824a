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
//   * attn_prep_kernel, launched before it, norms and rotates the queries into a prepared
//     buffer and appends the new (normed, rotated) key and value to the cache; the attention
//     kernel's producer waits for it (griddepcontrol.wait) before its first copy;
//   * the kernel is persistent, and the producer streams the tiles of all of a CTA's work
//     items through one ring without draining between items. The items are either splits of
//     a fixed chunk dealt round-robin (CTA c takes items c, c + grid, ...) or, when the
//     launcher's cost model prefers it, the balanced partition: every (sequence, kv head)
//     pair's tiles laid end to end and an equal run of them per CTA, computed on the device
//     from the positions. Split partials are merged in split order by attn_merge_kernel.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>

#include "attn_tiles.cuh"
#include "common.cuh"
#include "kernels.h"
#include "umma.cuh"

namespace ab2 {

constexpr int kAttnStages = 3;
constexpr int kCompWarps = 4;
constexpr int kAttnMmaThreads = (kCompWarps + 1) * 32;  // + one TMA producer warp
constexpr int kPStride = kT + 8;  // bf16 elements per P row (padding avoids ldmatrix bank conflicts)

template <int HD>
struct AttnSmem {
    static constexpr int kNDB = HD / 64;                   // 64-dim TMA boxes per row
    static constexpr int kTileBytes = kT * HD * 2;         // one K (or V) tile
    static constexpr int k_off(int s) { return s * kTileBytes; }
    static constexpr int v_off(int s) { return (kAttnStages + s) * kTileBytes; }
    static constexpr int s_off() { return 2 * kAttnStages * kTileBytes; }     // scores [4][kT] f32
    static constexpr int p_off() { return s_off() + kGQ * kT * 4; }           // P [16][kPStride] bf16
    static constexpr int q_off(int j) { return p_off() + 16 * kPStride * 2 + j * kGQ * HD * 4; }  // q [2][4][HD]
    static constexpr int o_off() { return q_off(2); }                         // O of an item [4][HD] f32
    static constexpr int misc_off() { return o_off() + kGQ * HD * 4; }        // corr[4], m[4], l[4]
    static constexpr int bar_off() { return misc_off() + 16 * 4; }            // full[S], empty[S], q_full[2], q_free[2]
    static constexpr int bytes() { return bar_off() + (2 * kAttnStages + 4) * 8; }
};

// Work item `item` = (split, sequence, kv head): item = split * pairs + (b * Hkv + kvh).
struct AttnItem {
    int b, kvh, split, t0, t1, ntiles, nsplit_b;
    bool has_new;  // the split holding the new position (its last tile)
};
__device__ __forceinline__ bool attn_item(const AttnParams& p, int item, int pairs, AttnItem& it) {
    const int pair = item % pairs;
    it.split = item / pairs;
    it.b = pair / p.Hkv;
    it.kvh = pair % p.Hkv;
    const int pos = p.pos[it.b], L = pos + 1;
    if (!attn_pos_ok(p, pos)) return false;  // skipped; the prep kernel reports it
    it.t0 = it.split * p.chunk;
    if (it.t0 >= L) return false;
    it.t1 = min(L, it.t0 + p.chunk);
    it.ntiles = (it.t1 - it.t0 + kT - 1) / kT;
    it.has_new = pos < it.t0 + p.chunk;
    it.nsplit_b = (L + p.chunk - 1) / p.chunk;
    return true;
}

// ---- balanced partition (p.sk_grid > 0). Pair q = b * Hkv + kvh holds n_b = ceil((pos[b] + 1)
// / kT) tiles (none for a skipped sequence); the pairs' tiles are laid end to end (pair q starts
// at tile P(q)), and CTA c takes tiles [c * per, (c + 1) * per). Split s of a pair is its piece
// in the s-th CTA that holds part of it, so split order is token order, as the merge needs.
__device__ __forceinline__ int sk_tiles(const AttnParams& p, int b) {
    const int pos = p.pos[b];
    return attn_pos_ok(p, pos) ? pos / kT + 1 : 0;
}
// tiles per CTA: an equal share, at least kSkMinTiles, and enough that no pair of nmax tiles
// spans more than kMaxSplits CTAs (a run of n tiles meets at most ceil(n / per) + 1 of them)
constexpr int kSkMinTiles = 4;
__host__ __device__ inline int sk_per(int64_t total, int nmax, int grid) {
    int64_t per = (total + grid - 1) / grid;
    const int64_t by_splits = (nmax + kMaxSplits - 2) / (kMaxSplits - 1);
    if (per < by_splits) per = by_splits;
    return (int)(per < kSkMinTiles ? kSkMinTiles : per);
}
// warp-wide: total tiles, the longest pair, and the first tile of sequence `bq`'s pairs
// (every lane gets all three)
__device__ __forceinline__ void sk_scan(const AttnParams& p, int B, int bq, int lane, int64_t& total, int& nmax,
                                        int64_t& before) {
    int64_t t = 0, pre = 0;
    int m = 0;
    for (int b = lane; b < B; b += 32) {
        const int n = sk_tiles(p, b);
        t += n;
        if (b < bq) pre += n;
        m = max(m, n);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        t += __shfl_xor_sync(0xffffffffu, t, o);
        pre += __shfl_xor_sync(0xffffffffu, pre, o);
        m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    }
    total = t * p.Hkv;
    before = pre * p.Hkv;
    nmax = m;
}

// where CTA c's run starts, found once per CTA by warp 0
struct SkStart {
    int64_t lo, hi;  // the CTA's tiles [lo, hi)
    int64_t P;       // first tile of pair (b, kvh)
    int b, kvh, per;
};
__device__ __forceinline__ void sk_find_start(const AttnParams& p, int B, int c, int lane, SkStart& s) {
    int64_t total, before;
    int nmax;
    sk_scan(p, B, 0, lane, total, nmax, before);
    const int per = sk_per(total, nmax, p.sk_grid);
    const int64_t lo = (int64_t)c * per, hi = min(lo + per, total);
    // the sequence whose pairs hold tile lo: an inclusive prefix over the sequences, 32 at a time
    int64_t run = 0;  // tiles of the sequences before this group of 32
    int bs = B, ns = 0;
    int64_t ps = 0;
    for (int b0 = 0; b0 < B && lo < total; b0 += 32) {
        const int b = b0 + lane;
        const int n = b < B ? sk_tiles(p, b) : 0;
        int64_t v = (int64_t)n * p.Hkv;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int64_t y = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += y;
        }
        const bool hit = b < B && n > 0 && run + v > lo;
        const unsigned m = __ballot_sync(0xffffffffu, hit);
        if (m) {
            const int src = __ffs(m) - 1;
            bs = b0 + src;
            ns = __shfl_sync(0xffffffffu, n, src);
            ps = run + __shfl_sync(0xffffffffu, v, src) - (int64_t)ns * p.Hkv;  // first tile of sequence bs
            break;
        }
        run += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) {
        s.lo = lo;
        s.hi = hi;
        s.per = per;
        if (bs < B) {
            const int kvh = (int)((lo - ps) / ns);
            s.b = bs;
            s.kvh = kvh;
            s.P = ps + (int64_t)kvh * ns;
        } else {
            s.b = B;  // no tiles for this CTA
            s.kvh = 0;
            s.P = total;
        }
    }
}

// Walks this CTA's items in order: splits of `chunk` tokens (item c, c + grid, ...) or, with
// the balanced partition, the pieces of the pairs that meet the CTA's run of tiles.
struct ItemIter {
    int item, n_items, pairs, B;
    int64_t lo = 0, hi = 0, P = 0;
    int b = 0, kvh = 0, per = 1;
    __device__ ItemIter(const AttnParams& p, const SkStart& s, int pairs_, int n_items_)
        : item(blockIdx.x), n_items(n_items_), pairs(pairs_), B(pairs_ / p.Hkv) {
        if (p.sk_grid > 0) {
            lo = s.lo, hi = s.hi, P = s.P, b = s.b, kvh = s.kvh, per = s.per;
        }
    }
    __device__ __forceinline__ bool next(const AttnParams& p, AttnItem& it) {
        if (p.sk_grid <= 0) {
            while (item < n_items) {
                const int cur = item;
                item += gridDim.x;
                if (attn_item(p, cur, pairs, it)) return true;
            }
            return false;
        }
        while (b < B && P < hi) {
            const int n = sk_tiles(p, b);
            const int64_t P0 = P;
            const int bb = b, kv = kvh;
            P += n;
            if (++kvh == p.Hkv) kvh = 0, b++;
            if (n == 0 || P0 + n <= lo) continue;
            const int s0 = (int)(max(lo, P0) - P0), s1 = (int)(min(hi, P0 + n) - P0);
            it.b = bb;
            it.kvh = kv;
            it.split = (int)((int64_t)blockIdx.x - P0 / per);
            it.nsplit_b = (int)((P0 + n - 1) / per - P0 / per + 1);
            it.t0 = s0 * kT;
            it.t1 = min(p.pos[bb] + 1, s1 * kT);
            it.ntiles = s1 - s0;
            it.has_new = s1 == n;
            return true;
        }
        return false;
    }
};

// the number of kernels launch_attention_mma enqueues: the query/K/V prologue, the attention
// kernel, and the merge when any split is cut
int attn_mma_launches(int max_len, int chunk) { return (max_len + chunk - 1) / chunk > 1 ? 3 : 2; }

// Prologue of every (sequence, kv head), before the attention kernel (deltanet.rs:565-625):
// the kGQ queries RMS-normed with q_norm and rotated into qprep; the new key normed with
// k_norm and rotated, and the new key and value appended to the bf16 cache at `pos`.
template <int HD>
__global__ void __launch_bounds__(128) attn_prep_kernel(AttnParams p) {
    static_assert(HD % 4 == 0 && kGQ * HD % (4 * 128) == 0 && HD / 4 <= 128, "prep tiling");
    __shared__ __align__(16) float q_s[kGQ * HD];
    __shared__ __align__(16) float kn_s[HD];
    __shared__ __align__(16) float qw_s[HD], kw_s[HD];
    __shared__ float2 rope_s[HD / 2];
    __shared__ float sc[kGQ + 1];
    const int kvh = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    // the norm weights are constants: fetched before the grid dependency wait
    if (tid < HD / 4) {
        if (p.q_norm) reinterpret_cast<float4*>(qw_s)[tid] = reinterpret_cast<const float4*>(p.q_norm)[tid];
        if (p.k_norm) reinterpret_cast<float4*>(kw_s)[tid] = reinterpret_cast<const float4*>(p.k_norm)[tid];
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // every input load in flight at once: position, queries, key, value
    const int pos = p.pos[b];
    if (!attn_pos_ok(p, pos)) {  // nothing is appended or read at an out-of-range position
        if (tid == 0 && kvh == 0 && p.err) atomicOr(p.err, kAttnErrPos);
        return;
    }
    const float* proj = p.proj + (size_t)b * p.ldp;
    // the projection holds every head of the model; this launch runs kv heads kvh0 + kvh
    const int kvg = p.kvh0 + kvh, Hkv_all = p.Hkv_all ? p.Hkv_all : p.Hkv;
    const int koff = p.Hq * 2 * HD, voff = koff + Hkv_all * HD;
    constexpr int kQ4 = kGQ * HD / 4 / 128;  // float4 of queries per thread
    float4 qv[kQ4], kv4 = make_float4(0.f, 0.f, 0.f, 0.f), vv4 = kv4;
#pragma unroll
    for (int i = 0; i < kQ4; i++) {
        const int e = (tid + i * 128) * 4, hh = e / HD, d = e % HD;
        qv[i] = *reinterpret_cast<const float4*>(proj + (size_t)(kvg * kGQ + hh) * 2 * HD + d);
    }
    if (tid < HD / 4) {
        kv4 = *reinterpret_cast<const float4*>(proj + koff + kvg * HD + tid * 4);
        vv4 = *reinterpret_cast<const float4*>(proj + voff + kvg * HD + tid * 4);
    }
    const int half_rot = p.rot / 2;
    const float2* rope = p.rope + (size_t)pos * half_rot;
    for (int j = tid; j < half_rot; j += 128) rope_s[j] = rope[j];
#pragma unroll
    for (int i = 0; i < kQ4; i++) reinterpret_cast<float4*>(q_s)[tid + i * 128] = qv[i];
    const size_t cache_off = (size_t)b * p.kv_slot_stride + (size_t)kvh * p.cap * HD + (size_t)pos * HD;
    if (tid < HD / 4) {
        reinterpret_cast<float4*>(kn_s)[tid] = kv4;
        // the value is appended as it is (deltanet.rs:618-625)
        __nv_bfloat162* vc = reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<__nv_bfloat16*>(p.vc) + cache_off);
        vc[2 * tid] = __floats2bfloat162_rn(vv4.x, vv4.y);
        vc[2 * tid + 1] = __floats2bfloat162_rn(vv4.z, vv4.w);
    }
    __syncthreads();
    // warps 0..3: query heads; warp 0 also the key
    {
        float ss = 0.0f;
        for (int d = lane; d < HD; d += 32) ss += q_s[warp * HD + d] * q_s[warp * HD + d];
        ss = warp_sum(ss);
        if (lane == 0) sc[warp] = p.q_norm ? 1.0f / sqrtf(ss / (float)HD + 1e-6f) : 1.0f;
        if (warp == 0) {
            float sk = 0.0f;
            for (int d = lane; d < HD; d += 32) sk += kn_s[d] * kn_s[d];
            sk = warp_sum(sk);
            if (lane == 0) sc[kGQ] = p.k_norm ? 1.0f / sqrtf(sk / (float)HD + 1e-6f) : 1.0f;
        }
    }
    __syncthreads();
    // RMSNorm then RoPE on the first `rot` dims, one (head, dim pair) per thread step; the
    // queries go to qprep, the key to the cache (deltanet.rs:565-617)
    float* qo = p.qprep + ((size_t)b * p.Hkv + kvh) * kGQ * HD;
    __nv_bfloat162* kc = reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<__nv_bfloat16*>(p.kc) + cache_off);
    for (int e = tid; e < (kGQ + 1) * (HD / 2); e += 128) {
        const int hh = e / (HD / 2), j = e % (HD / 2);
        const bool is_q = hh < kGQ;
        const float* src = is_q ? q_s + hh * HD : kn_s;
        float a0 = src[2 * j], a1 = src[2 * j + 1];
        if (is_q ? p.q_norm != nullptr : p.k_norm != nullptr) {
            const float* nw = is_q ? qw_s : kw_s;
            a0 = a0 * sc[hh] * nw[2 * j];
            a1 = a1 * sc[hh] * nw[2 * j + 1];
        }
        if (j < half_rot) {
            const float2 cs = rope_s[j];
            const float r0 = a0 * cs.x - a1 * cs.y, r1 = a0 * cs.y + a1 * cs.x;
            a0 = r0;
            a1 = r1;
        }
        if (is_q)
            *reinterpret_cast<float2*>(qo + hh * HD + 2 * j) = make_float2(a0, a1);
        else
            kc[j] = __floats2bfloat162_rn(a0, a1);
    }
}

__device__ __forceinline__ void comp_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kCompWarps * 32) : "memory"); }
// comp_bar that also returns the OR of `v` over the compute threads: a wait outcome that every
// compute thread then acts on alike, so none of them is left at a later barrier alone
__device__ __forceinline__ bool comp_bar_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.or.pred p, 1, %2, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(kCompWarps * 32)
        : "memory");
    return r != 0;
}

// Persistent kernel: CTA c takes items c, c + gridDim.x, ...; the producer warp streams the
// tiles of all of them through one ring, so the pipeline does not drain between items, and
// with each item's first tile it copies the item's prepared queries (attn_prep_kernel) into
// one of two query slots, so a new item starts without a prologue.
template <int HD>
__global__ void __launch_bounds__(kAttnMmaThreads, 1)
    attn_mma_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv, AttnParams p,
                    int64_t row_base, int pairs, int n_items) {
    using L = AttnSmem<HD>;
    constexpr int NDB = L::kNDB;
    constexpr int kCT = kCompWarps * 32;
    constexpr uint32_t kQBytes = kGQ * HD * 4;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    float* S_s = reinterpret_cast<float*>(smem + L::s_off());
    __nv_bfloat16* P_s = reinterpret_cast<__nv_bfloat16*>(smem + L::p_off());
    float* o_s = reinterpret_cast<float*>(smem + L::o_off());
    float* corr_s = reinterpret_cast<float*>(smem + L::misc_off());
    float* m_s = corr_s + 4;
    float* l_s = corr_s + 8;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::bar_off());
    uint64_t* empty = full + kAttnStages;
    uint64_t* q_full = empty + kAttnStages;
    uint64_t* q_free = q_full + 2;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr uint32_t kStageTx = 2u * L::kTileBytes;
    const uint32_t WL = p.wt.wait_ns;  // the limit of every wait below

    if (threadIdx.x == 0) {
        for (int s = 0; s < kAttnStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kCT);
        }
        for (int j = 0; j < 2; j++) {
            mbar_init(&q_full[j], 1);
            mbar_init(&q_free[j], kCT);
        }
        mbar_fence_init();
    }
    // rows 8-15 of the P operand stay zero; rows 0-7 are rewritten for every tile
    for (int i = threadIdx.x; i < 16 * kPStride; i += kAttnMmaThreads) P_s[i] = __float2bfloat16_rn(0.0f);
    __shared__ SkStart sk_s;
    if (p.sk_grid > 0) {
        // the balanced partition reads the positions: after the predecessor, like every role below
        asm volatile("griddepcontrol.wait;" ::: "memory");
        if (warp == 0) sk_find_start(p, pairs / p.Hkv, blockIdx.x, lane, sk_s);
    }
    __syncthreads();

    if (warp == kCompWarps) {
        // ---------------- producer: queries and K/V tiles of every item of this CTA, in order
        if (lane == 0) {
            asm volatile("griddepcontrol.wait;" ::: "memory");  // prepared queries and appended K/V
            int i = 0, k = 0;
            bool ok = true;
            ItemIter items(p, sk_s, pairs, n_items);
            AttnItem it;
            while (ok && items.next(p, it)) {
                const int pair = it.b * p.Hkv + it.kvh;
                const int qs = k & 1;
                if (k >= 2 && !mbar_wait(&q_free[qs], ((k >> 1) - 1) & 1, WL)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&q_full[qs], kQBytes);
                bulk_g2s(smem + L::q_off(qs), p.qprep + (size_t)pair * kGQ * HD, kQBytes, &q_full[qs]);
                k++;
                const int64_t seq_rows = p.seq_rows < 0 ? (int64_t)p.Hkv * p.cap : p.seq_rows;
                const int rows0 = (int)(row_base + it.b * seq_rows + (int64_t)it.kvh * p.cap + it.t0);
                for (int t = 0; t < it.ntiles; t++, i++) {
                    const int s = i % kAttnStages;
                    if (i >= kAttnStages && !mbar_wait(&empty[s], ((i / kAttnStages) - 1) & 1, WL)) {
                        ok = false;
                        break;
                    }
                    if (i == p.wt.withhold) continue;  // test hook: this tile is never copied
                    mbar_arrive_expect_tx(&full[s], kStageTx);
#pragma unroll
                    for (int d = 0; d < NDB; d++) {
                        tma_load_2d(smem + L::k_off(s) + d * 8192, &tmk, d * 64, rows0 + t * kT, &full[s]);
                        tma_load_2d(smem + L::v_off(s) + d * 8192, &tmv, d * 64, rows0 + t * kT, &full[s]);
                    }
                }
            }
            if (!ok && p.err) atomicOr(p.err, 4096u);
            // all K/V copies of this CTA are issued: pull its share of the output projection's
            // weights into L2 for the GEMM that follows
            prefetch_share_l2(p.pf, p.pf_bytes, blockIdx.x, gridDim.x);
            // every issued copy lands before the CTA can exit
            for (int j = max(0, i - kAttnStages); j < i; j++)
                if (j != p.wt.withhold) mbar_wait(&full[j % kAttnStages], (j / kAttnStages) & 1, WL);
            for (int j = max(0, k - 2); j < k; j++) mbar_wait(&q_full[j & 1], (j >> 1) & 1, WL);
        }
        __syncwarp();
        return;
    }

    // ---------------- compute warps
    const int ct = threadIdx.x;
    const int g = lane >> 2, t = lane & 3;
    const int hq = g & 3;  // head of this lane's operand row (rows 0-3 hi, 4-7 lo)
    const bool lo_row = g >= 4;
    const float sq = sqrtf((float)HD);
    const uint32_t pbase = smem_u32(P_s);
    constexpr int NPV = HD / 32;  // 8-dim n-tiles of this warp's HD/4 output dims
    asm volatile("griddepcontrol.wait;" ::: "memory");  // outputs may be read by earlier kernels
    int i = 0, k = 0;  // tile and item counters, in step with the producer
    ItemIter items(p, sk_s, pairs, n_items);
    AttnItem it;
    while (items.next(p, it)) {
        const int b = it.b, kvh = it.kvh;
        const float* proj = p.proj + (size_t)b * p.ldp;

        // Q A-fragments for every k16 step: a0 = (row g, k 2t..2t+1), a2 = (row g, k 2t+8..+9)
        // A wait that times out is not acted on alone: the outcome is combined over the compute
        // threads at the tile's first barrier (below), and all of them stop there together.
        // Until then a thread whose wait timed out reads stale (in-bounds) shared memory.
        const int qs = k & 1;
        const bool q_ok = mbar_wait(&q_full[qs], (k >> 1) & 1, WL);
        const float* q_s = reinterpret_cast<const float*>(smem + L::q_off(qs));
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
        k++;
        float o[NPV][4];
#pragma unroll
        for (int n = 0; n < NPV; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
        float m_run = -INFINITY, l_run = 0.0f;  // head `warp` (warps 0..3 own heads 0..3)

        bool ok = true;
        for (int tt0 = 0; tt0 < it.ntiles; tt0++, i++) {
            const int s = i % kAttnStages;
            const bool w_ok = mbar_wait(&full[s], (i / kAttnStages) & 1, WL);
            const uint32_t kb = smem_u32(smem + L::k_off(s)), vb = smem_u32(smem + L::v_off(s));
            const int tbase = it.t0 + tt0 * kT;
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
                    S_s[g * kT + tt] = (tbase + tt < it.t1) ? s0 / sq : -INFINITY;
                    S_s[g * kT + tt + 1] = (tbase + tt + 1 < it.t1) ? s1 / sq : -INFINITY;
                }
            }
            if (comp_bar_or(!(q_ok && w_ok))) {
                ok = false;
                break;
            }
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
            comp_bar();
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
        // The query slot is released after the item's tiles: the MMAs above consumed the
        // registers loaded from it, so those loads are complete before the next copy into the
        // slot can start (an arrival right after issuing them would not guarantee that).
        mbar_arrive(&q_free[qs]);
        if (!ok) {
            // a timed-out wait: report it and stop; the results of this launch are invalid
            if (ct == 0 && p.err) atomicOr(p.err, 4096u);
            break;
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
        // unnormalised O of this item into o_s [4][HD]
        if (g < 4) {
#pragma unroll
            for (int n = 0; n < NPV; n++) {
                const int d = warp * (HD / 4) + 8 * n + 2 * t;
                o_s[g * HD + d] = o[n][0];
                o_s[g * HD + d + 1] = o[n][1];
            }
        }
        comp_bar();
        if (it.nsplit_b == 1) {
            // a lone split: the output itself
            for (int e = ct; e < kGQ * HD; e += kCT) {
                const int hh = e / HD, d = e % HD, h = (p.kvh0 + kvh) * kGQ + hh;  // head in the model
                float ov = o_s[e] / l_s[hh];
                ov *= ref_sigmoid(proj[(size_t)h * 2 * HD + HD + d]);
                act_store(p.out, b, h * HD + d, ov);
                if (p.o_out) p.o_out[(size_t)b * p.Hq * HD + h * HD + d] = ov;
            }
        } else {
            // a split of several: its partial (m, l, unnormalised O) for attn_merge_kernel
            const size_t part_floats = (size_t)kGQ * 2 + (size_t)kGQ * HD;
            float* mypart = p.ws + (((size_t)b * p.Hkv + kvh) * kMaxSplits + it.split) * part_floats;
            for (int e = ct; e < kGQ * HD; e += kCT) __stcg(mypart + 2 * kGQ + e, o_s[e]);
            if (ct < kGQ) {
                __stcg(mypart + ct, m_s[ct]);
                __stcg(mypart + kGQ + ct, l_s[ct]);
            }
        }
        comp_bar();  // o_s, m_s, l_s are reused by the next item
    }
}

// Merge of the split partials of one (sequence, kv head) per CTA, in split order: weights
// e_s = exp(m_s - M) per (split, head), O = sum_s e_s O_s / sum_s e_s l_s, times the sigmoid
// output gate. Sequences handled by a single split were written by attn_mma_kernel.
template <int HD>
__global__ void __launch_bounds__(256) attn_merge_kernel(AttnParams p) {
    __shared__ float e_s[kMaxSplits * kGQ], lsum_s[kGQ];
    const int kvh = blockIdx.x, b = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (!attn_pos_ok(p, p.pos[b])) return;
    const int L = p.pos[b] + 1;
    int nsplit = (L + p.chunk - 1) / p.chunk;
    if (p.sk_grid > 0) {
        // the balanced partition: the CTAs that held a piece of this pair (every warp computes it)
        int64_t total, before;
        int nmax;
        sk_scan(p, gridDim.y, b, lane, total, nmax, before);
        const int per = sk_per(total, nmax, p.sk_grid);
        const int n = sk_tiles(p, b);
        const int64_t P = before + (int64_t)kvh * n;
        nsplit = (int)((P + n - 1) / per - P / per + 1);
    }
    if (nsplit <= 1) return;
    static_assert(kGQ * HD % 4 == 0 && kGQ * HD <= 4 * 256 && kMaxSplits <= 64, "merge tiling: a float4 of outputs per thread");
    const size_t part_floats = (size_t)kGQ * 2 + (size_t)kGQ * HD;
    const float* parts = p.ws + (((size_t)b * p.Hkv + kvh) * kMaxSplits) * part_floats;
    const float* proj = p.proj + (size_t)b * p.ldp;
    // this thread's four outputs (head hh, dims d..d+3) and their output gates, loaded first
    const int e4 = threadIdx.x * 4, hh = e4 / HD, d = e4 % HD, h = (p.kvh0 + kvh) * kGQ + hh;
    const bool has = e4 < kGQ * HD;
    float4 gt = make_float4(0.f, 0.f, 0.f, 0.f);
    if (has) gt = *reinterpret_cast<const float4*>(proj + (size_t)h * 2 * HD + HD + d);
    if (warp < kGQ) {
        // lane s and s + 32 hold split s's (m, l) for head `warp`
        float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
        if (lane < nsplit) {
            m0 = __ldcg(parts + lane * part_floats + warp);
            l0 = __ldcg(parts + lane * part_floats + kGQ + warp);
        }
        if (lane + 32 < nsplit) {
            m1 = __ldcg(parts + (lane + 32) * part_floats + warp);
            l1 = __ldcg(parts + (lane + 32) * part_floats + kGQ + warp);
        }
        const float M = warp_max(fmaxf(m0, m1));
        const float e0 = (m0 == -INFINITY) ? 0.0f : expf(m0 - M);
        const float e1 = (m1 == -INFINITY) ? 0.0f : expf(m1 - M);
        if (lane < nsplit) e_s[lane * kGQ + warp] = e0;
        if (lane + 32 < nsplit) e_s[(lane + 32) * kGQ + warp] = e1;
        float Ls = l0 * e0;
        Ls += l1 * e1;
        Ls = warp_sum(Ls);
        if (lane == 0) lsum_s[warp] = Ls;
    }
    __syncthreads();
    if (!has) return;
    float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int s = 0; s < nsplit; s++) {
        const float4 o = __ldcg(reinterpret_cast<const float4*>(parts + s * part_floats + 2 * kGQ + e4));
        const float w = e_s[s * kGQ + hh];
        A.x += o.x * w;
        A.y += o.y * w;
        A.z += o.z * w;
        A.w += o.w * w;
    }
    const float inv_l = lsum_s[hh];
    const float av[4] = {A.x, A.y, A.z, A.w}, gv[4] = {gt.x, gt.y, gt.z, gt.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float ov = av[i] / inv_l;
        ov *= ref_sigmoid(gv[i]);
        act_store(p.out, b, h * HD + d + i, ov);
        if (p.o_out) p.o_out[(size_t)b * p.Hq * HD + h * HD + d + i] = ov;
    }
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

// Tokens per split of the persistent kernel. Items (split, sequence, kv head) are dealt to
// the SMs round-robin, so the item count should sit just below a multiple of the SM count;
// each item also costs about one tile of fixed work (prologue, partial write, merge). The
// chunk minimising ceil(items / SMs) * (tiles per item + 1) wins, with at least
// kMinSplitTiles tiles per split and at most kMaxSplits splits.
constexpr int kMinSplitTiles = 4;
int attn_mma_chunk(int batch, int hkv, int max_len, int num_sms) {
    const int64_t pairs = (int64_t)batch * hkv;
    int best_chunk = 0;
    int64_t best_cost = INT64_MAX;
    const int min_chunk = std::max(kMinSplitTiles * kT, (max_len + kMaxSplits - 1) / kMaxSplits);
    for (int chunk = (min_chunk + kT - 1) / kT * kT; ; chunk += kT) {
        const int64_t splits = (max_len + chunk - 1) / chunk;
        const int64_t items = pairs * splits;
        const int64_t per_cta = (items + num_sms - 1) / num_sms;
        const int64_t cost = per_cta * (chunk / kT + 1);
        if (cost < best_cost) {
            best_cost = cost;
            best_chunk = chunk;
        }
        if (splits == 1) break;
    }
    return best_chunk;
}

// splits per (sequence, kv head) never exceed kMaxSplits: the workspace is sized for that
int attn_mma_nsplit_bound(int batch, int hkv, int cap, int num_sms) {
    (void)batch, (void)hkv, (void)cap, (void)num_sms;
    return kMaxSplits;
}

template <int HD>
static int launch_mma_t(const void* tmk, const void* tmv, const AttnParams& p, int64_t row_base, int batch,
                        int max_len, int num_sms, cudaStream_t st, cudaEvent_t core_begin, cudaEvent_t core_end) {
    const int smem = AttnSmem<HD>::bytes() + 1024;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev & 63]) {
        if (cudaFuncSetAttribute(attn_mma_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return -1;
        attr_set[dev & 63] = true;
    }
    const int pairs = batch * p.Hkv;
    const int splits = attn_nsplit(max_len, p.chunk);
    if (splits > kMaxSplits || !p.qprep) return -1;
    const int n_items = pairs * splits;
    int grid = std::min(n_items, num_sms);
    AttnParams pm = p;
    pm.sk_grid = 0;
    if (splits > 1) {
        // the balanced partition when it beats the chunk plan: per CTA, the chunk plan costs its
        // items' tiles plus one tile of fixed work per item; the balanced one an equal share of
        // the tiles plus at most ceil(share / tiles per pair) + 1 items
        const int max_tiles = (max_len + kT - 1) / kT;
        const int64_t chunk_cost = (int64_t)((n_items + grid - 1) / grid) * (p.chunk / kT + 1);
        const int per = sk_per((int64_t)pairs * max_tiles, max_tiles, num_sms);
        const int64_t sk_cost = per + (per + max_tiles - 1) / max_tiles + 1;
        if (sk_cost < chunk_cost) {
            pm.sk_grid = num_sms;
            grid = num_sms;
        }
    }
    if (launch_pdl(attn_prep_kernel<HD>, dim3(p.Hkv, batch), dim3(128), 0, st, p) != cudaSuccess) return -2;
    if (core_begin) cudaEventRecord(core_begin, st);
    pm.wt = take_wait_test(kWaitTestAttention, st);
    if (launch_pdl(attn_mma_kernel<HD>, dim3(grid), dim3(kAttnMmaThreads), smem, st,
                   *reinterpret_cast<const CUtensorMap*>(tmk), *reinterpret_cast<const CUtensorMap*>(tmv), pm,
                   row_base, pairs, n_items) != cudaSuccess)
        return -2;
    if (core_end) cudaEventRecord(core_end, st);
    AttnParams mp = p;
    mp.sk_grid = pm.sk_grid;
    if (splits > 1) launch_pdl(attn_merge_kernel<HD>, dim3(p.Hkv, batch), dim3(256), 0, st, mp);
    return 0;
}

// the query/K/V prologue and the split merge alone, for the prefill kernel (attn_prefill.cu)
int launch_attn_prep(const AttnParams& p, int batch, int hd, cudaStream_t st) {
    if (hd == 256) return launch_pdl(attn_prep_kernel<256>, dim3(p.Hkv, batch), dim3(128), 0, st, p) == cudaSuccess ? 0 : -2;
    if (hd == 128) return launch_pdl(attn_prep_kernel<128>, dim3(p.Hkv, batch), dim3(128), 0, st, p) == cudaSuccess ? 0 : -2;
    return -1;
}
int launch_attn_merge(const AttnParams& p, int batch, int hd, cudaStream_t st) {
    if (hd == 256) return launch_pdl(attn_merge_kernel<256>, dim3(p.Hkv, batch), dim3(256), 0, st, p) == cudaSuccess ? 0 : -2;
    if (hd == 128) return launch_pdl(attn_merge_kernel<128>, dim3(p.Hkv, batch), dim3(256), 0, st, p) == cudaSuccess ? 0 : -2;
    return -1;
}

int launch_attention_mma(const void* tmk, const void* tmv, const AttnParams& p, int64_t row_base, int batch, int hd,
                         int max_len, int num_sms, cudaStream_t st, cudaEvent_t core_begin, cudaEvent_t core_end) {
    if (p.Hq != kGQ * (p.Hkv_all ? p.Hkv_all : p.Hkv)) return -1;
    if (hd == 256) return launch_mma_t<256>(tmk, tmv, p, row_base, batch, max_len, num_sms, st, core_begin, core_end);
    if (hd == 128) return launch_mma_t<128>(tmk, tmv, p, row_base, batch, max_len, num_sms, st, core_begin, core_end);
    return -1;
}

}  // namespace ab2
