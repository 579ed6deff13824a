// misc.cu -- RMSNorm into GEMM activation fragments, f32 -> fragments, greedy argmax.
#include "common.cuh"
#include "kernels.h"

namespace ab2 {

// out = x * (1 / sqrt(mean(x^2) + eps)) * w, written as activation fragments for the next
// GEMM (rmsnorm_vec, crates/cli/src/main.rs:1106-1113). One CTA per batch row.
// out = x * (1 / sqrt(mean(x^2) + eps)) * w, written in the next GEMM's activation layout
// (rmsnorm_vec, crates/cli/src/main.rs:1106-1113). One CTA per batch row. Rows of up to
// kNormChunks * 2048 elements with D a multiple of 8 take the fast path: each thread holds 8 consecutive elements per chunk in
// registers, so x is read once; the norm weights do not depend on the previous kernel and
// are loaded before the grid dependency wait.
constexpr int kNormChunks = 2;

__global__ void __launch_bounds__(256) rmsnorm_act_kernel(const float* __restrict__ x, int ldx,
                                                          const float* __restrict__ w, int D, float eps, ActOut out,
                                                          float* __restrict__ zero_ptr, int zero_ld, int zero_n) {
    __shared__ float red[8];
    const int b = blockIdx.x, tid = threadIdx.x;
    const bool fast = D % 8 == 0 && D <= kNormChunks * 256 * 8 && (ldx & 3) == 0;
    float4 wv[kNormChunks][2];
    if (fast) {
#pragma unroll
        for (int ch = 0; ch < kNormChunks; ch++) {
            const int k0 = (tid + ch * 256) * 8;
            if (k0 < D) {
                wv[ch][0] = *reinterpret_cast<const float4*>(w + k0);
                wv[ch][1] = *reinterpret_cast<const float4*>(w + k0 + 4);
            }
        }
    }
    // The GEMM that follows may start (and stream its constant weights into shared memory on
    // the SMs the previous GEMM leaves idle) while this kernel still waits for its own input:
    // its activation loads wait for this grid to complete.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const float* xb = x + (size_t)b * ldx;
    if (!fast) {
        if (zero_ptr)
            for (int i = tid; i < zero_n; i += 256) zero_ptr[(size_t)b * zero_ld + i] = 0.0f;
        float ss = 0.0f;
        for (int i = tid; i < D; i += 256) ss += xb[i] * xb[i];
        ss = block_sum<256>(ss, red);
        ss = ss / (float)D;
        const float inv = 1.0f / sqrtf(ss + eps);
        for (int i = tid; i < D; i += 256) act_store(out, b, i, xb[i] * inv * w[i]);
        return;
    }
    float4 xv[kNormChunks][2];
#pragma unroll
    for (int ch = 0; ch < kNormChunks; ch++) {
        const int k0 = (tid + ch * 256) * 8;
        if (k0 < D) {
            xv[ch][0] = *reinterpret_cast<const float4*>(xb + k0);
            xv[ch][1] = *reinterpret_cast<const float4*>(xb + k0 + 4);
        }
    }
    // a K-split GEMM that follows adds into these projection rows: clear them
    if (zero_ptr) {
        float* zr = zero_ptr + (size_t)b * zero_ld;
        if ((zero_n & 3) == 0 && (zero_ld & 3) == 0 && (reinterpret_cast<uintptr_t>(zero_ptr) & 15) == 0) {
            for (int i = tid * 4; i < zero_n; i += 256 * 4) *reinterpret_cast<float4*>(zr + i) = make_float4(0.f, 0.f, 0.f, 0.f);
        } else {
            for (int i = tid; i < zero_n; i += 256) zr[i] = 0.0f;
        }
    }
    float ss = 0.0f;
#pragma unroll
    for (int ch = 0; ch < kNormChunks; ch++) {
        if ((tid + ch * 256) * 8 < D) {
#pragma unroll
            for (int h = 0; h < 2; h++) {
                ss += xv[ch][h].x * xv[ch][h].x;
                ss += xv[ch][h].y * xv[ch][h].y;
                ss += xv[ch][h].z * xv[ch][h].z;
                ss += xv[ch][h].w * xv[ch][h].w;
            }
        }
    }
    ss = block_sum<256>(ss, red);
    ss = ss / (float)D;
    const float inv = 1.0f / sqrtf(ss + eps);
#pragma unroll
    for (int ch = 0; ch < kNormChunks; ch++) {
        const int k0 = (tid + ch * 256) * 8;
        if (k0 >= D) continue;
        const float xs[8] = {xv[ch][0].x, xv[ch][0].y, xv[ch][0].z, xv[ch][0].w,
                             xv[ch][1].x, xv[ch][1].y, xv[ch][1].z, xv[ch][1].w};
        const float ws[8] = {wv[ch][0].x, wv[ch][0].y, wv[ch][0].z, wv[ch][0].w,
                             wv[ch][1].x, wv[ch][1].y, wv[ch][1].z, wv[ch][1].w};
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] = xs[e] * inv * ws[e];
        if (out.x16) {
            // 8 consecutive k of one row are one 16-byte chunk of the x16 image
            uint32_t pk[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                __half2 t = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
                pk[e] = *reinterpret_cast<uint32_t*>(&t);
            }
            *reinterpret_cast<uint4*>(out.buf + x16_offset(out.npad, b, k0)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        } else {
#pragma unroll
            for (int e = 0; e < 8; e++) act_store(out, b, k0 + e, v[e]);
        }
    }
}

// The x16 layout pads K to a multiple of 64; the pad is cleared, because it meets zero
// weights in the GEMM and a stale non-finite value there would poison the sums.
__global__ void to_act_kernel(const float* __restrict__ x, int ldx, int K, ActOut out) {
    const int b = blockIdx.x;
    const int kp = out.x16 ? (K + 63) / 64 * 64 : K;
    for (int i = threadIdx.x; i < kp; i += blockDim.x) act_store(out, b, i, i < K ? x[(size_t)b * ldx + i] : 0.0f);
}

// Two-pass argmax under f32::total_cmp with ties going to the last index, as
// Iterator::max_by (greedy_sample, crates/cli/src/main.rs:1767-1785): pass 1 reduces chunk c
// of row b to (key, index) in part[b][c]
__global__ void __launch_bounds__(512) argmax_part_kernel(const float* __restrict__ logits, int ld, int V,
                                                           int2* __restrict__ part) {
    __shared__ int32_t sk[16], si[16];
    const int b = blockIdx.y, c = blockIdx.x, nch = gridDim.x;
    const int per = (V + nch - 1) / nch;
    const int lo = c * per, hi = min(V, lo + per);
    const float* l = logits + (size_t)b * ld;
    int32_t bk = INT32_MIN, bi = -1;
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const int32_t k = total_key(l[i]);
        if (k > bk || (k == bk && i > bi)) {
            bk = k;
            bi = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const int32_t ok = __shfl_xor_sync(kFull, bk, o), oi = __shfl_xor_sync(kFull, bi, o);
        if (ok > bk || (ok == bk && oi > bi)) {
            bk = ok;
            bi = oi;
        }
    }
    const int w = threadIdx.x >> 5, ln = threadIdx.x & 31;
    if (ln == 0) {
        sk[w] = bk;
        si[w] = bi;
    }
    __syncthreads();
    if (w == 0) {
        const int nw = blockDim.x >> 5;
        bk = ln < nw ? sk[ln] : INT32_MIN;
        bi = ln < nw ? si[ln] : -1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const int32_t ok = __shfl_xor_sync(kFull, bk, o), oi = __shfl_xor_sync(kFull, bi, o);
            if (ok > bk || (ok == bk && oi > bi)) {
                bk = ok;
                bi = oi;
            }
        }
        if (ln == 0) part[(size_t)b * nch + c] = make_int2(bk, bi);
    }
}

// pass 2: one warp per row over its nch partials
__global__ void argmax_final_kernel(const int2* __restrict__ part, int nch, int32_t* __restrict__ out) {
    const int b = blockIdx.x, ln = threadIdx.x;
    int32_t bk = INT32_MIN, bi = -1;
    for (int c = ln; c < nch; c += 32) {
        const int2 v = part[(size_t)b * nch + c];
        if (v.y >= 0 && (v.x > bk || (v.x == bk && v.y > bi))) {
            bk = v.x;
            bi = v.y;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const int32_t ok = __shfl_xor_sync(kFull, bk, o), oi = __shfl_xor_sync(kFull, bi, o);
        if (ok > bk || (ok == bk && oi > bi)) {
            bk = ok;
            bi = oi;
        }
    }
    if (ln == 0) out[b] = bi < 0 ? 0 : bi;
}

void launch_argmax2(const float* logits, int ld, int V, int batch, int32_t* out, int2* part, int nch,
                    cudaStream_t st) {
    argmax_part_kernel<<<dim3(nch, batch), 512, 0, st>>>(logits, ld, V, part);
    argmax_final_kernel<<<batch, 32, 0, st>>>(part, nch, out);
}

void launch_rmsnorm_act(const float* x, int ldx, const float* w, int D, float eps, int batch, const ActOut& out,
                        cudaStream_t st, float* zero_ptr, int zero_ld, int zero_n) {
    launch_pdl(rmsnorm_act_kernel, dim3(batch), dim3(256), 0, st, x, ldx, w, D, eps, out, zero_ptr, zero_ld, zero_n);
}

void launch_to_act(const float* x, int ldx, int K, int batch, const ActOut& out, cudaStream_t st) {
    to_act_kernel<<<batch, 256, 0, st>>>(x, ldx, K, out);
}

__global__ void pos_advance_kernel(int32_t* pos, int batch) {
    int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < batch) pos[b] += 1;
}

// counter-based normal samples: splitmix64 hash of (seed, stream, index) -> Box-Muller
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}
__device__ __forceinline__ float hash_normal(uint64_t seed, uint64_t stream, uint64_t i) {
    uint64_t h = mix64(seed ^ mix64(stream * 0x632be59bd9b4e019ull + i));
    float u1 = ((float)(h >> 40) + 1.0f) * (1.0f / 16777217.0f);   // (0, 1]
    float u2 = (float)((h >> 16) & 0xffffffu) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

// dst[i] = sample (i0 + i) of the stream
__global__ void seed_f32_kernel(float* dst, int64_t n, uint64_t seed, uint64_t stream, float std, int64_t i0) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i < n; i += (int64_t)gridDim.x * blockDim.x) dst[i] = std * hash_normal(seed, stream, (uint64_t)(i0 + i));
}

// rows of hd values at [row][0, hd) for rows with (row % cap) < n_tokens, bf16-representable;
// element i takes sample (i0 + i) of the stream (i0 a multiple of cap * hd)
template <typename T>
__global__ void seed_kv_kernel(T* dst, int64_t rows, int cap, int64_t n_tokens, int hd, uint64_t seed,
                               uint64_t stream, float std, int64_t i0) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t n = rows * hd;
    for (; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t row = i / hd;
        if (row % cap >= n_tokens) continue;
        float v = __bfloat162float(__float2bfloat16_rn(std * hash_normal(seed, stream, (uint64_t)(i0 + i))));
        if constexpr (sizeof(T) == 4) dst[i] = v;
        else dst[i] = __float2bfloat16_rn(v);
    }
}

void launch_pos_advance(int32_t* pos, int batch, cudaStream_t st) {
    pos_advance_kernel<<<(batch + 127) / 128, 128, 0, st>>>(pos, batch);
}

__global__ void pos_fill_kernel(int32_t* pos, int p0, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) pos[i] = p0 + i;
}

void launch_pos_fill(int32_t* pos, int p0, int n, cudaStream_t st) {
    pos_fill_kernel<<<(n + 127) / 128, 128, 0, st>>>(pos, p0, n);
}

void launch_seed_f32(float* dst, int64_t n, uint64_t seed, uint64_t stream, float std, cudaStream_t st,
                     int64_t i0) {
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 64) blocks = 148 * 64;
    seed_f32_kernel<<<(unsigned)blocks, 256, 0, st>>>(dst, n, seed, stream, std, i0);
}

void launch_seed_kv(void* dst, bool bf16, int64_t rows, int cap, int64_t n_tokens, int hd, uint64_t seed,
                    uint64_t stream, float std, cudaStream_t st, int64_t i0) {
    int64_t blocks = (rows * hd + 255) / 256;
    if (blocks > 148 * 64) blocks = 148 * 64;
    if (bf16)
        seed_kv_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, st>>>((__nv_bfloat16*)dst, rows, cap, n_tokens,
                                                                       hd, seed, stream, std, i0);
    else
        seed_kv_kernel<float><<<(unsigned)blocks, 256, 0, st>>>((float*)dst, rows, cap, n_tokens, hd, seed, stream,
                                                               std, i0);
}

}  // namespace ab2
