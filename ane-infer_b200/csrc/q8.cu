// q8.cu -- Q8_0 weight kernels: upload repack, exact dequant, dequant-GEMV/GEMM, embedding.
//
// Reference semantics: a Q8_0 weight w = (f32)(i8 q) * (f32)(f16 d) per 32-element block
// (crates/gguf/src/dequant.rs:29-38), and the GEMV y[r] = sum_b d_b * sum_i q_i x_i
// (crates/engine/src/q8_gemv.rs:230-244). The device GEMM keeps the weights exact: the int8
// q becomes an exact f16 in registers, each 32-wide block is contracted on the tensor core
// into a fresh f32 fragment and then scaled by its f16 d in f32 (acc += d * block_sum),
// which is the reference's per-block order. Activations enter as an f16 hi/lo pair that
// represents the f32 value to 2^-22, so the result tracks the f32 reference closely.
#include "common.cuh"
#include "kernels.h"

namespace ab2 {

// ------------------------------------------------------------------------------ repack
// One thread per source (row, block): scatter 32 q bytes and one d into the q8p layout.
// dst_row = base + (row / grp) * stride + row % grp   (concatenation and 8-row interleave)
__global__ void q8_repack_kernel(const uint8_t* __restrict__ src, int64_t rows, int KB, uint8_t* __restrict__ qs,
                                 uint16_t* __restrict__ dh, int64_t base, int64_t grp, int64_t stride) {
    int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (id >= rows * KB) return;
    int64_t r = id / KB;
    int kb = (int)(id % KB);
    const uint8_t* blk = src + id * 34;
    int64_t R = base + (r / grp) * stride + (r % grp);
    int64_t mt = R >> 4;
    int rr = (int)(R & 15), g = rr & 7, upper = rr >> 3;
    uint8_t* tile = qs + ((mt * KB + kb) * 32) * 16;
#pragma unroll 4
    for (int c = 0; c < 32; c++) {
        int s16 = c >> 4, c16 = c & 15, hi8 = c16 >> 3, c8 = c16 & 7, t = c8 >> 1, p = c8 & 1;
        int lane = 4 * g + t;
        tile[lane * 16 + s16 * 8 + (hi8 * 2 + upper) * 2 + p] = (uint8_t)(blk[2 + c] ^ 0x80u);
    }
    uint16_t d = (uint16_t)blk[0] | ((uint16_t)blk[1] << 8);
    dh[((mt * KB + kb) * 8 + g) * 2 + upper] = d;
}

// raw GGUF Q8_0 blocks -> f32, bit-exact with dequant_q8_0_block
__global__ void q8_dequant_raw_kernel(const uint8_t* __restrict__ src, int64_t n_blocks, float* __restrict__ out) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_blocks * 32) return;
    int64_t b = i >> 5;
    const uint8_t* blk = src + b * 34;
    float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
    out[i] = (float)(int8_t)blk[2 + (i & 31)] * d;
}

__device__ __forceinline__ float q8p_get(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dh, int KB,
                                         int64_t row, int k) {
    int64_t mt = row >> 4;
    int rr = (int)(row & 15), g = rr & 7, upper = rr >> 3;
    int kb = k >> 5, c = k & 31;
    int s16 = c >> 4, c16 = c & 15, hi8 = c16 >> 3, c8 = c16 & 7, t = c8 >> 1, p = c8 & 1;
    int lane = 4 * g + t;
    size_t tb = (size_t)(mt * KB + kb);
    int8_t q = (int8_t)(qs[(tb * 32 + lane) * 16 + s16 * 8 + (hi8 * 2 + upper) * 2 + p] ^ 0x80u);
    float d = __half2float(__ushort_as_half(dh[(tb * 8 + g) * 2 + upper]));
    return (float)q * d;
}

// packed layout -> f32 [rows][K] (checks the repack round trip bit-exactly)
__global__ void q8p_dequant_kernel(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dh, int KB,
                                   int64_t rows, float* __restrict__ out) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int K = KB * 32;
    if (i >= rows * K) return;
    out[i] = q8p_get(qs, dh, KB, i / K, (int)(i % K));
}

// x[b][k] = dequant(embedding row tokens[b]); out-of-range ids give a zero row
// (qwen35_forward_token, crates/cli/src/main.rs:966-970)
__global__ void embed_kernel(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dh, int KB, int vocab,
                             const int32_t* __restrict__ tokens, float* __restrict__ x, int ldx) {
    int b = blockIdx.x;
    int tok = tokens[b];
    int K = KB * 32;
    for (int k = threadIdx.x; k < K; k += blockDim.x)
        x[(size_t)b * ldx + k] = (tok >= 0 && tok < vocab) ? q8p_get(qs, dh, KB, tok, k) : 0.0f;
}

// ------------------------------------------------------------------------------ GEMM
__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint32_t ld_stream32(const uint32_t* p) {
    uint32_t r;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
}

template <int NT, bool PACKED>
__device__ __forceinline__ void gemm_epilogue(float acc[NT][4], int mt, int lane, int batch, const GemmEpi& ep) {
    const int g = lane >> 2, t = lane & 3;
    if (PACKED) {
        // columns 0..3 hold the hi part of batch rows 0..3, columns 4..7 the lo part
#pragma unroll
        for (int i = 0; i < 4; i++) acc[0][i] += __shfl_xor_sync(kFull, acc[0][i], 2);
        if (t >= 2) return;
    }
#pragma unroll
    for (int j = 0; j < NT; j++) {
#pragma unroll
        for (int c = 0; c < 2; c++) {
            int b = PACKED ? 2 * t + c : j * 8 + 2 * t + c;
            if (b >= batch) continue;
            float v0 = acc[j][c], v1 = acc[j][2 + c];  // rows g and g+8 of the m16 tile
            if (ep.mode == EPI_SWIGLU) {
                // rows g (gate) and g+8 (up) of tile mt are output mt*8+g (ffn_forward,
                // crates/cli/src/main.rs:1115-1135; silu_mul as in scratch.rs:181-186)
                int o = mt * 8 + g;
                if (o < ep.m_out) {
                    float h = (v0 / (1.0f + expf(-v0))) * v1;
                    if (ep.out.buf) act_store(ep.out, b, o, h);
                    if (ep.y) ep.y[(size_t)b * ep.ldy + o] = h;
                }
            } else {
                int r0 = mt * 16 + g, r1 = r0 + 8;
                float* yb = ep.y + (size_t)b * ep.ldy;
                if (ep.mode == EPI_RESID) {
                    if (r0 < ep.m_out) yb[r0] += v0;
                    if (r1 < ep.m_out) yb[r1] += v1;
                } else {
                    if (r0 < ep.m_out) yb[r0] = v0;
                    if (r1 < ep.m_out) yb[r1] = v1;
                }
            }
        }
    }
}

// One warp = one m16 tile over a K range; WARPS consecutive tiles per CTA; grid.y splits K.
// Split-K partials are reduced deterministically by the CTA that arrives last (an atomic
// ticket per m-tile group, no waiting): it sums the partials in split order and runs the
// epilogue, then re-arms the ticket for the next launch.
template <int NT, bool PACKED, int WARPS>
__global__ void __launch_bounds__(WARPS * 32) q8_gemm_kernel(const uint4* __restrict__ qs,
                                                             const uint32_t* __restrict__ dsc, int M16, int KB,
                                                             const uint4* __restrict__ xf, int batch, int kps,
                                                             float4* __restrict__ ws,
                                                             unsigned* __restrict__ tickets, GemmEpi ep) {
    constexpr int NTILE = PACKED ? 1 : 2 * NT;
    constexpr int U = 4;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int mt = blockIdx.x * WARPS + warp;
    const int nsplit = gridDim.y, split = blockIdx.y;
    const int kb0 = split * kps, kb1 = min(KB, kb0 + kps);

    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; j++) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;

    // Launched with programmatic dependent launch: the next kernel may start setting up now,
    // and this one loads its first weight blocks (constants) before waiting for the kernel
    // that produced its activations; every read of activations, split partials, tickets and
    // outputs comes after the wait.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const uint4* qp = qs + (size_t)mt * KB * 32 + lane;
    const uint32_t* dp = dsc + (size_t)mt * KB * 8 + (lane >> 2);
    uint4 q[U];
    uint32_t d[U];
    if (mt < M16) {
#pragma unroll
        for (int u = 0; u < U; u++) {
            if (kb0 + u < kb1) {
                q[u] = ld_stream(qp + (size_t)(kb0 + u) * 32);
                d[u] = ld_stream32(dp + (size_t)(kb0 + u) * 8);
            }
        }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (mt < M16) {
        for (int kb = kb0; kb < kb1; kb += U) {
            if (kb != kb0) {
#pragma unroll
                for (int u = 0; u < U; u++) {
                    if (kb + u < kb1) {
                        q[u] = ld_stream(qp + (size_t)(kb + u) * 32);
                        d[u] = ld_stream32(dp + (size_t)(kb + u) * 8);
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                if (kb + u < kb1) {
                    uint32_t a[8];
                    q8_unpack(q[u], a);
                    const float dg = f16bits_to_f32(d[u]), dg8 = f16bits_to_f32(d[u] >> 16);
                    const uint4* xp = xf + (size_t)(kb + u) * NTILE * 32 + lane;
#pragma unroll
                    for (int j = 0; j < NT; j++) {
                        float tq[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                        const uint4 bh = __ldg(xp + j * 32);
                        mma_f16(tq, a, bh.x, bh.y);
                        mma_f16(tq, a + 4, bh.z, bh.w);
                        if (!PACKED) {
                            const uint4 bl = __ldg(xp + (NT + j) * 32);
                            mma_f16(tq, a, bl.x, bl.y);
                            mma_f16(tq, a + 4, bl.z, bl.w);
                        }
                        acc[j][0] = fmaf(dg, tq[0], acc[j][0]);
                        acc[j][1] = fmaf(dg, tq[1], acc[j][1]);
                        acc[j][2] = fmaf(dg8, tq[2], acc[j][2]);
                        acc[j][3] = fmaf(dg8, tq[3], acc[j][3]);
                    }
                }
            }
        }
    }

    if (nsplit > 1) {
        __shared__ unsigned s_last;
        if (mt < M16) {
#pragma unroll
            for (int j = 0; j < NT; j++)
                __stcg(&ws[(((size_t)split * M16 + mt) * NT + j) * 32 + lane],
                       make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]));
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned prev = atomicAdd(&tickets[blockIdx.x], 1u);
            s_last = (prev == (unsigned)nsplit - 1u) ? 1u : 0u;
        }
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        if (mt < M16) {
#pragma unroll
            for (int j = 0; j < NT; j++) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
            for (int s = 0; s < nsplit; s++) {
#pragma unroll
                for (int j = 0; j < NT; j++) {
                    float4 p = __ldcg(&ws[(((size_t)s * M16 + mt) * NT + j) * 32 + lane]);
                    acc[j][0] += p.x;
                    acc[j][1] += p.y;
                    acc[j][2] += p.z;
                    acc[j][3] += p.w;
                }
            }
        }
        if (threadIdx.x == 0) tickets[blockIdx.x] = 0u;
    }
    if (mt >= M16) return;
    gemm_epilogue<NT, PACKED>(acc, mt, lane, batch, ep);
}

// ------------------------------------------------------------------------------ launchers
constexpr int kGemmWarps = 8;

int gemm_grid_x(int M16) { return (M16 + kGemmWarps - 1) / kGemmWarps; }

// split-K so that the grid covers about three waves of the 148 SMs
int gemm_nsplit(int M16, int KB, int num_sms) {
    int gx = gemm_grid_x(M16);
    int want = (3 * num_sms + gx - 1) / gx;
    int maxs = KB / 4 > 0 ? KB / 4 : 1;
    int s = want < maxs ? want : maxs;
    if (s < 1) s = 1;
    int kps = (KB + s - 1) / s;
    return (KB + kps - 1) / kps;
}

size_t gemm_ws_floats(int M16, int KB, int batch, int num_sms) {
    int ns = gemm_nsplit(M16, KB, num_sms);
    if (ns <= 1) return 0;
    int nt = batch <= 4 ? 1 : (batch + 7) / 8;
    return (size_t)ns * M16 * nt * 32 * 4;
}

template <int NT, bool PACKED>
static void launch_gemm_t(const Q8Weight& w, const uint8_t* xf, int batch, float* ws, unsigned* tickets,
                          const GemmEpi& ep, int num_sms, cudaStream_t st) {
    int ns = gemm_nsplit(w.M16, w.KB, num_sms);
    int kps = (w.KB + ns - 1) / ns;
    dim3 grid(gemm_grid_x(w.M16), ns);
    launch_pdl(q8_gemm_kernel<NT, PACKED, kGemmWarps>, grid, dim3(kGemmWarps * 32), 0, st,
               reinterpret_cast<const uint4*>(w.qs), reinterpret_cast<const uint32_t*>(w.d), w.M16, w.KB,
               reinterpret_cast<const uint4*>(xf), batch, kps, reinterpret_cast<float4*>(ws), tickets, ep);
}

void launch_q8_gemm(const Q8Weight& w, const uint8_t* xf, int batch, float* ws, unsigned* tickets,
                    const GemmEpi& ep, int num_sms, cudaStream_t st) {
    if (batch <= 4) return launch_gemm_t<1, true>(w, xf, batch, ws, tickets, ep, num_sms, st);
    switch ((batch + 7) / 8) {
        case 1: return launch_gemm_t<1, false>(w, xf, batch, ws, tickets, ep, num_sms, st);
        case 2: return launch_gemm_t<2, false>(w, xf, batch, ws, tickets, ep, num_sms, st);
        case 3: return launch_gemm_t<3, false>(w, xf, batch, ws, tickets, ep, num_sms, st);
        case 4: return launch_gemm_t<4, false>(w, xf, batch, ws, tickets, ep, num_sms, st);
        case 5: return launch_gemm_t<5, false>(w, xf, batch, ws, tickets, ep, num_sms, st);
        case 6: return launch_gemm_t<6, false>(w, xf, batch, ws, tickets, ep, num_sms, st);
        case 7: return launch_gemm_t<7, false>(w, xf, batch, ws, tickets, ep, num_sms, st);
        default: return launch_gemm_t<8, false>(w, xf, batch, ws, tickets, ep, num_sms, st);
    }
}

void launch_q8_repack(const uint8_t* src, int64_t rows, int KB, Q8Weight& w, int64_t base, int64_t grp,
                      int64_t stride, cudaStream_t st) {
    int64_t n = rows * KB;
    int blocks = (int)((n + 255) / 256);
    q8_repack_kernel<<<blocks, 256, 0, st>>>(src, rows, KB, w.qs, reinterpret_cast<uint16_t*>(w.d), base, grp, stride);
}

void launch_q8_dequant_raw(const uint8_t* src, int64_t n_blocks, float* out, cudaStream_t st) {
    int64_t n = n_blocks * 32;
    q8_dequant_raw_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(src, n_blocks, out);
}

void launch_q8p_dequant(const Q8Weight& w, int64_t rows, float* out, cudaStream_t st) {
    int64_t n = rows * (int64_t)w.KB * 32;
    q8p_dequant_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(w.qs, reinterpret_cast<const uint16_t*>(w.d),
                                                                      w.KB, rows, out);
}

void launch_embed(const Q8Weight& w, int vocab, const int32_t* tokens, int batch, float* x, int ldx, cudaStream_t st) {
    embed_kernel<<<batch, 256, 0, st>>>(w.qs, reinterpret_cast<const uint16_t*>(w.d), w.KB, vocab, tokens, x, ldx);
}

}  // namespace ab2
