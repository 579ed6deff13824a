// kernels.h -- host-side declarations of the device buffers and kernel launchers.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace ab2 {

// Launch with programmatic stream serialization so the kernel can start (and prefetch what
// does not depend on its predecessor) while the previous kernel on the stream finishes.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// The bounded waits of the pipelined kernels (tcgen05 GEMM, tensor-core attention, DeltaNet):
// each mbarrier wait gives up after wait_ns (2 s) and the kernel reports an error bit, drains
// its copies in flight and returns. A test can arm one launch to withhold its asynchronous
// copy number `withhold` (counted per CTA) with a short wait_ns, so that those waits expire
// without any fault (ab2_debug_arm_wait_timeout); otherwise nothing is withheld.
struct WaitTest {
    uint32_t wait_ns = 2000000000u;
    int withhold = -1;
};
enum { kWaitTestGemm = 1, kWaitTestAttention = 2, kWaitTestDeltaNet = 3 };
// the armed setting for the next launch of kernel family `which` on a stream that is not
// capturing (then disarmed), else the production setting
WaitTest take_wait_test(int which, cudaStream_t st);

// A Q8_0 weight on the device, in one or both packed layouts:
//   q8p (qs, d): mma.sync fragment order, used for batches <= 8 (exact weights);
//   q8u (qt):    128-row x 64-column tiles for the tcgen05 GEMM, used for larger batches:
//                [4 chunks][128 rows][16 B] offset-binary int8 + [128 rows][2] f16 d per tile,
//                stored as [MT/2 row-tile pairs][KT][2 tiles] so that one K tile of a 256-row
//                pair is one contiguous 17 KB block (MT rounded up to even, padding zero).
constexpr int kUTileRows = 128;
constexpr int kUTileBytes = 4 * kUTileRows * 16 + kUTileRows * 4;  // 8704
struct Q8Weight {
    uint8_t* qs = nullptr;  // [M16][KB][32][16]
    uint8_t* d = nullptr;   // [M16][KB][8] x (f16, f16)
    uint8_t* qt = nullptr;  // [MT][KT][kUTileBytes]
    int64_t M = 0;          // logical rows
    int M16 = 0;            // ceil(M/16)
    int KB = 0;             // K / 32
    int MT = 0;             // ceil(M/128)
    int KT = 0;             // ceil(K/64)
    size_t qs_bytes() const { return (size_t)M16 * KB * 512; }
    size_t d_bytes() const { return (size_t)M16 * KB * 32; }
    size_t qt_bytes() const { return (size_t)(MT + 1) / 2 * 2 * KT * kUTileBytes; }
};

// EPI_ADD: y += Wx with reductions into a y the caller zeroed (the tcgen05 path runs the
// SwiGLU gate/up projection this way, K-split, and the down projection applies silu(g)*u)
enum EpiMode { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_ADD = 3 };

struct GemmEpi {
    int mode = EPI_STORE;
    float* y = nullptr;  // STORE / RESID: y[b*ldy + row]; SWIGLU: optional f32 copy of h
    int ldy = 0;
    int m_out = 0;       // valid output rows (M, or ffn for SWIGLU)
    ActOut out{};        // SWIGLU: activations of the next GEMM
    const void* pf = nullptr;  // optional: the next GEMM's weights, prefetched into L2 by this launch
    int64_t pf_bytes = 0;
    WaitTest wt{};             // wait limit and the test hook (tcgen05 path)
};

// the batch above which the tcgen05 path (q8t weights, x16 activations) is used
constexpr int kUmmaMinBatch = 9;

// q8.cu
int gemm_nsplit(int M16, int KB, int num_sms);
int gemm_grid_x(int M16);
size_t gemm_ws_floats(int M16, int KB, int batch, int num_sms);
void launch_q8_gemm(const Q8Weight& w, const uint8_t* xf, int batch, float* ws, unsigned* tickets,
                    const GemmEpi& ep, int num_sms, cudaStream_t st);
void launch_q8_repack(const uint8_t* src, int64_t rows, int KB, Q8Weight& w, int64_t base, int64_t grp,
                      int64_t stride, cudaStream_t st);
void launch_q8_dequant_raw(const uint8_t* src, int64_t n_blocks, float* out, cudaStream_t st);
void launch_q8p_dequant(const Q8Weight& w, int64_t rows, float* out, cudaStream_t st);
void launch_embed(const Q8Weight& w, int vocab, const int32_t* tokens, int batch, float* x, int ldx, cudaStream_t st);

// q8_umma.cu
// How the tcgen05 GEMM cuts a weight into work units: main_units units (row-tile pair, K
// split) over the first pairs - tail_pairs pairs with ks splits each, then the last
// tail_pairs pairs cut into ks_tail K pieces each. A launch with more whole-pair units than
// CTAs would otherwise leave its last round to a few CTAs (the 2B lm_head: 594 pairs on 148
// SMs); those last pairs are split instead. A unit of a split pair adds its partial sums into
// y, so for a STORE the output rows from zero_row0 on must start at zero (zero_row0 = M: none).
struct UmmaPlan {
    int pairs = 0, ks = 1, kper = 0, main_units = 0, tail_pairs = 0, ks_tail = 1, kper_tail = 0, units = 0;
    int64_t zero_row0 = 0;
};
UmmaPlan umma_plan(int MT, int KT, int64_t M, int num_sms);
// K splits of the main units
int umma_nsplit(int MT, int KT, int mode, int num_sms);
void launch_q8t_repack(const uint8_t* src, int64_t rows, int KB, Q8Weight& w, int64_t base, int64_t grp,
                       int64_t stride, cudaStream_t st);
// batch <= 128 (x16 holds x16_npad(batch) rows). h2 (optional): the activations are
// silu(g) * u of this f32 gate/up scratch ([batch][h2_ld], gate and up interleaved per 64
// columns) instead of the x16 image
int launch_q8_umma(const Q8Weight& w, const uint8_t* x16, int batch, unsigned* err, const GemmEpi& ep, int num_sms,
                   cudaStream_t st, const float* h2 = nullptr, int h2_ld = 0);

// misc.cu
// zero (optional): rows [0, batch) x [0, zero_n) of zero_ptr (leading dim zero_ld) are cleared
void launch_rmsnorm_act(const float* x, int ldx, const float* w, int D, float eps, int batch, const ActOut& out,
                        cudaStream_t st, float* zero_ptr = nullptr, int zero_ld = 0, int zero_n = 0);
void launch_to_act(const float* x, int ldx, int K, int batch, const ActOut& out, cudaStream_t st);
// argmax under f32::total_cmp with ties going to the last index (greedy_sample,
// crates/cli/src/main.rs:1767-1785), split over nch chunks per row (part: [batch][nch] scratch)
constexpr int kArgmaxChunks = 32;
void launch_argmax2(const float* logits, int ld, int V, int batch, int32_t* out, int2* part, int nch,
                    cudaStream_t st);
void launch_pos_advance(int32_t* pos, int batch, cudaStream_t st);
// pos[i] = p0 + i for i < n (the positions of a prefill chunk's tokens)
void launch_pos_fill(int32_t* pos, int p0, int n, cudaStream_t st);
void launch_seed_f32(float* dst, int64_t n, uint64_t seed, uint64_t stream, float std, cudaStream_t st,
                     int64_t i0 = 0);
void launch_seed_kv(void* dst, bool bf16, int64_t rows, int cap, int64_t n_tokens, int hd, uint64_t seed,
                    uint64_t stream, float std, cudaStream_t st, int64_t i0 = 0);

// deltanet.cu
struct DnParams {
    const float* proj;   // [B][ldp]: qkv (3D) | gate (D) | beta_raw (H) | alpha_raw (H)
    int ldp;
    float* conv;         // [B][3D][K] (per-slot stride conv_stride floats)
    int64_t conv_stride;
    const float* conv_w; // [3D][K]
    int K;
    float* S;            // [B][H][128][128] (per-slot stride s_stride floats)
    int64_t s_stride;
    const float* ssm_a;  // [H]
    const float* dt_bias;
    const float* ssm_norm;  // [128]
    float eps;
    int D, H;            // H: heads this launch runs (the state buffer S holds exactly these)
    int h0 = 0;          // index in the model of its first head (head-parallel split; 0 otherwise)
    int H_all = 0;       // heads of the model (0: = H); the projection holds all of them
    ActOut out;          // activations of the ssm_out GEMM (K = D)
    float* o_out;        // optional f32 copy of the gated output [B][D]
    int row0 = 0;        // prefill: the first output row (of out and o_out) of this launch
    unsigned* err = nullptr;  // bit 1024 set when a state copy did not arrive in time
    const void* pf = nullptr;  // optional: weights of the following GEMM, prefetched into L2
    int64_t pf_bytes = 0;
    WaitTest wt{};             // wait limit and the test hook
};
void launch_deltanet(const DnParams& p, int batch, cudaStream_t st);
// dn_prefill.cu: the DeltaNet mixer of `tokens` (<= kPrefillChunk) consecutive tokens of one
// sequence (proj rows are tokens, out rows are row0 + token; S and conv point at that
// sequence's state); chunked form of the recurrence. Returns 0, or -1 for an unsupported
// shape, -2 for a launch failure.
constexpr int kPrefillChunk = 64;
// tokens per prefill step (the rows of its GEMMs): kPrefillChunk on the exact mma.sync path,
// kPrefillRowsTc on the tcgen05 path (N = 128), whose DeltaNet mixer runs as two launches
constexpr int kPrefillRowsTc = 128;
int launch_dn_prefill(const DnParams& p, int tokens, cudaStream_t st);
// recurrence core only (op API): q,k,v bf16 [B][H][128], beta/decay f32 [B][H], o f32 [B][H][128]
void launch_gated_delta(float* S, const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* beta,
                        const float* decay, int B, int H, float* o, cudaStream_t st);

// attention.cu
struct AttnParams {
    const float* proj;   // [B][ldp]: q_full (Hq*2*HD, per head [q | gate]) | k (Hkv*HD) | v (Hkv*HD)
    int ldp;
    const float* q_norm; // [HD] or null
    const float* k_norm; // [HD] or null
    const float2* rope;  // [rope_rows][rot/2] (cos, sin)
    int rot;
    void* kc;            // K cache [slots][Hkv][cap][HD] (float or bf16)
    void* vc;
    int64_t kv_slot_stride;  // elements between consecutive slots
    int cap;
    const int32_t* pos;  // [B] position of the new token per slot
    int Hq, Hkv;         // Hq: every query head (the projection layout); Hkv: the kv heads this launch runs
    int kvh0 = 0;        // index in the model of its first kv head (head-parallel split; 0 otherwise)
    // cache rows (tokens) between consecutive sequences in the tensor map of the bf16 cache:
    // -1 = Hkv * cap (each sequence its own slot); 0 = every query row reads one shared slot
    // (the prefill of one sequence's tokens, kv_slot_stride 0 likewise)
    int64_t seq_rows = -1;
    int Hkv_all = 0;     // kv heads of the model (0: = Hkv); the caches hold only this launch's Hkv
    int chunk;           // tokens per split
    // tensor-core decode kernel and its merge: > 0 = the balanced partition over this many CTAs
    // (every (sequence, kv head) pair's 64-token tiles laid end to end, CTA c taking an equal
    // run of them, so a pair cut by CTA boundaries becomes consecutive splits); 0 = splits of
    // `chunk` tokens dealt to the CTAs round-robin
    int sk_grid = 0;
    float* ws;           // split partials
    float* qprep = nullptr;  // tensor-core kernel: normed, rotated queries [B][Hkv][Hq/Hkv][HD]
    unsigned* tickets;   // [B*Hkv]
    ActOut out;          // activations of the wo GEMM (K = Hq*HD)
    float* o_out;        // optional f32 copy [B][Hq*HD]
    unsigned* err = nullptr;  // pipeline error word: bit 4096 when a wait of the tensor-core kernel timed out,
                              // bit kAttnErrPos when a sequence's position is outside [0, max_pos]
    // The largest position the launch plan covers (split count x chunk - 1, at most cap - 1).
    // Every kernel checks 0 <= pos[b] <= max_pos < cap before it appends at pos or reads the
    // rotation table at pos; a sequence outside that range is skipped and bit kAttnErrPos set.
    int max_pos = 0;
    WaitTest wt{};       // wait limit and the test hook (tensor-core kernel)
    const void* pf = nullptr;  // optional: weights of the following GEMM, prefetched into L2
    int64_t pf_bytes = 0;
};
constexpr unsigned kAttnErrPos = 8192;
__host__ __device__ inline bool attn_pos_ok(const AttnParams& p, int pos) {
    return pos >= 0 && pos <= p.max_pos && pos < p.cap;
}
// attn_mma.cu: tensor-core flash-decode over a bf16 cache read through two TMA tensor maps
// (K and V viewed as [rows][hd]); row_base = row of (first slot, kv head 0, token 0)
int make_kv_tensor_map(void* map_out /*128 bytes, 64-aligned*/, void* base, int64_t rows, int hd);
int attn_mma_chunk(int batch, int hkv, int max_len, int num_sms);
int attn_mma_nsplit_bound(int batch, int hkv, int cap, int num_sms);
int attn_mma_launches(int max_len, int chunk);
// core_begin / core_end (optional): events recorded around the attention kernel alone, not
// its query-prep and split-merge kernels (per-kernel profiling)
int launch_attention_mma(const void* tmk, const void* tmv, const AttnParams& p, int64_t row_base, int batch, int hd,
                         int max_len, int num_sms, cudaStream_t st, cudaEvent_t core_begin = nullptr,
                         cudaEvent_t core_end = nullptr);
int attn_nsplit(int max_len, int chunk);
// attn_prefill.cu: causal attention of a prefill step's B rows (consecutive positions of one
// sequence, all reading one cache slot: p.seq_rows = 0) on the tensor cores, in query blocks
// of 8 tokens x the kv head's query heads; enqueues the query prep, the kernel and, when the
// plan cuts the prefix into several splits, the merge. p.chunk from attn_prefill_chunk.
int attn_prefill_chunk(int rows, int hkv, int max_len, int num_sms);
int launch_attention_prefill(const void* tmk, const void* tmv, const AttnParams& p, int64_t row_base, int rows,
                             int hd, int max_len, int num_sms, cudaStream_t st, cudaEvent_t core_begin = nullptr,
                             cudaEvent_t core_end = nullptr);
// attn_mma.cu: the query/K/V prologue and the split merge of the tensor-core attention alone
int launch_attn_prep(const AttnParams& p, int batch, int hd, cudaStream_t st);
int launch_attn_merge(const AttnParams& p, int batch, int hd, cudaStream_t st);
int attn_chunk(int batch, int hkv, int max_len, int num_sms);
int attn_nsplit_bound(int batch, int hkv, int cap, int num_sms);
size_t attn_ws_floats(int batch, int hkv, int nsplit, int hd, int gq);
int launch_attention(const AttnParams& p, int batch, int hd, bool kv_bf16, int max_len, cudaStream_t st);

}  // namespace ab2
