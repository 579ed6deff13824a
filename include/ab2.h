/* ab2.h -- C ABI of the B200 decode backend for the Qwen3.5 hybrid (Gated DeltaNet + GQA)
 * model with GGUF Q8_0 weights.
 *
 * This is the drop-in boundary for the reference's decode path (thebasedcapital/ane-infer,
 * crates/engine Metal backend + its CPU twin). Every entry point below names the reference
 * interface it replaces, as path:line inside that project. All functions return 0 on success
 * or a negative AB2_ERR_* code; the message of the last failure on the calling thread is
 * available from ab2_last_error(). No entry point aborts the process.
 *
 * Threading: one ab2_ctx per GPU; a context is not thread-safe, distinct contexts may be
 * driven from distinct host threads. Host-buffer calls are synchronous at return.
 */
#ifndef AB2_H
#define AB2_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AB2_OK 0
#define AB2_ERR_ARG (-1)      /* bad argument (null pointer, index out of range)          */
#define AB2_ERR_FORMAT (-2)   /* malformed or truncated GGUF, missing tensor or key        */
#define AB2_ERR_SHAPE (-3)    /* tensor shapes inconsistent or not supported               */
#define AB2_ERR_OOM (-4)      /* device or pinned host allocation failed                   */
#define AB2_ERR_CUDA (-5)     /* a CUDA call failed                                        */
#define AB2_ERR_CAPACITY (-6) /* batch larger than max_batch, or context full              */
#define AB2_ERR_DEVICE (-7)   /* no usable CUDA device                                     */

typedef struct ab2_ctx ab2_ctx;
typedef struct ab2_q8 ab2_q8;

typedef struct ab2_options {
    int32_t kv_bf16;   /* 1 (default): bf16 KV cache; 0: f32 KV cache like the reference  */
    int32_t rope_dims; /* rotated dims per head; 0 (default) = head_dim, the reference's  */
    /* Steps of at most this many sequences multiply the Q8_0 weights exactly (mma.sync, the
     * weights q*d kept exact in f32 sums, activations as an f16 hi/lo pair); larger steps use
     * the tcgen05 path, whose operands are rounded once to f16. 0 (default) = 1: one sequence
     * exact, every batched step on the tensor-core path. -1: no exact path, one sequence on
     * the tensor-core path too (lower latency, the batched path's declared rounding). At most
     * 64. ab2_prefill runs its prompt in 64-row steps, so a prefill is exact only with 64 here.
     * Unless it is 64, the context holds the tensor-core copy of the weights too. */
    int32_t exact_max_batch;
    int32_t reserved[5];
} ab2_options;

typedef struct ab2_config {
    int64_t dim, ffn, n_layers, vocab;
    int64_t n_heads, n_kv_heads, head_dim; /* GQA layers                                 */
    int64_t dn_heads, dn_state, conv_kernel; /* Gated DeltaNet layers                     */
    int64_t n_dn, n_attn;
    int64_t max_batch, max_ctx;              /* 0 from ab2_gguf_inspect                   */
    int64_t context_length;                  /* GGUF qwen35.context_length (0 if absent)  */
    float rope_base, eps;
    int32_t kv_bf16, rope_dims;
} ab2_config;

/* Message of the last failure on this thread ("" if none). */
const char* ab2_last_error(void);

/* Host-only: parse GGUF bytes and derive the model configuration.
 * Replaces GgufFile::parse (crates/gguf/src/parser.rs:299) + Qwen35Config::from_gguf
 * (crates/engine/src/model.rs:70). Needs no GPU. */
int ab2_gguf_inspect(const uint8_t* gguf, uint64_t len, ab2_config* out);

/* Load a qwen35 GGUF onto `device`: repack Q8_0 weights, allocate per-slot recurrent state,
 * conv state and KV cache for max_batch sequences of up to max_ctx tokens.
 * Replaces GpuContext::new (crates/engine/src/metal_graph.rs:79), upload_model_weights
 * (crates/engine/src/gpu_decode.rs:152), GpuLayerScratch::new and GpuConstantPool::new
 * (crates/engine/src/gpu_full_decode.rs:175, :104) and HybridCache::new
 * (crates/engine/src/deltanet_cache.rs:76). opt may be NULL. */
int ab2_create(const uint8_t* gguf, uint64_t len, int device, int max_batch, int max_ctx,
               const ab2_options* opt, ab2_ctx** out);
void ab2_destroy(ab2_ctx* ctx);
int ab2_get_config(ab2_ctx* ctx, ab2_config* out);

/* ---- head-parallel split over tp_world GPUs (one process or thread per GPU) ---------- *
 * No reference counterpart: the reference runs one device (README.md:258). Each rank holds
 * every weight, runs the DeltaNet heads [rank*H/W, (rank+1)*H/W) and the kv heads
 * [rank*Hkv/W, (rank+1)*Hkv/W) with their query heads, and keeps only those heads'
 * recurrent state and KV cache; after each split mixer the ranks all-gather its output over
 * NCCL (loaded at run time: libnccl.so.2, or the file AB2_NCCL_LIB names). A mixer kind whose
 * heads do not divide over the ranks, or attention with an f32 cache, runs replicated on
 * every rank. Every rank makes the same calls with the same arguments (tokens, slots,
 * positions) in the same order; each returns the full logits / next tokens.
 * State I/O (ab2_{set,get}_dn_state, ab2_{set,get}_kv) keeps its full-size host arrays and
 * moves the rank's own heads' part of them; ab2_seed_state seeds each rank's part of what
 * one GPU seeds. */
#define AB2_TP_ID_BYTES 128
/* A fresh id for one split (ncclGetUniqueId); made on one rank and passed to all. */
int ab2_tp_unique_id(uint8_t* id, uint64_t id_len);
/* ab2_create for rank tp_rank of tp_world (1..8); returns once all ranks have joined.
 * tp_world = 1 is ab2_create (id may be NULL). A rank that never joins (it failed before
 * this call) leaves the others waiting in NCCL's bootstrap on the host, with no device work
 * pending: bound the call with a timeout of the caller's own. */
int ab2_create_tp(const uint8_t* gguf, uint64_t len, int device, int max_batch, int max_ctx,
                  const ab2_options* opt, int tp_rank, int tp_world, const uint8_t* tp_id,
                  uint64_t id_len, ab2_ctx** out);
/* out = {tp_rank, tp_world, first DeltaNet head, DeltaNet heads, first kv head, kv heads}. */
int ab2_get_tp(ab2_ctx* ctx, int32_t out[6]);
/* 1 if `layer` is a Gated DeltaNet layer (GgufFile::is_deltanet_layer, parser.rs:483). */
int ab2_layer_is_deltanet(ab2_ctx* ctx, int layer);

/* ---- per-slot state (host buffers). Layer indices are model layer indices. ---------- *
 * These calls are synchronous, but they do not wait for steps queued with
 * ab2_decode_step_device on other streams: call ab2_sync (or synchronise those streams)
 * first. */
/* Zero a slot's states and set its position to 0 (HybridCache::new for one sequence). */
int ab2_reset_slot(ab2_ctx* ctx, int slot);
/* Position of the next token of a slot (HybridCache::pos, deltanet_cache.rs:72). */
int ab2_set_pos(ab2_ctx* ctx, int slot, int64_t pos);
int ab2_get_pos(ab2_ctx* ctx, int slot, int64_t* pos);
/* Recurrent state [H][dk][dv] and conv state [3*dim][K] of a DeltaNet layer
 * (DeltaNetLayerState, deltanet_cache.rs:5-65). Either pointer may be NULL. */
int ab2_set_dn_state(ab2_ctx* ctx, int layer, int slot, const float* rec, const float* conv);
int ab2_get_dn_state(ab2_ctx* ctx, int layer, int slot, float* rec, float* conv);
/* K and V caches of an attention layer as f32 [n_kv][n_tokens][head_dim] for positions
 * [0, n_tokens) (LayerKvCache::write_range / key_head, kv_cache.rs:43-67); values are
 * rounded to bf16 when the cache is bf16. */
int ab2_set_kv(ab2_ctx* ctx, int layer, int slot, const float* k, const float* v, int64_t n_tokens);
int ab2_get_kv(ab2_ctx* ctx, int layer, int slot, float* k, float* v, int64_t n_tokens);
/* Fill slots [0, n_slots) with seeded synthetic state on the device: recurrent state
 * N(0, dn_std), conv state N(0, conv_std), K/V for positions [0, n_tokens) N(0, kv_std)
 * (bf16-representable), and set each position to n_tokens. Benchmark helper for the
 * prefilled-cache workload; the reference gets these from its prefill. */
int ab2_seed_state(ab2_ctx* ctx, uint64_t seed, int n_slots, int64_t n_tokens, float dn_std,
                   float conv_std, float kv_std);

/* ---- decode ------------------------------------------------------------------------- */
/* One greedy decode step for slots [0, batch): token ids in, logits and/or argmax ids out,
 * each slot's position advanced by one. Host buffers; synchronous.
 * Batched replacement of encode_full_token_gpu (crates/engine/src/gpu_full_decode.rs:221)
 * and of qwen35_forward_token + greedy_sample (crates/cli/src/main.rs:953, :1767).
 * logits: [batch][vocab] or NULL; next_tokens: [batch] or NULL. Token ids outside
 * [0, vocab) are rejected with AB2_ERR_ARG before any work is queued. */
int ab2_decode_step(ab2_ctx* ctx, const int32_t* tokens, int batch, float* logits, int32_t* next_tokens);
/* Prefill: run n prompt tokens of one slot through the model from the slot's position on,
 * updating its recurrent, conv and KV state and advancing its position by n; the last
 * token's logits [vocab] and argmax come back (either pointer may be NULL). Host buffers;
 * synchronous. Replaces the reference's prompt loop over qwen35_forward_token
 * (crates/cli/src/main.rs:358-362) and ane_prefill_tokens (main.rs:1168). The tokens go
 * through in steps of 128 (of 64 when exact_max_batch is 64): every projection as one GEMM
 * over the step's rows, the DeltaNet recurrence in its chunkwise form over 64 tokens at a
 * time (the plan of HANDOVER.md:67-72), each token's attention over the slot's cache. Needs
 * the bf16 KV cache and conv kernel 4. Ids outside [0, vocab) and prompts that do not fit in
 * max_ctx are rejected before any work is queued. */
int ab2_prefill(ab2_ctx* ctx, int slot, const int32_t* tokens, int64_t n, float* logits, int32_t* next_token);
/* Same with device buffers, enqueued on `stream` (a cudaStream_t; NULL = the context's own
 * stream) without synchronising. tokens_dev may alias next_dev of the previous step. The
 * ids are not checked on the host here: an id outside [0, vocab) embeds as a zero vector. */
int ab2_decode_step_device(ab2_ctx* ctx, const int32_t* tokens_dev, int batch, float* logits_dev,
                           int32_t* next_dev, void* stream);
/* Wait for all work of the context (including ab2_decode_step_device calls) and report a
 * tensor-core pipeline timeout recorded by the device, if any. No reference counterpart:
 * the Metal path waits with wait_until_completed (crates/engine/src/gpu_full_decode.rs:1031). */
int ab2_sync(ab2_ctx* ctx);
/* Kernel launches per decode step of `batch` sequences (for launch accounting). */
int ab2_launches_per_step(ab2_ctx* ctx, int batch, int64_t* out);
/* Per-kernel-class device time: enable recording CUDA events around every launch
 * (classes: 0 attention, 1 deltanet, 2 q8 gemm, 3 other), read and reset the sums. */
int ab2_profile(ab2_ctx* ctx, int enable);
int ab2_profile_read(ab2_ctx* ctx, double ms[4], int64_t launches[4]);
/* Whole-step CUDA graphs: when enabled, a decode step is captured once per launch plan
 * (batch, attention split plan, token/logit/next-token buffers; up to 4 plans cached) and
 * replayed with one graph launch instead of ~200 kernel launches: the same kernels with
 * the same arguments as the stream form. Replaces the per-token command-buffer encoding of
 * encode_full_token_gpu (crates/engine/src/gpu_full_decode.rs:221-1044). Profiling
 * (ab2_profile) runs the stream form. */
int ab2_step_graph(ab2_ctx* ctx, int enable);
/* Number of step graphs captured so far (a capture happens when no cached plan matches). */
int ab2_step_graph_captures(ab2_ctx* ctx, int64_t* out);

/* ---- per-layer parity entry points (one slot, host buffers) ------------------------- */
/* Mixer of one layer on an already RMS-normed hidden vector x[dim] -> out[dim]:
 * deltanet_decode_step (crates/engine/src/deltanet.rs:429) for DeltaNet layers,
 * full_attn_decode_step (deltanet.rs:541) at the slot's position for attention layers.
 * Updates the slot's state; does not advance its position. */
int ab2_mixer_layer(ab2_ctx* ctx, int layer, int slot, const float* x, float* out);
/* SwiGLU FFN of one layer: ffn_forward (crates/cli/src/main.rs:1115). */
int ab2_ffn_layer(ab2_ctx* ctx, int layer, const float* x, float* out);

/* ---- op-level entry points (device pointers) ---------------------------------------- */
/* Upload m x n Q8_0 blocks (GGUF layout, host memory) as a packed device tensor.
 * Replaces Q8Tensor::from_raw (crates/engine/src/q8_gemv.rs:33) + upload_quant_weights
 * (crates/engine/src/metal_graph.rs:208). */
int ab2_q8_create(const uint8_t* blocks, int64_t m, int64_t n, int device, ab2_q8** out);
void ab2_q8_destroy(ab2_q8* w);
/* y[b][m] = W x[b] for b < batch (f32 device buffers [batch][n] -> [batch][m]).
 * Replaces q8_gemv (crates/engine/src/q8_gemv.rs:130) and encode_gemv_prealloc
 * (crates/engine/src/gpu_full_decode.rs:1048). stream may be NULL (legacy default). */
int ab2_q8_gemv(ab2_q8* w, const float* x, int batch, float* y, void* stream);
/* batch is 1..128. Batches of 9 or more run on the tcgen05 path, whose f16 weights are q*d
 * rounded once (relative error <= 2^-11 per weight); smaller batches keep the weights exact. */
/* ab2_q8_gemv for batch 1..8 that allocates nothing: no reference counterpart. For callers
 * that cannot call cudaMalloc (device memory already carved up by their own pool, or a
 * thread where cudaMalloc's implicit synchronisation would stall other streams). Its
 * activation buffer, split-K workspace and tickets live in one fixed 4 MiB device array of
 * the library (16 KiB of it for tickets); a shape whose scratch does not fit, or a batch
 * above 8, returns AB2_ERR_CAPACITY with the sizes in the message. The first call on a
 * device looks up that array's address (cudaGetSymbolAddress) and should come before any
 * stream capture. All calls on a device share the one array: calls that can overlap on the
 * device (different streams or host threads) race, so serialise them. Same results as
 * ab2_q8_gemv at the same batch. */
int ab2_q8_gemv_noalloc(ab2_q8* w, const float* x, int batch, float* y, void* stream);
/* Synchronise the current device and return (then clear) the error word of the op-level
 * tensor-core calls: 0, or the code of a pipeline wait that timed out. */
int ab2_op_error(uint32_t* code);
/* Test hook; no counterpart in the reference. Arms the next launch (from this process, on a
 * stream that is not capturing) of one pipelined kernel to leave its asynchronous copy number
 * copy_index (counted per CTA from 0) unissued and to give each of its waits wait_ns
 * nanoseconds instead of 2 s. The waits on that copy then expire without any fault: the
 * kernel sets its error bit (tcgen05 GEMM 128 with others of its pipeline, attention 4096,
 * DeltaNet 1024), waits for the copies it did issue, frees its tensor memory and returns; that
 * launch's results are invalid. The error is reported as any other: ab2_op_error for the
 * op-level calls, AB2_ERR_CUDA from the context's step or ab2_sync. which: 1 the tcgen05
 * GEMM's weight copy, 2 the tensor-core attention's K/V tile copy, 3 the DeltaNet state copy.
 * wait_ns = 0 disarms; otherwise at least 1000. Nothing is withheld unless this is called. */
int ab2_debug_arm_wait_timeout(int which, int copy_index, uint32_t wait_ns);
/* The packed tensor expanded back to f32 [m][n] (exact). */
int ab2_q8_unpack(ab2_q8* w, float* out, void* stream);
/* n_blocks raw Q8_0 blocks (device) -> f32 (device), bit-exact with dequant_q8_0_block
 * (crates/gguf/src/dequant.rs:29). */
int ab2_q8_dequant(const uint8_t* blocks, int64_t n_blocks, float* out, void* stream);
/* Gated delta-rule step for B x H heads (the recurrence of deltanet_decode_step,
 * crates/engine/src/deltanet.rs:485-512): S [B][H][dk][dv] f32 updated in place;
 * q, k [B][H][dk] and v [B][H][dv] as bf16 bits; beta, decay [B][H] f32; o [B][H][dv] f32.
 * dk = dv = 128. */
int ab2_gated_delta(float* S, const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* beta,
                    const float* decay, int B, int H, int dk, int dv, float* o, void* stream);
/* GQA decode attention for B sequences (full_attn_decode_step without its projections,
 * crates/engine/src/deltanet.rs:575-669): proj [B][Hq*2*hd + 2*Hkv*hd] holds per-head
 * [q | gate] then k then v as the attn_q/attn_k/attn_v projections produce them;
 * caches [B][Hkv][cap][hd] (bf16 bits if kv_bf16 else f32); pos [B] int32 (device) is the
 * position of the new token, which is appended. q_norm/k_norm may be NULL (no norm).
 * RoPE on adjacent pairs of the first rope_dims dims. out [B][Hq*hd] f32.
 * max_pos (< cap, checked on the host) bounds the positions: the kernels check
 * 0 <= pos[b] <= max_pos on the device, skip a sequence outside that range (nothing is
 * appended or read for it, its output is left unwritten) and set bit 8192 of the word
 * ab2_op_error returns. */
int ab2_attn_decode(const float* proj, void* k_cache, void* v_cache, int64_t cap, const int32_t* pos, int B,
                    int Hq, int Hkv, int hd, int kv_bf16, const float* q_norm, const float* k_norm,
                    float rope_base, int rope_dims, int max_pos, float* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* AB2_H */
