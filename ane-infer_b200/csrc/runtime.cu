// runtime.cu -- host runtime and C ABI (include/ab2.h) of the B200 decode backend.
//
// Owns the GGUF parse, the Qwen3.5 hybrid configuration, the packed device weights, the
// per-slot recurrent / conv / KV state and the decode-step driver that launches the kernels
// of q8.cu, deltanet.cu, attention.cu and misc.cu on a context-owned stream.
#include <dlfcn.h>
#include <nccl.h>

#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/ab2.h"
#include "kernels.h"

#define AB2_API extern "C" __attribute__((visibility("default")))

using namespace ab2;

namespace {

thread_local std::string g_err;

int seterr(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

#define CK(call)                                                                                     \
    do {                                                                                             \
        cudaError_t e_ = (call);                                                                     \
        if (e_ != cudaSuccess) {                                                                     \
            return seterr(e_ == cudaErrorMemoryAllocation ? AB2_ERR_OOM : AB2_ERR_CUDA, "%s: %s (%s:%d)", \
                          #call, cudaGetErrorString(e_), __FILE__, __LINE__);                        \
        }                                                                                            \
    } while (0)

#define RET(expr)               \
    do {                        \
        int r_ = (expr);        \
        if (r_ != 0) return r_; \
    } while (0)

// Makes `dev` the calling thread's current device for the duration of an entry point and
// restores the caller's device on every return path: a host thread that drives another GPU
// (through torch, say) between calls into this library keeps its own current device.
struct DeviceGuard {
    int prev = -1;
    cudaError_t err = cudaSuccess;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        err = cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
    DeviceGuard(const DeviceGuard&) = delete;
    DeviceGuard& operator=(const DeviceGuard&) = delete;
};

// ------------------------------------------------------------------------------------- NCCL
// The head-parallel split all-gathers mixer outputs with NCCL, loaded at run time so that the
// library links without it: "libnccl.so.2" (a copy the host process has loaded already, such
// as PyTorch's, answers to that name first), or the file AB2_NCCL_LIB names.
struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    std::string why;  // empty when loaded
};

const NcclApi& nccl_api() {
    static NcclApi api = [] {
        NcclApi a;
        const char* env = getenv("AB2_NCCL_LIB");
        const char* name = env && *env ? env : "libnccl.so.2";
        void* h = dlopen(name, RTLD_NOW | RTLD_LOCAL);
        if (!h) {
            const char* e = dlerror();
            a.why = std::string("cannot load ") + name + ": " + (e ? e : "?");
            return a;
        }
        a.get_unique_id = (decltype(a.get_unique_id))dlsym(h, "ncclGetUniqueId");
        a.comm_init_rank = (decltype(a.comm_init_rank))dlsym(h, "ncclCommInitRank");
        a.comm_destroy = (decltype(a.comm_destroy))dlsym(h, "ncclCommDestroy");
        a.all_gather = (decltype(a.all_gather))dlsym(h, "ncclAllGather");
        a.error_string = (decltype(a.error_string))dlsym(h, "ncclGetErrorString");
        if (!a.get_unique_id || !a.comm_init_rank || !a.comm_destroy || !a.all_gather || !a.error_string)
            a.why = std::string(name) + " lacks an NCCL entry point";
        return a;
    }();
    return api;
}

#define NCK(call)                                                                                   \
    do {                                                                                            \
        ncclResult_t n_ = (call);                                                                   \
        if (n_ != ncclSuccess)                                                                      \
            return seterr(AB2_ERR_CUDA, "%s: %s", #call, nccl_api().error_string(n_));              \
    } while (0)

// ------------------------------------------------------------------------------------- GGUF
// Same byte format and accessor semantics as the reference parser
// (crates/gguf/src/parser.rs:17-347, :354-486), written for this runtime.
enum : uint32_t { G_U8 = 0, G_I8, G_U16, G_I16, G_U32, G_I32, G_F32, G_BOOL, G_STRING, G_ARRAY, G_U64, G_I64, G_F64 };

struct GValue {
    uint32_t type = 0;
    uint64_t u = 0;
    double f = 0.0;
    std::string s;
    uint64_t count = 0;  // arrays
};

struct GTensor {
    std::string name;
    std::vector<uint64_t> dims;
    uint32_t type = 0;
    uint64_t offset = 0;
    uint64_t nbytes = 0;
    const uint8_t* data = nullptr;  // inside the caller's buffer
};

struct Gguf {
    std::unordered_map<std::string, GValue> kv;
    std::unordered_map<std::string, GTensor> tensors;
    std::string arch;

    const GValue* get(const std::string& k) const {
        auto it = kv.find(k);
        return it == kv.end() ? nullptr : &it->second;
    }
    bool u32(const std::string& key, uint64_t* v) const {  // MetadataValue::as_u32: exact type only
        const GValue* g = get(arch + "." + key);
        if (!g || g->type != G_U32) return false;
        *v = g->u;
        return true;
    }
    bool f32(const std::string& key, float* v) const {
        const GValue* g = get(arch + "." + key);
        if (!g || g->type != G_F32) return false;
        *v = (float)g->f;
        return true;
    }
    const GTensor* tensor(const std::string& n) const {
        auto it = tensors.find(n);
        return it == tensors.end() ? nullptr : &it->second;
    }
};

struct Reader {
    const uint8_t* p;
    uint64_t n, o = 0;
    template <typename T>
    bool rd(T* v) {
        if (sizeof(T) > n - o) return false;
        memcpy(v, p + o, sizeof(T));
        o += sizeof(T);
        return true;
    }
    bool str(std::string* s) {
        uint64_t len;
        if (!rd(&len) || len > n - o) return false;
        if (s) s->assign((const char*)p + o, len);
        o += len;
        return true;
    }
    bool value(uint32_t t, GValue* v, int depth) {
        v->type = t;
        switch (t) {
            case G_U8: case G_I8: case G_BOOL: { uint8_t x; if (!rd(&x)) return false; v->u = x; return true; }
            case G_U16: case G_I16: { uint16_t x; if (!rd(&x)) return false; v->u = x; return true; }
            case G_U32: case G_I32: { uint32_t x; if (!rd(&x)) return false; v->u = x; return true; }
            case G_U64: case G_I64: { uint64_t x; if (!rd(&x)) return false; v->u = x; return true; }
            case G_F32: { float x; if (!rd(&x)) return false; v->f = x; return true; }
            case G_F64: { double x; if (!rd(&x)) return false; v->f = x; return true; }
            case G_STRING: return str(&v->s);
            case G_ARRAY: {
                uint32_t et;
                uint64_t cnt;
                if (depth > 3 || !rd(&et) || !rd(&cnt) || et > G_F64) return false;
                v->count = cnt;
                GValue tmp;
                for (uint64_t i = 0; i < cnt; i++) {
                    if (et == G_STRING) {
                        if (!str(nullptr)) return false;
                    } else if (!value(et, &tmp, depth + 1)) {
                        return false;
                    }
                }
                return true;
            }
            default: return false;
        }
    }
};

// block size / bytes per block of the GGML types the reference parser accepts (parser.rs:93-137)
bool ggml_sizes(uint32_t t, uint64_t* bs, uint64_t* bpb) {
    switch (t) {
        case 0: *bs = 1; *bpb = 4; return true;     // F32
        case 1: *bs = 1; *bpb = 2; return true;     // F16
        case 2: *bs = 32; *bpb = 18; return true;   // Q4_0
        case 3: *bs = 32; *bpb = 20; return true;   // Q4_1
        case 6: *bs = 32; *bpb = 22; return true;   // Q5_0
        case 7: *bs = 32; *bpb = 24; return true;   // Q5_1
        case 8: *bs = 32; *bpb = 34; return true;   // Q8_0
        case 12: *bs = 256; *bpb = 144; return true;  // Q4_K
        case 13: *bs = 256; *bpb = 176; return true;  // Q5_K
        case 14: *bs = 256; *bpb = 210; return true;  // Q6_K
        default: return false;
    }
}

int parse_gguf(const uint8_t* data, uint64_t len, Gguf* g) {
    if (!data) return seterr(AB2_ERR_ARG, "gguf: null buffer");
    Reader r{data, len};
    uint32_t magic, version;
    uint64_t nt, nkv;
    if (!r.rd(&magic)) return seterr(AB2_ERR_FORMAT, "gguf: truncated header");
    if (magic != 0x46554747u) return seterr(AB2_ERR_FORMAT, "gguf: bad magic 0x%08x", magic);
    if (!r.rd(&version) || !r.rd(&nt) || !r.rd(&nkv)) return seterr(AB2_ERR_FORMAT, "gguf: truncated header");
    if (version < 2 || version > 3) return seterr(AB2_ERR_FORMAT, "gguf: unsupported version %u", version);
    for (uint64_t i = 0; i < nkv; i++) {
        std::string key;
        uint32_t t;
        GValue v;
        if (!r.str(&key) || !r.rd(&t)) return seterr(AB2_ERR_FORMAT, "gguf: truncated metadata");
        if (!r.value(t, &v, 0)) return seterr(AB2_ERR_FORMAT, "gguf: bad metadata value for '%s'", key.c_str());
        g->kv[key] = std::move(v);
    }
    std::vector<GTensor> ts;
    for (uint64_t i = 0; i < nt; i++) {
        GTensor t;
        uint32_t nd;
        if (!r.str(&t.name) || !r.rd(&nd) || nd > 8) return seterr(AB2_ERR_FORMAT, "gguf: truncated tensor info");
        t.dims.resize(nd);
        for (auto& d : t.dims)
            if (!r.rd(&d)) return seterr(AB2_ERR_FORMAT, "gguf: truncated tensor info");
        if (!r.rd(&t.type) || !r.rd(&t.offset)) return seterr(AB2_ERR_FORMAT, "gguf: truncated tensor info");
        uint64_t bs, bpb, ne = 1;
        if (!ggml_sizes(t.type, &bs, &bpb)) return seterr(AB2_ERR_FORMAT, "gguf: unsupported GGML type %u (%s)", t.type, t.name.c_str());
        for (auto d : t.dims) ne *= d;
        t.nbytes = (ne + bs - 1) / bs * bpb;
        ts.push_back(std::move(t));
    }
    uint64_t align = 32;
    const GValue* a = g->get("general.alignment");
    if (a && a->type == G_U32) align = a->u;
    if (align == 0) return seterr(AB2_ERR_FORMAT, "gguf: zero alignment");
    const uint64_t base = (r.o + align - 1) / align * align;
    for (auto& t : ts) {
        if (t.offset > len || base > len - t.offset || t.nbytes > len - base - t.offset)
            return seterr(AB2_ERR_FORMAT, "gguf: tensor '%s' lies outside the file", t.name.c_str());
        t.data = data + base + t.offset;
        g->tensors[t.name] = t;
    }
    const GValue* ar = g->get("general.architecture");
    g->arch = (ar && ar->type == G_STRING) ? ar->s : std::string();
    return 0;
}

// ------------------------------------------------------------------------------------ config
struct Cfg {
    int64_t dim = 0, ffn = 0, n_layers = 0, vocab = 0, n_heads = 0, n_kv = 0, hd = 0;
    int64_t dn_heads = 0, dn_state = 0, conv_k = 0, ctx_len = 0;
    float rope_base = 1e4f, eps = 1e-6f;
    std::vector<uint8_t> is_dn;
    int64_t n_dn = 0, n_attn = 0;
};

// ModelConfig::from_gguf + Qwen35Config::from_gguf (crates/engine/src/model.rs:20-98) with
// the same defaults. The reference's 4096 context cap (model.rs:50) is not applied: the
// context capacity is the max_ctx given to ab2_create.
int derive_config(const Gguf& g, Cfg* c) {
    if (g.arch != "qwen35") return seterr(AB2_ERR_FORMAT, "architecture must be qwen35, got '%s'", g.arch.c_str());
    uint64_t v;
    if (!g.u32("embedding_length", &v)) return seterr(AB2_ERR_FORMAT, "missing embedding_length");
    c->dim = (int64_t)v;
    if (!g.u32("attention.head_count", &v)) return seterr(AB2_ERR_FORMAT, "missing head_count");
    c->n_heads = (int64_t)v;
    c->n_kv = g.u32("attention.head_count_kv", &v) ? (int64_t)v : c->n_heads;
    if (!g.u32("block_count", &v)) return seterr(AB2_ERR_FORMAT, "missing block_count");
    c->n_layers = (int64_t)v;
    if (!g.u32("feed_forward_length", &v)) return seterr(AB2_ERR_FORMAT, "missing feed_forward_length");
    c->ffn = (int64_t)v;
    const GValue* tok = g.get("tokenizer.ggml.tokens");
    c->vocab = (tok && tok->type == G_ARRAY) ? (int64_t)tok->count : 32000;
    if (!g.f32("rope.freq_base", &c->rope_base)) c->rope_base = 10000.0f;
    c->ctx_len = g.u32("context_length", &v) ? (int64_t)v : 0;
    if (!g.f32("attention.layer_norm_rms_epsilon", &c->eps)) c->eps = 1e-6f;
    if (c->n_heads <= 0 || c->dim <= 0 || c->n_layers <= 0) return seterr(AB2_ERR_SHAPE, "zero-sized model");
    c->hd = g.u32("attention.key_length", &v) ? (int64_t)v : c->dim / c->n_heads;
    c->dn_state = g.u32("ssm.state_size", &v) ? (int64_t)v : 128;
    c->conv_k = g.u32("ssm.conv_kernel", &v) ? (int64_t)v : 4;
    c->dn_heads = g.u32("ssm.group_count", &v) ? (int64_t)v : 16;
    c->is_dn.resize(c->n_layers);
    for (int64_t l = 0; l < c->n_layers; l++) {
        c->is_dn[l] = g.tensor("blk." + std::to_string(l) + ".ssm_a") != nullptr;
        (c->is_dn[l] ? c->n_dn : c->n_attn)++;
    }
    return 0;
}

void fill_config(const Cfg& c, ab2_config* o) {
    memset(o, 0, sizeof *o);
    o->dim = c.dim;
    o->ffn = c.ffn;
    o->n_layers = c.n_layers;
    o->vocab = c.vocab;
    o->n_heads = c.n_heads;
    o->n_kv_heads = c.n_kv;
    o->head_dim = c.hd;
    o->dn_heads = c.dn_heads;
    o->dn_state = c.dn_state;
    o->conv_kernel = c.conv_k;
    o->n_dn = c.n_dn;
    o->n_attn = c.n_attn;
    o->context_length = c.ctx_len;
    o->rope_base = c.rope_base;
    o->eps = c.eps;
}

// tensor lookups with shape checks (extract_tensor_raw / extract_tensor_f32, crates/gguf/src/to_ane.rs:12-44)
int find_q8(const Gguf& g, const std::string& name, int64_t m, int64_t n, const GTensor** out) {
    const GTensor* t = g.tensor(name);
    if (!t) return seterr(AB2_ERR_FORMAT, "tensor not found: %s", name.c_str());
    if (t->type != 8) return seterr(AB2_ERR_SHAPE, "%s: only Q8_0 projections are supported (type %u)", name.c_str(), t->type);
    int64_t ne0 = t->dims.empty() ? 0 : (int64_t)t->dims[0], ne1 = t->dims.size() > 1 ? (int64_t)t->dims[1] : 1;
    if (ne0 != n || ne1 != m)
        return seterr(AB2_ERR_SHAPE, "%s: shape %lldx%lld, expected %lldx%lld", name.c_str(), (long long)ne1,
                      (long long)ne0, (long long)m, (long long)n);
    if (n % 32) return seterr(AB2_ERR_SHAPE, "%s: n must be divisible by 32", name.c_str());
    *out = t;
    return 0;
}

int read_f32(const Gguf& g, const std::string& name, int64_t n, std::vector<float>* out) {
    const GTensor* t = g.tensor(name);
    if (!t) return seterr(AB2_ERR_FORMAT, "tensor not found: %s", name.c_str());
    int64_t ne = 1;
    for (auto d : t->dims) ne *= (int64_t)d;
    if (ne != n) return seterr(AB2_ERR_SHAPE, "%s: %lld elements, expected %lld", name.c_str(), (long long)ne, (long long)n);
    out->resize(n);
    if (t->type == 0) {
        memcpy(out->data(), t->data, n * 4);
    } else if (t->type == 1) {
        for (int64_t i = 0; i < n; i++) {
            uint16_t h;
            memcpy(&h, t->data + 2 * i, 2);
            uint32_t sign = (uint32_t)(h & 0x8000u) << 16, ex = (h >> 10) & 0x1f, man = h & 0x3ff, bits;
            if (ex == 0) {
                float f = (float)man * 5.9604644775390625e-08f;
                memcpy(&bits, &f, 4);
                bits |= sign;
            } else if (ex == 31) {
                bits = sign | 0x7f800000u | (man << 13);
            } else {
                bits = sign | ((ex + 112) << 23) | (man << 13);
            }
            memcpy(&(*out)[i], &bits, 4);
        }
    } else {
        return seterr(AB2_ERR_SHAPE, "%s: expected an F32 or F16 tensor", name.c_str());
    }
    return 0;
}

// an F32 or F16 tensor of n elements (the checks of read_f32, without reading)
int check_f32(const Gguf& g, const std::string& name, int64_t n) {
    const GTensor* t = g.tensor(name);
    if (!t) return seterr(AB2_ERR_FORMAT, "tensor not found: %s", name.c_str());
    int64_t ne = 1;
    for (auto d : t->dims) ne *= (int64_t)d;
    if (ne != n) return seterr(AB2_ERR_SHAPE, "%s: %lld elements, expected %lld", name.c_str(), (long long)ne, (long long)n);
    if (t->type != 0 && t->type != 1) return seterr(AB2_ERR_SHAPE, "%s: expected an F32 or F16 tensor", name.c_str());
    return 0;
}

// Everything the context build needs from the file, checked on the host before any device
// work: the shapes this build's kernels support (rot = rotated dims per head, 0 = head_dim)
// and the presence, type and shape of every tensor the build reads (tensor list of
// load_qwen35_weights, crates/cli/src/main.rs:1874-1994).
int validate_model(const Gguf& g, const Cfg& c, int rot) {
    const int64_t D = c.dim, F = c.ffn, H = c.dn_heads, hd = c.hd, Hq = c.n_heads, Hkv = c.n_kv;
    if (D % 128) return seterr(AB2_ERR_SHAPE, "embedding_length must be a multiple of 128");
    if (F % 32 || F % 8) return seterr(AB2_ERR_SHAPE, "feed_forward_length must be a multiple of 32");
    if (c.n_dn > 0) {
        if (c.dn_state != 128 || H <= 0 || D % H || D / H != 128)
            return seterr(AB2_ERR_SHAPE, "DeltaNet heads must have dk = dv = dim/heads = 128");
        if (c.conv_k < 1 || c.conv_k > 8) return seterr(AB2_ERR_SHAPE, "ssm.conv_kernel must be in [1, 8]");
    }
    if (c.n_attn > 0) {
        if (hd != 128 && hd != 256) return seterr(AB2_ERR_SHAPE, "attention head_dim must be 128 or 256");
        if (Hkv <= 0 || Hq % Hkv || Hq / Hkv != 4) return seterr(AB2_ERR_SHAPE, "GQA group must be 4 query heads per KV head");
        if ((Hq * hd) % 32) return seterr(AB2_ERR_SHAPE, "q dim must be a multiple of 32");
        const int r = rot > 0 ? rot : (int)hd;
        if (r % 2 || r > hd) return seterr(AB2_ERR_SHAPE, "rope_dims must be even and <= head_dim");
    }
    const GTensor* t;
    RET(find_q8(g, "token_embd.weight", c.vocab, D, &t));
    if (g.tensor("output.weight")) RET(find_q8(g, "output.weight", c.vocab, D, &t));
    RET(check_f32(g, "output_norm.weight", D));
    for (int64_t l = 0; l < c.n_layers; l++) {
        const std::string p = "blk." + std::to_string(l) + ".";
        RET(check_f32(g, p + "attn_norm.weight", D));
        RET(check_f32(g, p + "post_attention_norm.weight", D));
        if (c.is_dn[l]) {
            RET(find_q8(g, p + "attn_qkv.weight", 3 * D, D, &t));
            RET(find_q8(g, p + "attn_gate.weight", D, D, &t));
            RET(find_q8(g, p + "ssm_beta.weight", H, D, &t));
            RET(find_q8(g, p + "ssm_alpha.weight", H, D, &t));
            RET(find_q8(g, p + "ssm_out.weight", D, D, &t));
            RET(check_f32(g, p + "ssm_conv1d.weight", 3 * D * c.conv_k));
            RET(check_f32(g, p + "ssm_a", H));
            RET(check_f32(g, p + "ssm_dt.bias", H));
            RET(check_f32(g, p + "ssm_norm.weight", 128));
        } else {
            RET(find_q8(g, p + "attn_q.weight", 2 * Hq * hd, D, &t));
            RET(find_q8(g, p + "attn_k.weight", Hkv * hd, D, &t));
            RET(find_q8(g, p + "attn_v.weight", Hkv * hd, D, &t));
            RET(find_q8(g, p + "attn_output.weight", D, Hq * hd, &t));
            RET(check_f32(g, p + "attn_q_norm.weight", hd));
            RET(check_f32(g, p + "attn_k_norm.weight", hd));
        }
        RET(find_q8(g, p + "ffn_gate.weight", F, D, &t));
        RET(find_q8(g, p + "ffn_up.weight", F, D, &t));
        RET(find_q8(g, p + "ffn_down.weight", D, F, &t));
    }
    return 0;
}

// ------------------------------------------------------------------------------------- context
enum { PC_ATTN = 0, PC_DN = 1, PC_GEMM = 2, PC_OTHER = 3 };

struct Layer {
    bool dn = false;
    Q8Weight w_in, w_out, gate_up, down;
    float *attn_norm = nullptr, *post_norm = nullptr;
    float *conv_w = nullptr, *ssm_a = nullptr, *dt_bias = nullptr, *ssm_norm = nullptr;  // DeltaNet
    float *q_norm = nullptr, *k_norm = nullptr;                                          // GQA
    int local = 0;  // index among layers of the same kind
};

// One captured decode step (CUDA graph), replayable while everything its launches were
// planned from holds: the batch, the attention split plan (chunk length and split count,
// which follow the longest context) and the token / logit / next-token buffers.
struct StepGraph {
    int B = 0, chunk = 0, splits = 0;
    const int32_t* tok = nullptr;
    float* logits = nullptr;
    int32_t* next = nullptr;
    cudaGraphExec_t exec = nullptr;
    uint64_t last = 0;  // least recently used goes first
};
constexpr int kStepGraphs = 4;

struct Profile {
    bool on = false;
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> ev[4];
    size_t used[4] = {0, 0, 0, 0};
    double ms[4] = {0, 0, 0, 0};
    int64_t n[4] = {0, 0, 0, 0};
};

}  // namespace

struct ab2_ctx {
    int device = 0;
    int num_sms = 148;
    Cfg c;
    int max_batch = 0, cap = 0;
    bool kv_bf16 = true;
    int rot = 0;
    cudaStream_t stream = nullptr;
    std::vector<void*> allocs;
    std::vector<Layer> layers;
    Q8Weight embed, lm_head;
    float* final_norm = nullptr;
    // state
    float* dn_S = nullptr;      // [n_dn][max_batch][H][128][128]
    float* dn_conv = nullptr;   // [n_dn][max_batch][3D][K]
    void* kc = nullptr;         // [n_attn][max_batch][Hkv][cap][hd]
    void* vc = nullptr;
    int32_t* pos_d = nullptr;   // [max_batch]
    std::vector<int64_t> pos_h;
    int pf_rows = kPrefillChunk;  // tokens per prefill step (kPrefillRowsTc on the tcgen05 path)
    int32_t* pf_pos = nullptr;  // [pf_rows] positions of a prefill step's tokens
    int32_t* pf_tok = nullptr;  // [pf_rows] token ids of a prefill step
    int64_t s_stride = 0, conv_stride = 0, kv_slot = 0;
    // scratch, for `rows` = max(max_batch, pf_rows) rows (sequences of a step, or tokens of
    // a prefill step)
    int rows = 0;
    float* x = nullptr;         // residual stream [rows][D]
    float* proj = nullptr;      // [max_batch][ldp]
    int ldp = 0;
    uint8_t *xfa = nullptr, *xfb = nullptr;
    float* logits = nullptr;    // [max_batch][vocab]
    int32_t *tok_d = nullptr, *next_d = nullptr;
    int2* amax_part = nullptr;  // [max_batch][kArgmaxChunks] partial (key, index) of the argmax
    float* gws = nullptr;       // GEMM split-K partials
    unsigned* gtk = nullptr;    // GEMM tickets
    float* h2 = nullptr;        // tcgen05 path: f32 gate/up sums [max_batch][2*ffn]
    float* aws = nullptr;       // attention split partials
    float* aqp = nullptr;       // tensor-core attention: prepared queries [max_batch][Hq][hd]
    size_t aws_floats = 0;
    unsigned* atk = nullptr;    // attention tickets
    float2* rope = nullptr;     // [cap][rot/2]
    float* tmp_out = nullptr;   // [D] for per-layer entry points
    unsigned* err_d = nullptr;  // tensor-core pipeline error word (0 = ok)
    alignas(64) uint8_t tmap_k[128];  // TMA tensor maps over the bf16 K / V caches ([rows][hd])
    alignas(64) uint8_t tmap_v[128];
    int exact_max = 1;          // steps of at most this many sequences take the exact mma.sync GEMM
    // head-parallel split over tp_world GPUs: this rank runs DeltaNet heads [dn_h0, dn_h0 +
    // dn_hl) and kv heads [kv_h0, kv_h0 + kv_hl) and holds only their state; weights and the
    // rest of the step are replicated (tp_world = 1: one GPU runs every head)
    int tp_rank = 0, tp_world = 1;
    int dn_h0 = 0, dn_hl = 0, kv_h0 = 0, kv_hl = 0;
    bool dn_split = false, kv_split = false;  // which mixers are split (the others run replicated)
    ncclComm_t nccl = nullptr;  // the communicator of the split
    bool use_umma = false;      // some step has more rows than exact_max: q8t weights are packed too
    // pinned host staging
    int32_t *tok_h = nullptr, *next_h = nullptr;
    unsigned* err_h = nullptr;
    float* logits_h = nullptr;
    Profile prof;
    // whole-step CUDA graphs (off by default)
    bool graph_on = false;
    StepGraph graphs[kStepGraphs];
    uint64_t graph_tick = 0;
    int64_t graph_captures = 0;

    template <typename T>
    int dalloc(T** p, size_t bytes, bool zero = true) {
        void* q = nullptr;
        CK(cudaMalloc(&q, bytes ? bytes : 16));
        allocs.push_back(q);
        if (zero) CK(cudaMemsetAsync(q, 0, bytes ? bytes : 16, stream));
        *p = reinterpret_cast<T*>(q);
        return 0;
    }
};

namespace {

int upload_f32(ab2_ctx* x, const std::vector<float>& v, float** out) {
    RET(x->dalloc(out, v.size() * 4, false));
    CK(cudaMemcpyAsync(*out, v.data(), v.size() * 4, cudaMemcpyHostToDevice, x->stream));
    return 0;
}

constexpr int64_t kPlain = (int64_t)1 << 40;  // grp for plain concatenation

// A source tensor of a packed weight: its rows land at dst = base + (row/grp)*stride + row%grp.
// kind 0: plain concatenation at `base`; kind 1 / 2: gate / up rows of an interleaved SwiGLU
// pair (8-row groups in the q8p layout, 64-row groups in the q8u layout).
struct RepackSrc {
    const GTensor* t;
    int64_t rows, base;
    int kind = 0;
};

// upload Q8_0 tensors (same K) into one packed weight of M rows through a device staging buffer
int upload_q8(ab2_ctx* x, int64_t M, int64_t K, const std::vector<RepackSrc>& srcs, uint8_t* staging,
              Q8Weight* w) {
    w->M = M;
    w->M16 = (int)((M + 15) / 16);
    w->KB = (int)(K / 32);
    w->MT = (int)((M + kUTileRows - 1) / kUTileRows);
    w->KT = (int)((K + 63) / 64);
    RET(x->dalloc(&w->qs, w->qs_bytes(), true));
    RET(x->dalloc(&w->d, w->d_bytes(), true));
    if (x->use_umma) RET(x->dalloc(&w->qt, w->qt_bytes(), true));
    for (auto& s : srcs) {
        CK(cudaMemcpyAsync(staging, s.t->data, s.t->nbytes, cudaMemcpyHostToDevice, x->stream));
        const int64_t pg = s.kind ? 8 : kPlain, ps = s.kind ? 16 : 0, pb = s.kind == 2 ? 8 : s.base;
        launch_q8_repack(staging, s.rows, w->KB, *w, pb, pg, ps, x->stream);
        if (x->use_umma) {
            const int64_t tg = s.kind ? 64 : kPlain, ts = s.kind ? 128 : 0, tb = s.kind == 2 ? 64 : s.base;
            launch_q8t_repack(staging, s.rows, w->KB, *w, tb, tg, ts, x->stream);
        }
        CK(cudaGetLastError());
        // the staging buffer is reused by the next copy; the stream keeps the order
    }
    return 0;
}

// Head-parallel split over tp_world ranks: rank r runs DeltaNet heads [r*H/W, (r+1)*H/W) and
// kv heads [r*Hkv/W, (r+1)*Hkv/W) (with their query heads) and holds only their recurrent
// state and KV cache. A mixer kind whose heads do not divide over the ranks (or whose output
// slice would not be whole 64-column K tiles) runs replicated on every rank instead.
int plan_split(ab2_ctx* x) {
    const Cfg& c = x->c;
    const int W = x->tp_world, r = x->tp_rank;
    x->dn_split = c.n_dn > 0 && c.dn_heads % W == 0 && (c.dn_heads * 128 / W) % 64 == 0;
    x->kv_split = c.n_attn > 0 && x->kv_bf16 && c.n_kv % W == 0 && (c.n_heads * c.hd / W) % 64 == 0;
    if (!x->dn_split && !x->kv_split)
        return seterr(AB2_ERR_ARG, "head-parallel split: neither %lld DeltaNet heads nor %lld kv heads (bf16 cache) "
                      "divide over %d ranks", (long long)c.dn_heads, (long long)c.n_kv, W);
    x->dn_hl = (int)(x->dn_split ? c.dn_heads / W : c.dn_heads);
    x->dn_h0 = x->dn_split ? r * x->dn_hl : 0;
    x->kv_hl = (int)(x->kv_split ? c.n_kv / W : c.n_kv);
    x->kv_h0 = x->kv_split ? r * x->kv_hl : 0;
    return 0;
}

int build_context(ab2_ctx* x, const uint8_t* data, uint64_t len) {
    Gguf g;
    RET(parse_gguf(data, len, &g));
    RET(derive_config(g, &x->c));
    Cfg& c = x->c;
    const int64_t D = c.dim, F = c.ffn, H = c.dn_heads, hd = c.hd, Hq = c.n_heads, Hkv = c.n_kv;
    RET(validate_model(g, c, x->rot));
    x->rot = x->rot > 0 ? x->rot : (int)hd;
    if (x->tp_world > 1) RET(plan_split(x));

    // staging buffer for the largest Q8 tensor
    uint64_t maxb = 0;
    for (auto& kv : g.tensors)
        if (kv.second.type == 8) maxb = std::max(maxb, kv.second.nbytes);
    uint8_t* staging = nullptr;
    CK(cudaMalloc(&staging, maxb ? maxb : 16));

    int rc = 0;
    do {
        const GTensor *te, *tl;
        if ((rc = find_q8(g, "token_embd.weight", c.vocab, D, &te))) break;
        if ((rc = upload_q8(x, c.vocab, D, {{te, c.vocab, 0}}, staging, &x->embed))) break;
        if (g.tensor("output.weight")) {  // lm_head = output.weight or tied token_embd (main.rs:1903-1904)
            if ((rc = find_q8(g, "output.weight", c.vocab, D, &tl))) break;
            if ((rc = upload_q8(x, c.vocab, D, {{tl, c.vocab, 0}}, staging, &x->lm_head))) break;
        } else {
            x->lm_head = x->embed;
        }
        std::vector<float> fv;
        if ((rc = read_f32(g, "output_norm.weight", D, &fv)) || (rc = upload_f32(x, fv, &x->final_norm))) break;
        x->layers.resize(c.n_layers);
        int ndn = 0, nat = 0;
        for (int64_t l = 0; l < c.n_layers && !rc; l++) {
            Layer& L = x->layers[l];
            const std::string p = "blk." + std::to_string(l) + ".";
            L.dn = c.is_dn[l];
            L.local = L.dn ? ndn++ : nat++;
            if ((rc = read_f32(g, p + "attn_norm.weight", D, &fv)) || (rc = upload_f32(x, fv, &L.attn_norm))) break;
            if ((rc = read_f32(g, p + "post_attention_norm.weight", D, &fv)) || (rc = upload_f32(x, fv, &L.post_norm)))
                break;
            const GTensor *t0, *t1, *t2, *t3;
            if (L.dn) {
                // input projections concatenated: qkv (3D) | gate (D) | beta (H) | alpha (H)
                if ((rc = find_q8(g, p + "attn_qkv.weight", 3 * D, D, &t0)) ||
                    (rc = find_q8(g, p + "attn_gate.weight", D, D, &t1)) ||
                    (rc = find_q8(g, p + "ssm_beta.weight", H, D, &t2)) ||
                    (rc = find_q8(g, p + "ssm_alpha.weight", H, D, &t3)))
                    break;
                if ((rc = upload_q8(x, 4 * D + 2 * H, D,
                                    {{t0, 3 * D, 0}, {t1, D, 3 * D}, {t2, H, 4 * D},
                                     {t3, H, 4 * D + H}},
                                    staging, &L.w_in)))
                    break;
                if ((rc = find_q8(g, p + "ssm_out.weight", D, D, &t0)) ||
                    (rc = upload_q8(x, D, D, {{t0, D, 0}}, staging, &L.w_out)))
                    break;
                if ((rc = read_f32(g, p + "ssm_conv1d.weight", 3 * D * c.conv_k, &fv)) || (rc = upload_f32(x, fv, &L.conv_w)))
                    break;
                if ((rc = read_f32(g, p + "ssm_a", H, &fv)) || (rc = upload_f32(x, fv, &L.ssm_a))) break;
                if ((rc = read_f32(g, p + "ssm_dt.bias", H, &fv)) || (rc = upload_f32(x, fv, &L.dt_bias))) break;
                if ((rc = read_f32(g, p + "ssm_norm.weight", 128, &fv)) || (rc = upload_f32(x, fv, &L.ssm_norm))) break;
            } else {
                // q (per head [q | gate]) | k | v
                if ((rc = find_q8(g, p + "attn_q.weight", 2 * Hq * hd, D, &t0)) ||
                    (rc = find_q8(g, p + "attn_k.weight", Hkv * hd, D, &t1)) ||
                    (rc = find_q8(g, p + "attn_v.weight", Hkv * hd, D, &t2)))
                    break;
                if ((rc = upload_q8(x, 2 * Hq * hd + 2 * Hkv * hd, D,
                                    {{t0, 2 * Hq * hd, 0}, {t1, Hkv * hd, 2 * Hq * hd},
                                     {t2, Hkv * hd, 2 * Hq * hd + Hkv * hd}},
                                    staging, &L.w_in)))
                    break;
                if ((rc = find_q8(g, p + "attn_output.weight", D, Hq * hd, &t0)) ||
                    (rc = upload_q8(x, D, Hq * hd, {{t0, D, 0}}, staging, &L.w_out)))
                    break;
                if ((rc = read_f32(g, p + "attn_q_norm.weight", hd, &fv)) || (rc = upload_f32(x, fv, &L.q_norm))) break;
                if ((rc = read_f32(g, p + "attn_k_norm.weight", hd, &fv)) || (rc = upload_f32(x, fv, &L.k_norm))) break;
            }
            // FFN gate/up interleaved so that one tile holds the gate and up rows of the same
            // outputs (8 + 8 rows per m16 tile in q8p, 64 + 64 rows per 128-row tile in q8t)
            if ((rc = find_q8(g, p + "ffn_gate.weight", F, D, &t0)) || (rc = find_q8(g, p + "ffn_up.weight", F, D, &t1)) ||
                (rc = find_q8(g, p + "ffn_down.weight", D, F, &t2)))
                break;
            if ((rc = upload_q8(x, 2 * F, D, {{t0, F, 0, 1}, {t1, F, 0, 2}}, staging, &L.gate_up))) break;
            if ((rc = upload_q8(x, D, F, {{t2, D, 0}}, staging, &L.down))) break;
        }
    } while (0);
    cudaError_t se = cudaStreamSynchronize(x->stream);
    cudaFree(staging);
    if (rc) return rc;
    if (se != cudaSuccess) return seterr(AB2_ERR_CUDA, "weight upload: %s", cudaGetErrorString(se));

    // ---- per-slot state
    const int B = x->max_batch;
    if (x->tp_world <= 1) {
        x->dn_hl = (int)H;
        x->kv_hl = (int)Hkv;
    }
    x->s_stride = (int64_t)x->dn_hl * 128 * 128;  // this rank's heads only
    x->conv_stride = 3 * D * c.conv_k;             // every channel (a rank updates its heads')
    x->kv_slot = x->kv_hl * (int64_t)x->cap * hd;
    const size_t kvel = x->kv_bf16 ? 2 : 4;
    RET(x->dalloc(&x->dn_S, (size_t)std::max<int64_t>(c.n_dn, 1) * B * x->s_stride * 4));
    RET(x->dalloc(&x->dn_conv, (size_t)std::max<int64_t>(c.n_dn, 1) * B * x->conv_stride * 4));
    RET(x->dalloc(&x->kc, (size_t)std::max<int64_t>(c.n_attn, 1) * B * x->kv_slot * kvel));
    RET(x->dalloc(&x->vc, (size_t)std::max<int64_t>(c.n_attn, 1) * B * x->kv_slot * kvel));
    RET(x->dalloc(&x->pos_d, (size_t)B * 4));
    x->pos_h.assign(B, 0);

    // ---- scratch (rows: the sequences of a step or the tokens of a prefill chunk)
    const int R = std::max(B, x->pf_rows);
    x->rows = R;
    RET(x->dalloc(&x->pf_pos, (size_t)x->pf_rows * 4));
    RET(x->dalloc(&x->pf_tok, (size_t)x->pf_rows * 4));
    int64_t mproj = 0, maxk = D;
    for (auto& L : x->layers) mproj = std::max<int64_t>(mproj, L.w_in.M);
    maxk = std::max<int64_t>(maxk, F);
    maxk = std::max<int64_t>(maxk, Hq * hd);
    x->ldp = (int)((mproj + 3) / 4 * 4);
    RET(x->dalloc(&x->x, (size_t)R * D * 4));
    RET(x->dalloc(&x->proj, (size_t)R * x->ldp * 4));
    const size_t actb = std::max(xfrag_bytes((int)maxk, R), x16_bytes((int)maxk, R));
    RET(x->dalloc(&x->xfa, actb));
    RET(x->dalloc(&x->xfb, actb));
    RET(x->dalloc(&x->err_d, 16));
    RET(x->dalloc(&x->logits, (size_t)B * c.vocab * 4));
    RET(x->dalloc(&x->tok_d, (size_t)B * 4));
    RET(x->dalloc(&x->next_d, (size_t)B * 4));
    RET(x->dalloc(&x->amax_part, (size_t)B * kArgmaxChunks * sizeof(int2)));
    RET(x->dalloc(&x->tmp_out, (size_t)std::max<int64_t>(D, F) * 4));
    size_t gws = 0;
    int gtk = 1;
    auto acc_gemm = [&](const Q8Weight& w) {
        gws = std::max(gws, gemm_ws_floats(w.M16, w.KB, R, x->num_sms));
        gtk = std::max(gtk, gemm_grid_x(w.M16));
    };
    for (auto& L : x->layers) {
        acc_gemm(L.w_in);
        acc_gemm(L.w_out);
        acc_gemm(L.gate_up);
        acc_gemm(L.down);
    }
    acc_gemm(x->lm_head);
    RET(x->dalloc(&x->gws, gws * 4));
    RET(x->dalloc(&x->gtk, (size_t)gtk * 4));
    if (x->use_umma) RET(x->dalloc(&x->h2, (size_t)R * 2 * F * 4));
    if (c.n_attn > 0) {
        size_t aws = 0;
        const int hkl = x->kv_hl;
        for (int b = 1; b <= R; b++) {
            const int ns = x->kv_bf16 ? attn_mma_nsplit_bound(b, hkl, x->cap, x->num_sms)
                                      : attn_nsplit_bound(b, hkl, x->cap, x->num_sms);
            aws = std::max(aws, attn_ws_floats(b, hkl, ns, (int)hd, (int)(Hq / Hkv)));
        }
        x->aws_floats = aws;
        if (x->kv_bf16) {
            const int64_t rows = c.n_attn * (int64_t)B * x->kv_hl * x->cap;
            if (make_kv_tensor_map(x->tmap_k, x->kc, rows, (int)hd) || make_kv_tensor_map(x->tmap_v, x->vc, rows, (int)hd))
                return seterr(AB2_ERR_CUDA, "could not encode the TMA tensor maps of the KV cache");
        }
        RET(x->dalloc(&x->aws, aws * 4));
        if (x->kv_bf16) RET(x->dalloc(&x->aqp, (size_t)R * Hq * hd * 4));
        RET(x->dalloc(&x->atk, (size_t)R * x->kv_hl * 4));
        // RoPE (cos, sin) table built with the host libm exactly as the reference computes it:
        // freq = 1 / base^(i / rot) for even i, angle = pos * freq (deltanet.rs:600-623)
        const int hr = x->rot / 2;
        std::vector<float2> tab((size_t)x->cap * hr);
        for (int j = 0; j < hr; j++) {
            const float freq = 1.0f / powf(c.rope_base, (float)(2 * j) / (float)x->rot);
            for (int64_t p = 0; p < x->cap; p++) {
                const float val = (float)p * freq;
                tab[(size_t)p * hr + j] = make_float2(cosf(val), sinf(val));
            }
        }
        RET(x->dalloc(&x->rope, tab.size() * sizeof(float2), false));
        CK(cudaMemcpyAsync(x->rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice, x->stream));
    }
    CK(cudaMallocHost(&x->tok_h, (size_t)B * 4));
    CK(cudaMallocHost(&x->next_h, (size_t)B * 4));
    CK(cudaMallocHost(&x->err_h, 16));
    *x->err_h = 0;
    CK(cudaStreamSynchronize(x->stream));
    return 0;
}

// --------------------------------------------------------------------------------- profiling
// the next (begin, end) event pair of class cls while profiling, else (null, null)
std::pair<cudaEvent_t, cudaEvent_t> prof_pair(ab2_ctx* x, int cls) {
    if (!x->prof.on) return {nullptr, nullptr};
    auto& v = x->prof.ev[cls];
    size_t i = x->prof.used[cls]++;
    if (i >= v.size()) {
        cudaEvent_t a, b;
        cudaEventCreate(&a);
        cudaEventCreate(&b);
        v.push_back({a, b});
    }
    return v[i];
}

struct ProfScope {
    ab2_ctx* x;
    int cls;
    cudaStream_t st;
    cudaEvent_t stop = nullptr;
    ProfScope(ab2_ctx* x_, int cls_, cudaStream_t st_) : x(x_), cls(cls_), st(st_) {
        const auto e = prof_pair(x, cls);
        if (!e.first) return;
        cudaEventRecord(e.first, st);
        stop = e.second;
    }
    ~ProfScope() {
        if (stop) cudaEventRecord(stop, st);
    }
};

void prof_collect(ab2_ctx* x) {
    if (!x->prof.on) return;
    for (int c = 0; c < 4; c++) {
        for (size_t i = 0; i < x->prof.used[c]; i++) {
            float ms = 0;
            cudaEventElapsedTime(&ms, x->prof.ev[c][i].first, x->prof.ev[c][i].second);
            x->prof.ms[c] += ms;
            x->prof.n[c]++;
        }
        x->prof.used[c] = 0;
    }
}

// --------------------------------------------------------------------------------- the step
// steps of more than exact_max sequences run on the tcgen05 path
bool umma_for(const ab2_ctx* x, int B) { return x->use_umma && B > x->exact_max; }

ActOut act(const ab2_ctx* x, uint8_t* buf, int K, int B) { return act_out(buf, K, B, umma_for(x, B)); }

// L2 prefetch hint for a launch that precedes the tcgen05 GEMM on weight `w` (none on the
// mma.sync path, whose weights are in the other layout); at most `cap` bytes
void set_prefetch(ab2_ctx* x, int B, const Q8Weight* w, const void** pf, int64_t* pf_bytes,
                  int64_t cap = INT64_MAX) {
    *pf = nullptr;
    *pf_bytes = 0;
    if (!w || !w->qt || !umma_for(x, B)) return;
    *pf = w->qt;
    *pf_bytes = std::min<int64_t>((int64_t)w->qt_bytes(), cap);
}

// the part of a weight that one launch prefetches for its successor: L2 holds 126 MB, and the
// lm_head (330 MB for the 2B shape) streams from HBM anyway after its first stages
constexpr int64_t kPrefetchCap = 32ll << 20;

// rounds of DeltaNet items (one per CTA per round) whose states a batched step's DeltaNet
// input projection prefetches into L2
constexpr int kDnLeadRounds = 1;

// h2 (tcgen05 path only): take the activations as silu(g) * u of the gate/up scratch
int gemm(ab2_ctx* x, const Q8Weight& w, const uint8_t* xf, int B, const GemmEpi& ep, cudaStream_t st,
         const float* h2 = nullptr, int h2_ld = 0) {
    ProfScope ps(x, PC_GEMM, st);
    if (umma_for(x, B)) {
        if (launch_q8_umma(w, xf, B, x->err_d, ep, x->num_sms, st, h2, h2_ld))
            return seterr(AB2_ERR_CUDA, "tcgen05 GEMM launch failed: %s", cudaGetErrorString(cudaGetLastError()));
    } else {
        launch_q8_gemm(w, xf, B, x->gws, x->gtk, ep, x->num_sms, st);
    }
    return 0;
}

GemmEpi epi_store(float* y, int ldy, int64_t m) {
    GemmEpi e;
    e.mode = EPI_STORE;
    e.y = y;
    e.ldy = ldy;
    e.m_out = (int)m;
    return e;
}
GemmEpi epi_resid(float* y, int ldy, int64_t m) {
    GemmEpi e = epi_store(y, ldy, m);
    e.mode = EPI_RESID;
    return e;
}
GemmEpi epi_swiglu(const ActOut& out, int F) {
    GemmEpi e;
    e.mode = EPI_SWIGLU;
    e.m_out = F;
    e.out = out;
    return e;
}

// attention chunk length (tokens per split) of a step over B slots whose longest context is
// max_len; 0 without attention layers
int step_attn_chunk(const ab2_ctx* x, int B, int max_len) {
    if (x->c.n_attn == 0) return 0;
    const int hkv = x->kv_hl;
    return x->kv_bf16 ? attn_mma_chunk(B, hkv, max_len, x->num_sms) : attn_chunk(B, hkv, max_len, x->num_sms);
}

// mixer of layer L on the activation fragments in xfa (batch B starting at slot s0);
// the mixer output goes to `out` with epilogue `mode` (RESID into x, or STORE)
// With pf_p0 >= 0 the B rows are consecutive prompt tokens of sequence s0 at positions
// pf_p0.. (a prefill chunk): the chunked DeltaNet kernel, and attention over one shared slot.
int run_mixer(ab2_ctx* x, const Layer& L, int s0, int B, int max_len, float* out, int ldo, int mode,
              cudaStream_t st, int64_t pf_p0 = -1) {
    const Cfg& c = x->c;
    const int D = (int)c.dim;
    GemmEpi e_in = epi_store(x->proj, x->ldp, L.w_in.M);
    if (L.dn && pf_p0 < 0 && umma_for(x, B)) {
        // a batched decode step: the input projection pulls into L2 the recurrent states that
        // the DeltaNet kernel's CTAs load first (item i = slot i / H, head i % H is 64 KiB at
        // offset i * 64 KiB, and CTA c takes items c, c + grid, ...: the first kDnLeadRounds
        // items of every CTA are one contiguous range), so its pipeline fills from L2 instead
        // of waiting on HBM after the GEMM's CTAs leave the SMs
        const int64_t total = (int64_t)B * x->s_stride * (int64_t)sizeof(float);
        e_in.pf = x->dn_S + ((size_t)L.local * x->max_batch + s0) * x->s_stride;
        e_in.pf_bytes = std::min<int64_t>(total, (int64_t)kDnLeadRounds * x->num_sms * 128 * 128 * sizeof(float));
    }
    RET(gemm(x, L.w_in, x->xfa, B, e_in, st));
    if (L.dn) {
        DnParams p;
        p.proj = x->proj;
        p.ldp = x->ldp;
        p.conv = x->dn_conv + ((size_t)L.local * x->max_batch + s0) * x->conv_stride;
        p.conv_stride = x->conv_stride;
        p.conv_w = L.conv_w;
        p.K = (int)c.conv_k;
        p.S = x->dn_S + ((size_t)L.local * x->max_batch + s0) * x->s_stride;
        p.s_stride = x->s_stride;
        p.ssm_a = L.ssm_a;
        p.dt_bias = L.dt_bias;
        p.ssm_norm = L.ssm_norm;
        p.eps = c.eps;
        p.D = D;
        p.H = x->dn_hl;
        p.h0 = x->dn_h0;
        p.H_all = (int)c.dn_heads;
        p.out = act(x, x->xfb, D, B);
        p.o_out = nullptr;
        p.err = x->err_d;
        set_prefetch(x, B, &L.w_out, &p.pf, &p.pf_bytes);
        ProfScope ps(x, PC_DN, st);
        if (pf_p0 < 0) {
            launch_deltanet(p, B, st);
        } else {
            // the chunked kernel takes kPrefillChunk tokens per launch: a wider prefill step
            // runs as consecutive launches, each continuing from the state the last one left
            for (int r0 = 0; r0 < B; r0 += kPrefillChunk) {
                DnParams q = p;
                q.proj = p.proj + (size_t)r0 * p.ldp;
                q.row0 = r0;
                if (launch_dn_prefill(q, std::min(kPrefillChunk, B - r0), st))
                    return seterr(AB2_ERR_SHAPE, "DeltaNet prefill: unsupported shape");
            }
        }
    } else {
        const size_t kvel = x->kv_bf16 ? 2 : 4;
        AttnParams p;
        p.proj = x->proj;
        p.ldp = x->ldp;
        p.q_norm = L.q_norm;
        p.k_norm = L.k_norm;
        p.rope = x->rope;
        p.rot = x->rot;
        p.kc = (uint8_t*)x->kc + ((size_t)L.local * x->max_batch + s0) * x->kv_slot * kvel;
        p.vc = (uint8_t*)x->vc + ((size_t)L.local * x->max_batch + s0) * x->kv_slot * kvel;
        p.kv_slot_stride = x->kv_slot;
        p.cap = x->cap;
        p.pos = pf_p0 >= 0 ? x->pf_pos : x->pos_d + s0;
        if (pf_p0 >= 0) {
            // the chunk's tokens are rows of one sequence: every row reads (and the query prep
            // appends to) slot s0's cache
            p.kv_slot_stride = 0;
            p.seq_rows = 0;
        }
        p.Hq = (int)c.n_heads;
        p.Hkv = x->kv_hl;
        p.kvh0 = x->kv_h0;
        p.Hkv_all = (int)c.n_kv;
        // a prefill step on the bf16 cache runs the query-block kernel, which plans its own splits
        const bool pf_tc = pf_p0 >= 0 && x->kv_bf16;
        p.chunk = pf_tc ? attn_prefill_chunk(B, x->kv_hl, max_len, x->num_sms) : step_attn_chunk(x, B, max_len);
        // a replayed step graph keeps this plan while the longest context stays within its
        // split count, so every position up to the plan's last covered token is valid
        p.max_pos = std::min(x->cap - 1, attn_nsplit(max_len, p.chunk) * p.chunk - 1);
        if (attn_ws_floats(B, p.Hkv, attn_nsplit(max_len, p.chunk), (int)c.hd, p.Hq / p.Hkv_all) > x->aws_floats)
            return seterr(AB2_ERR_CAPACITY, "attention workspace too small for %d splits", attn_nsplit(max_len, p.chunk));
        p.ws = x->aws;
        p.qprep = x->aqp;
        p.tickets = x->atk;
        p.out = act(x, x->xfb, (int)(c.n_heads * c.hd), B);
        p.o_out = nullptr;
        p.err = x->err_d;
        set_prefetch(x, B, &L.w_out, &p.pf, &p.pf_bytes);
        if (x->kv_bf16) {
            // bf16 cache: TMA + tensor-core flash-decode; rows of (layer, slot s0, head 0, token 0).
            // Profiling times the attention kernel alone (its query prep and split merge are
            // small launches of their own).
            const int64_t row_base = ((int64_t)L.local * x->max_batch + s0) * x->kv_hl * x->cap;
            const auto ev = prof_pair(x, PC_ATTN);
            const int rc = pf_tc ? launch_attention_prefill(x->tmap_k, x->tmap_v, p, row_base, B, (int)c.hd, max_len,
                                                            x->num_sms, st, ev.first, ev.second)
                                 : launch_attention_mma(x->tmap_k, x->tmap_v, p, row_base, B, (int)c.hd, max_len,
                                                        x->num_sms, st, ev.first, ev.second);
            if (rc) return seterr(AB2_ERR_SHAPE, "attention: unsupported head configuration");
        } else {
            ProfScope ps(x, PC_ATTN, st);
            if (launch_attention(p, B, (int)c.hd, x->kv_bf16, max_len, st))
                return seterr(AB2_ERR_SHAPE, "attention: unsupported head configuration");
        }
    }
    if (L.dn ? x->dn_split : x->kv_split) {
        // head-parallel split: every rank wrote its heads' columns of the output projection's
        // activations; gather the other ranks' columns in place. Both activation layouts are
        // K-block-major, so a rank's columns are one contiguous byte range.
        const int K = L.dn ? D : (int)(c.n_heads * c.hd);
        const ActOut o = act(x, x->xfb, K, B);
        const size_t chunk = o.x16 ? (size_t)(K / x->tp_world / 64) * o.npad * 128
                                   : (size_t)(K / x->tp_world / 32) * o.xs.ntile * 512;
        ProfScope ps(x, PC_OTHER, st);
        NCK(nccl_api().all_gather(x->xfb + x->tp_rank * chunk, x->xfb, chunk, ncclUint8, x->nccl, st));
    }
    GemmEpi e = mode == EPI_RESID ? epi_resid(out, ldo, D) : epi_store(out, ldo, D);
    set_prefetch(x, B, &L.gate_up, &e.pf, &e.pf_bytes);
    return gemm(x, L.w_out, x->xfb, B, e, st);
}

// next: the weight of the GEMM that follows this FFN on the stream (prefetched into L2 by the
// down projection), or null
int run_ffn(ab2_ctx* x, const Layer& L, int B, float* out, int ldo, int mode, cudaStream_t st,
            const Q8Weight* next = nullptr) {
    const int D = (int)x->c.dim, F = (int)x->c.ffn;
    GemmEpi e = mode == EPI_RESID ? epi_resid(out, ldo, D) : epi_store(out, ldo, D);
    set_prefetch(x, B, next, &e.pf, &e.pf_bytes, kPrefetchCap);
    if (umma_for(x, B)) {
        // K-split gate/up sums into the f32 scratch (zeroed by the RMSNorm before), then the
        // down projection computes silu(g)*u from it as its activations
        GemmEpi gu;
        gu.mode = EPI_ADD;
        gu.y = x->h2;
        gu.ldy = 2 * F;
        gu.m_out = 2 * F;
        set_prefetch(x, B, &L.down, &gu.pf, &gu.pf_bytes);
        RET(gemm(x, L.gate_up, x->xfa, B, gu, st));
        return gemm(x, L.down, nullptr, B, e, st, x->h2, 2 * F);
    }
    RET(gemm(x, L.gate_up, x->xfa, B, epi_swiglu(act(x, x->xfb, F, B), F), st));
    return gemm(x, L.down, x->xfb, B, e, st);
}

int check_capacity(ab2_ctx* x, int B, int* max_len) {
    if (B < 1 || B > x->max_batch) return seterr(AB2_ERR_CAPACITY, "batch %d outside [1, %d]", B, x->max_batch);
    int64_t m = 0;
    for (int b = 0; b < B; b++) {
        if (x->pos_h[b] >= x->cap)
            return seterr(AB2_ERR_CAPACITY, "slot %d is full (pos %lld, max_ctx %d)", b, (long long)x->pos_h[b], x->cap);
        m = std::max<int64_t>(m, x->pos_h[b] + 1);
    }
    *max_len = (int)m;
    return 0;
}

// Embedding and every layer over B rows of the residual stream: the B sequences (slots
// [0, B)) of a decode step, or, with pf_p0 >= 0, B consecutive prompt tokens of sequence
// `slot` at positions pf_p0, pf_p0 + 1, ... (a prefill chunk)
int enqueue_body(ab2_ctx* x, const int32_t* tok_d, int B, int max_len, int slot, int64_t pf_p0, cudaStream_t st) {
    const Cfg& c = x->c;
    const int D = (int)c.dim;
    {
        ProfScope ps(x, PC_OTHER, st);
        launch_embed(x->embed, (int)c.vocab, tok_d, B, x->x, D, st);
        if (pf_p0 >= 0) launch_pos_fill(x->pf_pos, (int)pf_p0, B, st);
    }
    const ActOut xa = act(x, x->xfa, D, B);
    for (size_t li = 0; li < x->layers.size(); li++) {
        const Layer& L = x->layers[li];
        const Q8Weight* next = li + 1 < x->layers.size() ? &x->layers[li + 1].w_in : &x->lm_head;
        {
            // units of a split pair add into the STORE output: clear those projection rows
            const int64_t z0 = umma_for(x, B) ? umma_plan(L.w_in.MT, L.w_in.KT, L.w_in.M, x->num_sms).zero_row0 : L.w_in.M;
            ProfScope ps(x, PC_OTHER, st);
            launch_rmsnorm_act(x->x, D, L.attn_norm, D, c.eps, B, xa, st, z0 < L.w_in.M ? x->proj + z0 : nullptr,
                               x->ldp, (int)(L.w_in.M - z0));
        }
        RET(run_mixer(x, L, pf_p0 >= 0 ? slot : 0, B, max_len, x->x, D, EPI_RESID, st, pf_p0));
        {
            // on the tcgen05 path the gate/up projection adds into h2: clear it
            const int F2 = 2 * (int)c.ffn;
            ProfScope ps(x, PC_OTHER, st);
            launch_rmsnorm_act(x->x, D, L.post_norm, D, c.eps, B, xa, st, umma_for(x, B) ? x->h2 : nullptr, F2, F2);
        }
        RET(run_ffn(x, L, B, x->x, D, EPI_RESID, st, next));
    }
    return 0;
}

// final norm of the B residual rows at xrows, lm_head into logits_d [B][vocab], argmax
int enqueue_head(ab2_ctx* x, const float* xrows, int B, float* logits_d, int32_t* next_d, cudaStream_t st) {
    const Cfg& c = x->c;
    const int D = (int)c.dim;
    {
        // the lm_head's split units (all of them for small vocabularies, the K pieces of its
        // last pairs for large ones) add into the logits: clear those columns first
        const int64_t V = c.vocab;
        const int64_t z0 = umma_for(x, B) ? umma_plan(x->lm_head.MT, x->lm_head.KT, V, x->num_sms).zero_row0 : V;
        ProfScope ps(x, PC_OTHER, st);
        launch_rmsnorm_act(xrows, D, x->final_norm, D, c.eps, B, act(x, x->xfa, D, B), st,
                           z0 < V ? logits_d + z0 : nullptr, (int)V, (int)(V - z0));
    }
    RET(gemm(x, x->lm_head, x->xfa, B, epi_store(logits_d, (int)c.vocab, c.vocab), st));
    if (next_d) {
        ProfScope ps(x, PC_OTHER, st);
        launch_argmax2(logits_d, (int)c.vocab, (int)c.vocab, B, next_d, x->amax_part, kArgmaxChunks, st);
    }
    return 0;
}

// the kernels of one decode step, enqueued on st (or captured, when st is capturing)
int enqueue_kernels(ab2_ctx* x, const int32_t* tok_d, int B, int max_len, float* logits_d, int32_t* next_d,
                    cudaStream_t st) {
    RET(enqueue_body(x, tok_d, B, max_len, 0, -1, st));
    RET(enqueue_head(x, x->x, B, logits_d, next_d, st));
    {
        ProfScope ps(x, PC_OTHER, st);
        launch_pos_advance(x->pos_d, B, st);
    }
    CK(cudaGetLastError());
    return 0;
}

void graphs_clear(ab2_ctx* x) {
    for (StepGraph& g : x->graphs) {
        if (g.exec) cudaGraphExecDestroy(g.exec);
        g = StepGraph{};
    }
}

// Replay the captured step for this plan, capturing it first (on the context's stream) when
// no cached graph matches; the graph keeps the kernels' programmatic (PDL) dependencies.
int graph_step(ab2_ctx* x, const int32_t* tok_d, int B, int max_len, float* logits_d, int32_t* next_d,
               cudaStream_t st) {
    const int chunk = step_attn_chunk(x, B, max_len);
    const int splits = chunk ? attn_nsplit(max_len, chunk) : 0;
    StepGraph* g = nullptr;
    for (StepGraph& e : x->graphs)
        if (e.exec && e.B == B && e.chunk == chunk && e.splits == splits && e.tok == tok_d &&
            e.logits == logits_d && e.next == next_d)
            g = &e;
    if (!g) {
        g = &x->graphs[0];
        for (StepGraph& e : x->graphs)
            if (!e.exec || (g->exec && e.last < g->last)) g = &e;
        if (g->exec) cudaGraphExecDestroy(g->exec);
        *g = StepGraph{};
        cudaGraph_t graph = nullptr;
        CK(cudaStreamBeginCapture(x->stream, cudaStreamCaptureModeRelaxed));
        const int rc = enqueue_kernels(x, tok_d, B, max_len, logits_d, next_d, x->stream);
        const cudaError_t ce = cudaStreamEndCapture(x->stream, &graph);
        if (rc) {
            if (graph) cudaGraphDestroy(graph);
            return rc;
        }
        if (ce != cudaSuccess) return seterr(AB2_ERR_CUDA, "step graph capture failed: %s", cudaGetErrorString(ce));
        const cudaError_t ie = cudaGraphInstantiate(&g->exec, graph, 0);
        cudaGraphDestroy(graph);
        if (ie != cudaSuccess) {
            g->exec = nullptr;
            return seterr(AB2_ERR_CUDA, "step graph instantiation failed: %s", cudaGetErrorString(ie));
        }
        g->B = B;
        g->chunk = chunk;
        g->splits = splits;
        g->tok = tok_d;
        g->logits = logits_d;
        g->next = next_d;
        x->graph_captures++;
    }
    g->last = ++x->graph_tick;
    CK(cudaGraphLaunch(g->exec, st));
    return 0;
}

int enqueue_step(ab2_ctx* x, const int32_t* tok_d, int B, int max_len, float* logits_d, int32_t* next_d,
                 cudaStream_t st) {
    // profiling records events between launches, so it always runs the plain stream form
    if (x->graph_on && !x->prof.on)
        RET(graph_step(x, tok_d, B, max_len, logits_d, next_d, st));
    else
        RET(enqueue_kernels(x, tok_d, B, max_len, logits_d, next_d, st));
    for (int b = 0; b < B; b++) x->pos_h[b] += 1;
    return 0;
}

// a nonzero device error word means a tensor-core pipeline wait timed out: report it and re-arm
int take_device_error(ab2_ctx* x) {
    const unsigned e = *x->err_h;
    if (!e) return 0;
    *x->err_h = 0;
    cudaMemsetAsync(x->err_d, 0, 4, x->stream);
    cudaStreamSynchronize(x->stream);
    return seterr(AB2_ERR_CUDA, "device pipeline wait timed out (code 0x%x); results of this step are invalid", e);
}

int64_t launches_per_step(const ab2_ctx* x, int B) {
    // embed + 7 per layer + final norm + lm_head + 2 argmax passes + position advance
    const int64_t per_layer = 7;
    int64_t n = 1 + (int64_t)x->layers.size() * per_layer + 1 + 1 + 2 + 1;
    if (x->kv_bf16 && x->c.n_attn > 0) {
        // the tensor-core attention adds a merge kernel when the current context is split
        int max_len = 1;
        for (int b = 0; b < B && b < (int)x->pos_h.size(); b++) max_len = std::max(max_len, (int)x->pos_h[b] + 1);
        const int chunk = attn_mma_chunk(B, x->kv_hl, max_len, x->num_sms);
        n += x->c.n_attn * (attn_mma_launches(max_len, chunk) - 1);
    }
    return n;
}

// ------------------------------------------------------------------------- op-level cache
struct OpCache {
    std::mutex mu;
    void* ws = nullptr;
    size_t ws_bytes = 0;
    unsigned* tk = nullptr;
    size_t tk_n = 0;
    uint8_t* xf = nullptr;
    size_t xf_bytes = 0;
    float2* rope = nullptr;
    float* qp = nullptr;  // prepared queries of the tensor-core attention
    size_t qp_bytes = 0;
    int64_t rope_rows = 0;
    int rope_rot = 0;
    float rope_base = 0;
    unsigned* err = nullptr;
};
OpCache g_ops[64];

int ensure(void** p, size_t* have, size_t need) {
    if (*have >= need) return 0;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *have = 0;
    CK(cudaMalloc(p, need));
    CK(cudaMemset(*p, 0, need));
    *have = need;
    return 0;
}

}  // namespace

struct ab2_q8 {
    int device = 0;
    int num_sms = 148;
    Q8Weight w;
    int64_t n = 0;
};

// ================================================================================== C ABI
// ------------------------------------------------------------------------- wait-timeout test hook
static std::mutex g_wt_mu;
static std::atomic<bool> g_wt_any{false};
static WaitTest g_wt_armed[4];
static bool g_wt_on[4] = {false, false, false, false};

namespace ab2 {
WaitTest take_wait_test(int which, cudaStream_t st) {
    WaitTest w;
    if (!g_wt_any.load(std::memory_order_relaxed) || which < 1 || which > 3) return w;
    std::lock_guard<std::mutex> lk(g_wt_mu);
    if (!g_wt_on[which]) return w;
    // never baked into a captured graph: a capture keeps the production setting and the arm
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return w;
    g_wt_on[which] = false;
    g_wt_any.store(g_wt_on[1] || g_wt_on[2] || g_wt_on[3]);
    return g_wt_armed[which];
}
}  // namespace ab2

AB2_API const char* ab2_last_error(void) { return g_err.c_str(); }

AB2_API int ab2_debug_arm_wait_timeout(int which, int copy_index, uint32_t wait_ns) {
    if (which < kWaitTestGemm || which > kWaitTestDeltaNet)
        return seterr(AB2_ERR_ARG, "which must be 1 (GEMM), 2 (attention) or 3 (DeltaNet)");
    if (copy_index < 0) return seterr(AB2_ERR_ARG, "copy_index must be >= 0");
    if (wait_ns != 0 && wait_ns < 1000) return seterr(AB2_ERR_ARG, "wait_ns must be 0 (disarm) or >= 1000");
    std::lock_guard<std::mutex> lk(g_wt_mu);
    g_wt_on[which] = wait_ns != 0;
    g_wt_armed[which].wait_ns = wait_ns;
    g_wt_armed[which].withhold = copy_index;
    g_wt_any.store(g_wt_on[1] || g_wt_on[2] || g_wt_on[3]);
    return 0;
}

AB2_API int ab2_gguf_inspect(const uint8_t* gguf, uint64_t len, ab2_config* out) {
    if (!out) return seterr(AB2_ERR_ARG, "null config pointer");
    Gguf g;
    RET(parse_gguf(gguf, len, &g));
    Cfg c;
    RET(derive_config(g, &c));
    fill_config(c, out);
    return 0;
}

static int create_ctx(const uint8_t* gguf, uint64_t len, int device, int max_batch, int max_ctx,
                      const ab2_options* opt, int tp_rank, int tp_world, const uint8_t* tp_id, ab2_ctx** out) {
    if (!out) return seterr(AB2_ERR_ARG, "null output pointer");
    *out = nullptr;
    if (max_batch < 1 || max_batch > 64) return seterr(AB2_ERR_ARG, "max_batch must be in [1, 64]");
    if (max_ctx < 1) return seterr(AB2_ERR_ARG, "max_ctx must be positive");
    if (opt && (opt->exact_max_batch < -1 || opt->exact_max_batch > 64))
        return seterr(AB2_ERR_ARG, "exact_max_batch must be -1 or in [0, 64]");
    {
        // the file is checked on the host first, so a bad model fails the same way with or
        // without a GPU
        Gguf g;
        Cfg c;
        RET(parse_gguf(gguf, len, &g));
        RET(derive_config(g, &c));
        RET(validate_model(g, c, opt ? opt->rope_dims : 0));
    }
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return seterr(AB2_ERR_DEVICE, "no CUDA device available");
    }
    if (device < 0 || device >= ndev) return seterr(AB2_ERR_ARG, "device %d out of range", device);
    DeviceGuard dev_guard(device);
    CK(dev_guard.err);
    auto* x = new ab2_ctx();
    x->device = device;
    x->max_batch = max_batch;
    x->cap = max_ctx;
    x->kv_bf16 = opt ? opt->kv_bf16 != 0 : true;
    x->rot = opt ? opt->rope_dims : 0;
    // -1: no exact path, every step (one sequence too) on tcgen05; 0 (the default): 1
    x->exact_max = !opt || opt->exact_max_batch == 0 ? 1 : opt->exact_max_batch < 0 ? 0 : opt->exact_max_batch;
    // the tcgen05 weights are packed when a decode step or a prefill step (kPrefillChunk
    // rows on the exact path) can have more rows than exact_max; a prefill step then takes
    // kPrefillRowsTc tokens, the tcgen05 GEMM's widest N
    x->use_umma = std::max(max_batch, kPrefillChunk) > x->exact_max;
    x->pf_rows = x->use_umma ? kPrefillRowsTc : kPrefillChunk;
    x->tp_rank = tp_rank;
    x->tp_world = tp_world;
    cudaDeviceGetAttribute(&x->num_sms, cudaDevAttrMultiProcessorCount, device);
    int rc = 0;
    if (cudaStreamCreateWithFlags(&x->stream, cudaStreamNonBlocking) != cudaSuccess)
        rc = seterr(AB2_ERR_CUDA, "cudaStreamCreate failed");
    if (!rc) rc = build_context(x, gguf, len);
    if (!rc && tp_world > 1) {
        // every rank reaches this call after its own (identical) model checks; it returns once
        // all tp_world ranks have joined
        ncclUniqueId id;
        memcpy(id.internal, tp_id, sizeof id.internal);
        ncclComm_t comm = nullptr;
        const ncclResult_t nr = nccl_api().comm_init_rank(&comm, tp_world, id, tp_rank);
        if (nr != ncclSuccess) rc = seterr(AB2_ERR_CUDA, "ncclCommInitRank: %s", nccl_api().error_string(nr));
        else x->nccl = comm;
    }
    if (rc) {
        std::string keep = g_err;
        ab2_destroy(x);
        g_err = keep;
        return rc;
    }
    *out = x;
    return 0;
}

AB2_API int ab2_create(const uint8_t* gguf, uint64_t len, int device, int max_batch, int max_ctx,
                       const ab2_options* opt, ab2_ctx** out) {
    return create_ctx(gguf, len, device, max_batch, max_ctx, opt, 0, 1, nullptr, out);
}

AB2_API int ab2_tp_unique_id(uint8_t* id, uint64_t len) {
    if (!id || len < AB2_TP_ID_BYTES) return seterr(AB2_ERR_ARG, "the id buffer needs %d bytes", AB2_TP_ID_BYTES);
    const NcclApi& n = nccl_api();
    if (!n.why.empty()) return seterr(AB2_ERR_DEVICE, "%s", n.why.c_str());
    ncclUniqueId u;
    NCK(n.get_unique_id(&u));
    static_assert(sizeof u.internal == AB2_TP_ID_BYTES, "NCCL unique id size");
    memcpy(id, u.internal, AB2_TP_ID_BYTES);
    return 0;
}

AB2_API int ab2_create_tp(const uint8_t* gguf, uint64_t len, int device, int max_batch, int max_ctx,
                          const ab2_options* opt, int tp_rank, int tp_world, const uint8_t* tp_id, uint64_t id_len,
                          ab2_ctx** out) {
    if (!out) return seterr(AB2_ERR_ARG, "null output pointer");
    *out = nullptr;
    if (tp_world < 1 || tp_world > 8) return seterr(AB2_ERR_ARG, "tp_world must be in [1, 8]");
    if (tp_rank < 0 || tp_rank >= tp_world) return seterr(AB2_ERR_ARG, "tp_rank %d outside [0, %d)", tp_rank, tp_world);
    if (tp_world > 1 && (!tp_id || id_len != AB2_TP_ID_BYTES))
        return seterr(AB2_ERR_ARG, "tp_id must hold the %d bytes of ab2_tp_unique_id", AB2_TP_ID_BYTES);
    if (tp_world > 1) {
        const NcclApi& n = nccl_api();
        if (!n.why.empty()) return seterr(AB2_ERR_DEVICE, "%s", n.why.c_str());
    }
    return create_ctx(gguf, len, device, max_batch, max_ctx, opt, tp_rank, tp_world, tp_id, out);
}

AB2_API int ab2_get_tp(ab2_ctx* x, int32_t out[6]) {
    if (!x || !out) return seterr(AB2_ERR_ARG, "null argument");
    out[0] = x->tp_rank;
    out[1] = x->tp_world;
    out[2] = x->dn_h0;
    out[3] = x->dn_hl;
    out[4] = x->kv_h0;
    out[5] = x->kv_hl;
    return 0;
}

AB2_API void ab2_destroy(ab2_ctx* x) {
    if (!x) return;
    DeviceGuard dev_guard(x->device);
    if (x->stream) cudaStreamSynchronize(x->stream);
    // graphs that hold the split's collectives go before its communicator
    graphs_clear(x);
    if (x->nccl) nccl_api().comm_destroy(x->nccl);
    x->nccl = nullptr;
    for (void* p : x->allocs) cudaFree(p);
    if (x->tok_h) cudaFreeHost(x->tok_h);
    if (x->next_h) cudaFreeHost(x->next_h);
    if (x->err_h) cudaFreeHost(x->err_h);
    if (x->logits_h) cudaFreeHost(x->logits_h);
    for (auto& v : x->prof.ev)
        for (auto& e : v) {
            cudaEventDestroy(e.first);
            cudaEventDestroy(e.second);
        }
    graphs_clear(x);
    if (x->stream) cudaStreamDestroy(x->stream);
    delete x;
}

AB2_API int ab2_get_config(ab2_ctx* x, ab2_config* out) {
    if (!x || !out) return seterr(AB2_ERR_ARG, "null argument");
    fill_config(x->c, out);
    out->max_batch = x->max_batch;
    out->max_ctx = x->cap;
    out->kv_bf16 = x->kv_bf16 ? 1 : 0;
    out->rope_dims = x->rot;
    return 0;
}

AB2_API int ab2_layer_is_deltanet(ab2_ctx* x, int layer) {
    if (!x || layer < 0 || layer >= (int)x->layers.size()) return seterr(AB2_ERR_ARG, "bad layer");
    return x->layers[layer].dn ? 1 : 0;
}

static int check_slot(ab2_ctx* x, int slot) {
    if (!x) return seterr(AB2_ERR_ARG, "null context");
    if (slot < 0 || slot >= x->max_batch) return seterr(AB2_ERR_ARG, "slot %d out of range", slot);
    return 0;
}

AB2_API int ab2_reset_slot(ab2_ctx* x, int slot) {
    RET(check_slot(x, slot));
    DeviceGuard dev_guard(x->device);
    CK(dev_guard.err);
    const Cfg& c = x->c;
    const size_t kvel = x->kv_bf16 ? 2 : 4;
    for (int64_t i = 0; i < c.n_dn; i++) {
        CK(cudaMemsetAsync(x->dn_S + ((size_t)i * x->max_batch + slot) * x->s_stride, 0, x->s_stride * 4, x->stream));
        CK(cudaMemsetAsync(x->dn_conv + ((size_t)i * x->max_batch + slot) * x->conv_stride, 0, x->conv_stride * 4,
                           x->stream));
    }
    for (int64_t i = 0; i < c.n_attn; i++) {
        size_t off = ((size_t)i * x->max_batch + slot) * x->kv_slot * kvel;
        CK(cudaMemsetAsync((uint8_t*)x->kc + off, 0, x->kv_slot * kvel, x->stream));
        CK(cudaMemsetAsync((uint8_t*)x->vc + off, 0, x->kv_slot * kvel, x->stream));
    }
    CK(cudaStreamSynchronize(x->stream));
    return ab2_set_pos(x, slot, 0);
}

AB2_API int ab2_set_pos(ab2_ctx* x, int slot, int64_t pos) {
    RET(check_slot(x, slot));
    DeviceGuard dev_guard(x->device);
    CK(dev_guard.err);
    if (pos < 0 || pos > x->cap) return seterr(AB2_ERR_ARG, "pos %lld outside [0, %d]", (long long)pos, x->cap);
    int32_t p = (int32_t)pos;
    CK(cudaMemcpyAsync(x->pos_d + slot, &p, 4, cudaMemcpyHostToDevice, x->stream));
    CK(cudaStreamSynchronize(x->stream));
    x->pos_h[slot] = pos;
    return 0;
}

AB2_API int ab2_get_pos(ab2_ctx* x, int slot, int64_t* pos) {
    RET(check_slot(x, slot));
    if (!pos) return seterr(AB2_ERR_ARG, "null pos");
    *pos = x->pos_h[slot];
    return 0;
}

static int dn_layer(ab2_ctx* x, int layer, const Layer** L) {
    if (layer < 0 || layer >= (int)x->layers.size()) return seterr(AB2_ERR_ARG, "bad layer %d", layer);
    *L = &x->layers[layer];
    return 0;
}

static int dn_state_io(ab2_ctx* x, int layer, int slot, float* rec, float* conv, bool set) {
    if (!x) return seterr(AB2_ERR_ARG, "null context");
    DeviceGuard dev_guard(x->device);
    CK(dev_guard.err);
    RET(check_slot(x, slot));
    const Layer* L;
    RET(dn_layer(x, layer, &L));
    if (!L->dn) return seterr(AB2_ERR_ARG, "layer %d is not a DeltaNet layer", layer);
    float* S = x->dn_S + ((size_t)L->local * x->max_batch + slot) * x->s_stride;
    float* C = x->dn_conv + ((size_t)L->local * x->max_batch + slot) * x->conv_stride;
    auto kind = set ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToHost;
    // the host arrays hold every head; a head-parallel rank moves its own heads' part of the
    // recurrent state [H][128][128] only (and the whole conv state, of which it updates the
    // channels of its heads)
    float* rec_h = rec ? rec + (size_t)x->dn_h0 * 128 * 128 : nullptr;
    if (rec) CK(cudaMemcpyAsync(set ? (void*)S : rec_h, set ? (const void*)rec_h : S, x->s_stride * 4, kind, x->stream));
    if (conv) CK(cudaMemcpyAsync(set ? (void*)C : conv, set ? (const void*)conv : C, x->conv_stride * 4, kind, x->stream));
    CK(cudaStreamSynchronize(x->stream));
    return 0;
}

AB2_API int ab2_set_dn_state(ab2_ctx* x, int layer, int slot, const float* rec, const float* conv) {
    return dn_state_io(x, layer, slot, const_cast<float*>(rec), const_cast<float*>(conv), true);
}
AB2_API int ab2_get_dn_state(ab2_ctx* x, int layer, int slot, float* rec, float* conv) {
    return dn_state_io(x, layer, slot, rec, conv, false);
}

static inline uint16_t f32_to_bf16_rne(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x7fffffu)) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static int kv_io(ab2_ctx* x, int layer, int slot, float* k, float* v, int64_t n, bool set) {
    if (!x) return seterr(AB2_ERR_ARG, "null context");
    DeviceGuard dev_guard(x->device);
    CK(dev_guard.err);
    RET(check_slot(x, slot));
    const Layer* L;
    RET(dn_layer(x, layer, &L));
    if (L->dn) return seterr(AB2_ERR_ARG, "layer %d is not an attention layer", layer);
    if (n < 0 || n > x->cap) return seterr(AB2_ERR_ARG, "n_tokens %lld outside [0, %d]", (long long)n, x->cap);
    if (!k || !v) return seterr(AB2_ERR_ARG, "null k/v");
    const int64_t hd = x->c.hd;
    const size_t kvel = x->kv_bf16 ? 2 : 4;
    const size_t rowb = (size_t)n * hd * kvel;
    std::vector<uint8_t> tmp(rowb);
    for (int which = 0; which < 2; which++) {
        float* host = which ? v : k;
        uint8_t* dev = (uint8_t*)(which ? x->vc : x->kc) + ((size_t)L->local * x->max_batch + slot) * x->kv_slot * kvel;
        // the host arrays hold every kv head; a head-parallel rank moves its own heads only
        for (int64_t h = 0; h < x->kv_hl; h++) {
            uint8_t* d = dev + (size_t)h * x->cap * hd * kvel;
            float* hp = host + (size_t)(x->kv_h0 + h) * n * hd;
            if (set) {
                if (x->kv_bf16) {
                    uint16_t* t = (uint16_t*)tmp.data();
                    for (int64_t i = 0; i < n * hd; i++) t[i] = f32_to_bf16_rne(hp[i]);
                } else {
                    memcpy(tmp.data(), hp, rowb);
                }
                CK(cudaMemcpy(d, tmp.data(), rowb, cudaMemcpyHostToDevice));
            } else {
                CK(cudaMemcpy(tmp.data(), d, rowb, cudaMemcpyDeviceToHost));
                if (x->kv_bf16) {
                    const uint16_t* t = (const uint16_t*)tmp.data();
                    for (int64_t i = 0; i < n * hd; i++) {
                        uint32_t u = (uint32_t)t[i] << 16;
                        memcpy(&hp[i], &u, 4);
                    }
                } else {
                    memcpy(hp, tmp.data(), rowb);
                }
            }
        }
    }
    return 0;
}

AB2_API int ab2_set_kv(ab2_ctx* x, int layer, int slot, const float* k, const float* v, int64_t n) {
    return kv_io(x, layer, slot, const_cast<float*>(k), const_cast<float*>(v), n, true);
}
AB2_API int ab2_get_kv(ab2_ctx* x, int layer, int slot, float* k, float* v, int64_t n) {
    return kv_io(x, layer, slot, k, v, n, false);
}

AB2_API int ab2_seed_state(ab2_ctx* x, uint64_t seed, int n_slots, int64_t n_tokens, float dn_std, float conv_std,
                           float kv_std) {
    if (!x) return seterr(AB2_ERR_ARG, "null context");
    if (n_slots < 1 || n_slots > x->max_batch) return seterr(AB2_ERR_ARG, "n_slots outside [1, max_batch]");
    if (n_tokens < 0 || n_tokens >= x->cap) return seterr(AB2_ERR_ARG, "n_tokens outside [0, max_ctx)");
    DeviceGuard dev_guard(x->device);
    CK(dev_guard.err);
    const Cfg& c = x->c;
    // every value is a function of its index in the full (all heads) state, so a head-parallel
    // rank seeds exactly its heads' part of what one GPU seeds
    const bool whole_dn = x->dn_hl == (int)c.dn_heads, whole_kv = x->kv_hl == (int)c.n_kv;
    const int64_t s_all = c.dn_heads * 128 * 128;
    for (int64_t i = 0; i < c.n_dn; i++) {
        float* S = x->dn_S + (size_t)i * x->max_batch * x->s_stride;
        if (whole_dn) {
            launch_seed_f32(S, (int64_t)n_slots * x->s_stride, seed, (uint64_t)(3 * i), dn_std, x->stream);
        } else {
            for (int s = 0; s < n_slots; s++)
                launch_seed_f32(S + (size_t)s * x->s_stride, x->s_stride, seed, (uint64_t)(3 * i), dn_std, x->stream,
                                s * s_all + (int64_t)x->dn_h0 * 128 * 128);
        }
        launch_seed_f32(x->dn_conv + (size_t)i * x->max_batch * x->conv_stride, (int64_t)n_slots * x->conv_stride,
                        seed, (uint64_t)(3 * i + 1), conv_std, x->stream);
    }
    const size_t kvel = x->kv_bf16 ? 2 : 4;
    for (int64_t i = 0; i < c.n_attn; i++) {
        for (int s = 0; s < (whole_kv ? 1 : n_slots); s++) {
            const size_t off = ((size_t)i * x->max_batch + s) * x->kv_slot * kvel;
            const int64_t rows = whole_kv ? (int64_t)n_slots * c.n_kv * x->cap : (int64_t)x->kv_hl * x->cap;
            const int64_t i0 = whole_kv ? 0 : ((int64_t)s * c.n_kv + x->kv_h0) * x->cap * c.hd;
            launch_seed_kv((uint8_t*)x->kc + off, x->kv_bf16, rows, x->cap, n_tokens, (int)c.hd, seed,
                           (uint64_t)(1000 + 2 * i), kv_std, x->stream, i0);
            launch_seed_kv((uint8_t*)x->vc + off, x->kv_bf16, rows, x->cap, n_tokens, (int)c.hd, seed,
                           (uint64_t)(1001 + 2 * i), kv_std, x->stream, i0);
        }
    }
    CK(cudaGetLastError());
    CK(cudaStreamSynchronize(x->stream));
    for (int s = 0; s < n_slots; s++) RET(ab2_set_pos(x, s, n_tokens));
    return 0;
}

AB2_API int ab2_decode_step_device(ab2_ctx* x, const int32_t* tok_d, int B, float* logits_d, int32_t* next_d,
                                   void* stream) {
    if (!x || !tok_d) return seterr(AB2_ERR_ARG, "null argument");
    DeviceGuard dev_guard(x->device);
    CK(dev_guard.err);
    int max_len;
    RET(check_capacity(x, B, &max_len));
    cudaStream_t st = stream ? (cudaStream_t)stream : x->stream;
    return enqueue_step(x, tok_d, B, max_len, logits_d ? logits_d : x->logits, next_d, st);
}

AB2_API int ab2_decode_step(ab2_ctx* x, const int32_t* tokens, int B, float* logits, int32_t* next_tokens) {
    if (!x || !tokens) return seterr(AB2_ERR_ARG, "null argument");
    DeviceGuard dev_guard(x->device);
    CK(dev_guard.err);
    int max_len;
    RET(check_capacity(x, B, &max_len));
    for (int b = 0; b < B; b++)  // the reference indexes its embedding with the id (a panic when out of range)
        if (tokens[b] < 0 || tokens[b] >= x->c.vocab)
            return seterr(AB2_ERR_ARG, "token id %d of slot %d is outside [0, %lld)", tokens[b], b, (long long)x->c.vocab);
    memcpy(x->tok_h, tokens, (size_t)B * 4);
    CK(cudaMemcpyAsync(x->tok_d, x->tok_h, (size_t)B * 4, cudaMemcpyHostToDevice, x->stream));
    RET(enqueue_step(x, x->tok_d, B, max_len, x->logits, x->next_d, x->stream));
    if (next_tokens) CK(cudaMemcpyAsync(x->next_h, x->next_d, (size_t)B * 4, cudaMemcpyDeviceToHost, x->stream));
    if (logits) CK(cudaMemcpyAsync(logits, x->logits, (size_t)B * x->c.vocab * 4, cudaMemcpyDeviceToHost, x->stream));
    CK(cudaMemcpyAsync(x->err_h, x->err_d, 4, cudaMemcpyDeviceToHost, x->stream));
    CK(cudaStreamSynchronize(x->stream));
    prof_collect(x);
    RET(take_device_error(x));
    if (next_tokens) memcpy(next_tokens, x->next_h, (size_t)B * 4);
    return 0;
}

AB2_API int ab2_prefill(ab2_ctx* x, int slot, const int32_t* tokens, int64_t n, float* logits, int32_t* next_token) {
    RET(check_slot(x, slot));
    if (!tokens || n < 1) return seterr(AB2_ERR_ARG, "prefill needs at least one token");
    DeviceGuard dev_guard(x->device);
    CK(dev_guard.err);
    const Cfg& c = x->c;
    if (c.n_attn > 0 && !x->kv_bf16) return seterr(AB2_ERR_SHAPE, "prefill needs the bf16 KV cache");
    if (c.n_dn > 0 && c.conv_k != 4) return seterr(AB2_ERR_SHAPE, "prefill supports conv kernel 4 only");
    const int64_t p0 = x->pos_h[slot];
    if (p0 + n > x->cap)
        return seterr(AB2_ERR_CAPACITY, "slot %d: %lld prompt tokens at pos %lld exceed max_ctx %d", slot, (long long)n,
                      (long long)p0, x->cap);
    for (int64_t i = 0; i < n; i++)
        if (tokens[i] < 0 || tokens[i] >= c.vocab)
            return seterr(AB2_ERR_ARG, "prompt token %lld (id %d) is outside [0, %lld)", (long long)i, tokens[i],
                          (long long)c.vocab);
    cudaStream_t st = x->stream;
    // steps of up to pf_rows tokens, in stream order (each step's id copy follows the
    // previous step's kernels on the stream)
    for (int64_t t0 = 0; t0 < n; t0 += x->pf_rows) {
        const int T = (int)std::min<int64_t>(x->pf_rows, n - t0);
        CK(cudaMemcpyAsync(x->pf_tok, tokens + t0, (size_t)T * 4, cudaMemcpyHostToDevice, st));
        RET(enqueue_body(x, x->pf_tok, T, (int)(p0 + t0 + T), slot, p0 + t0, st));
        if (t0 + T == n) RET(enqueue_head(x, x->x + (size_t)(T - 1) * c.dim, 1, x->logits, x->next_d, st));
    }
    const int32_t pn = (int32_t)(p0 + n);
    CK(cudaMemcpyAsync(x->pos_d + slot, &pn, 4, cudaMemcpyHostToDevice, st));
    if (next_token) CK(cudaMemcpyAsync(x->next_h, x->next_d, 4, cudaMemcpyDeviceToHost, st));
    if (logits) CK(cudaMemcpyAsync(logits, x->logits, (size_t)c.vocab * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(x->err_h, x->err_d, 4, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    prof_collect(x);
    x->pos_h[slot] = p0 + n;
    RET(take_device_error(x));
    if (next_token) *next_token = x->next_h[0];
    return 0;
}

AB2_API int ab2_sync(ab2_ctx* x) {
    if (!x) return seterr(AB2_ERR_ARG, "null context");
    DeviceGuard dev_guard(x->device);
    CK(dev_guard.err);
    CK(cudaMemcpyAsync(x->err_h, x->err_d, 4, cudaMemcpyDeviceToHost, x->stream));
    CK(cudaDeviceSynchronize());
    prof_collect(x);
    return take_device_error(x);
}

AB2_API int ab2_launches_per_step(ab2_ctx* x, int B, int64_t* out) {
    if (!x || !out) return seterr(AB2_ERR_ARG, "null argument");
    *out = launches_per_step(x, B);
    return 0;
}

AB2_API int ab2_profile(ab2_ctx* x, int enable) {
    if (!x) return seterr(AB2_ERR_ARG, "null context");
    DeviceGuard dev_guard(x->device);
    CK(dev_guard.err);
    CK(cudaStreamSynchronize(x->stream));
    prof_collect(x);
    x->prof.on = enable != 0;
    return 0;
}

AB2_API int ab2_step_graph(ab2_ctx* x, int enable) {
    if (!x) return seterr(AB2_ERR_ARG, "null context");
    DeviceGuard dev_guard(x->device);
    CK(dev_guard.err);
    CK(cudaStreamSynchronize(x->stream));
    if (!enable) graphs_clear(x);
    x->graph_on = enable != 0;
    return 0;
}

AB2_API int ab2_step_graph_captures(ab2_ctx* x, int64_t* out) {
    if (!x || !out) return seterr(AB2_ERR_ARG, "null argument");
    *out = x->graph_captures;
    return 0;
}

AB2_API int ab2_profile_read(ab2_ctx* x, double ms[4], int64_t n[4]) {
    if (!x || !ms || !n) return seterr(AB2_ERR_ARG, "null argument");
    DeviceGuard dev_guard(x->device);
    CK(dev_guard.err);
    CK(cudaDeviceSynchronize());
    prof_collect(x);
    for (int c = 0; c < 4; c++) {
        ms[c] = x->prof.ms[c];
        n[c] = x->prof.n[c];
        x->prof.ms[c] = 0;
        x->prof.n[c] = 0;
    }
    return 0;
}

AB2_API int ab2_mixer_layer(ab2_ctx* x, int layer, int slot, const float* xin, float* out) {
    if (!x) return seterr(AB2_ERR_ARG, "null context");
    DeviceGuard dev_guard(x->device);
    CK(dev_guard.err);
    RET(check_slot(x, slot));
    if (!xin || !out) return seterr(AB2_ERR_ARG, "null argument");
    const Layer* L;
    RET(dn_layer(x, layer, &L));
    if (x->pos_h[slot] >= x->cap) return seterr(AB2_ERR_CAPACITY, "slot %d is full", slot);
    const int D = (int)x->c.dim;
    CK(cudaMemcpyAsync(x->x, xin, (size_t)D * 4, cudaMemcpyHostToDevice, x->stream));
    launch_to_act(x->x, D, D, 1, act(x, x->xfa, D, 1), x->stream);
    RET(run_mixer(x, *L, slot, 1, (int)x->pos_h[slot] + 1, x->tmp_out, D, EPI_STORE, x->stream));
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(out, x->tmp_out, (size_t)D * 4, cudaMemcpyDeviceToHost, x->stream));
    CK(cudaStreamSynchronize(x->stream));
    prof_collect(x);
    return 0;
}

AB2_API int ab2_ffn_layer(ab2_ctx* x, int layer, const float* xin, float* out) {
    if (!x) return seterr(AB2_ERR_ARG, "null context");
    DeviceGuard dev_guard(x->device);
    CK(dev_guard.err);
    if (!xin || !out) return seterr(AB2_ERR_ARG, "null argument");
    const Layer* L;
    RET(dn_layer(x, layer, &L));
    const int D = (int)x->c.dim;
    CK(cudaMemcpyAsync(x->x, xin, (size_t)D * 4, cudaMemcpyHostToDevice, x->stream));
    launch_to_act(x->x, D, D, 1, act(x, x->xfa, D, 1), x->stream);
    RET(run_ffn(x, *L, 1, x->tmp_out, D, EPI_STORE, x->stream));
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(out, x->tmp_out, (size_t)D * 4, cudaMemcpyDeviceToHost, x->stream));
    CK(cudaStreamSynchronize(x->stream));
    prof_collect(x);
    return 0;
}

// ------------------------------------------------------------------------------- op level
AB2_API int ab2_q8_create(const uint8_t* blocks, int64_t m, int64_t n, int device, ab2_q8** out) {
    if (!blocks || !out) return seterr(AB2_ERR_ARG, "null argument");
    *out = nullptr;
    if (m < 1 || n < 32 || n % 32) return seterr(AB2_ERR_SHAPE, "n must be a positive multiple of 32");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return seterr(AB2_ERR_DEVICE, "no CUDA device available");
    }
    DeviceGuard dev_guard(device);
    CK(dev_guard.err);
    auto* w = new ab2_q8();
    w->device = device;
    w->n = n;
    cudaDeviceGetAttribute(&w->num_sms, cudaDevAttrMultiProcessorCount, device);
    w->w.M = m;
    w->w.M16 = (int)((m + 15) / 16);
    w->w.KB = (int)(n / 32);
    w->w.MT = (int)((m + kUTileRows - 1) / kUTileRows);
    w->w.KT = (int)((n + 63) / 64);
    const size_t raw = (size_t)m * (n / 32) * 34;
    uint8_t* staging = nullptr;
    cudaError_t e = cudaMalloc(&w->w.qs, w->w.qs_bytes());
    if (e == cudaSuccess) e = cudaMalloc(&w->w.d, w->w.d_bytes());
    if (e == cudaSuccess) e = cudaMalloc(&w->w.qt, w->w.qt_bytes());
    if (e == cudaSuccess) e = cudaMalloc(&staging, raw);
    if (e == cudaSuccess) e = cudaMemset(w->w.qs, 0, w->w.qs_bytes());
    if (e == cudaSuccess) e = cudaMemset(w->w.d, 0, w->w.d_bytes());
    if (e == cudaSuccess) e = cudaMemset(w->w.qt, 0, w->w.qt_bytes());
    if (e == cudaSuccess) e = cudaMemcpy(staging, blocks, raw, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        launch_q8_repack(staging, m, w->w.KB, w->w, 0, kPlain, 0, 0);
        launch_q8t_repack(staging, m, w->w.KB, w->w, 0, kPlain, 0, 0);
        e = cudaDeviceSynchronize();
    }
    if (staging) cudaFree(staging);
    if (e != cudaSuccess) {
        ab2_q8_destroy(w);
        return seterr(e == cudaErrorMemoryAllocation ? AB2_ERR_OOM : AB2_ERR_CUDA, "ab2_q8_create: %s",
                      cudaGetErrorString(e));
    }
    *out = w;
    return 0;
}

AB2_API void ab2_q8_destroy(ab2_q8* w) {
    if (!w) return;
    DeviceGuard dev_guard(w->device);
    if (w->w.qs) cudaFree(w->w.qs);
    if (w->w.d) cudaFree(w->w.d);
    if (w->w.qt) cudaFree(w->w.qt);
    delete w;
}

AB2_API int ab2_q8_gemv(ab2_q8* w, const float* xin, int batch, float* y, void* stream) {
    if (!w || !xin || !y) return seterr(AB2_ERR_ARG, "null argument");
    if (batch < 1 || batch > 128) return seterr(AB2_ERR_CAPACITY, "batch must be in [1, 128]");
    DeviceGuard dev_guard(w->device);
    CK(dev_guard.err);
    OpCache& oc = g_ops[w->device & 63];
    std::lock_guard<std::mutex> lk(oc.mu);
    cudaStream_t st = (cudaStream_t)stream;
    const bool tc = batch >= kUmmaMinBatch;
    RET(ensure((void**)&oc.xf, &oc.xf_bytes, std::max(xfrag_bytes((int)w->n, batch), x16_bytes((int)w->n, batch))));
    size_t wsf = gemm_ws_floats(w->w.M16, w->w.KB, batch, w->num_sms);
    RET(ensure(&oc.ws, &oc.ws_bytes, std::max<size_t>(16, wsf * 4)));
    size_t tkb = oc.tk_n * 4;
    RET(ensure((void**)&oc.tk, &tkb, (size_t)gemm_grid_x(w->w.M16) * 4));
    oc.tk_n = tkb / 4;
    size_t errb = oc.err ? 16 : 0;
    RET(ensure((void**)&oc.err, &errb, 16));
    const ActOut in = act_out(oc.xf, (int)w->n, batch, tc);
    launch_to_act(xin, (int)w->n, (int)w->n, batch, in, st);
    const GemmEpi ep = epi_store(y, (int)w->w.M, w->w.M);
    if (tc) {
        // units of a split pair add into y: clear the rows they cover
        const int64_t z0 = umma_plan(w->w.MT, w->w.KT, w->w.M, w->num_sms).zero_row0;
        if (z0 < w->w.M)
            CK(cudaMemset2DAsync(y + z0, (size_t)w->w.M * 4, 0, (size_t)(w->w.M - z0) * 4, batch, st));
        if (launch_q8_umma(w->w, oc.xf, batch, oc.err, ep, w->num_sms, st))
            return seterr(AB2_ERR_CUDA, "tcgen05 GEMM launch failed: %s", cudaGetErrorString(cudaGetLastError()));
    } else {
        launch_q8_gemm(w->w, oc.xf, batch, (float*)oc.ws, oc.tk, ep, w->num_sms, st);
    }
    CK(cudaGetLastError());
    return 0;
}

// device error word of the op-level calls on the current device (tcgen05 wait timeouts)
AB2_API int ab2_op_error(uint32_t* code) {
    if (!code) return seterr(AB2_ERR_ARG, "null argument");
    int dev;
    CK(cudaGetDevice(&dev));
    OpCache& oc = g_ops[dev & 63];
    std::lock_guard<std::mutex> lk(oc.mu);
    *code = 0;
    if (!oc.err) return 0;
    CK(cudaDeviceSynchronize());
    CK(cudaMemcpy(code, oc.err, 4, cudaMemcpyDeviceToHost));
    CK(cudaMemset(oc.err, 0, 4));
    return 0;
}

AB2_API int ab2_q8_unpack(ab2_q8* w, float* out, void* stream) {
    if (!w || !out) return seterr(AB2_ERR_ARG, "null argument");
    DeviceGuard dev_guard(w->device);
    CK(dev_guard.err);
    launch_q8p_dequant(w->w, w->w.M, out, (cudaStream_t)stream);
    CK(cudaGetLastError());
    return 0;
}

AB2_API int ab2_q8_dequant(const uint8_t* blocks, int64_t n_blocks, float* out, void* stream) {
    if (!blocks || !out || n_blocks < 0) return seterr(AB2_ERR_ARG, "bad argument");
    if (n_blocks == 0) return 0;
    launch_q8_dequant_raw(blocks, n_blocks, out, (cudaStream_t)stream);
    CK(cudaGetLastError());
    return 0;
}

AB2_API int ab2_gated_delta(float* S, const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* beta,
                            const float* decay, int B, int H, int dk, int dv, float* o, void* stream) {
    if (!S || !q || !k || !v || !beta || !decay || !o) return seterr(AB2_ERR_ARG, "null argument");
    if (dk != 128 || dv != 128) return seterr(AB2_ERR_SHAPE, "dk = dv = 128 required");
    if (B < 0 || H < 0) return seterr(AB2_ERR_ARG, "negative size");
    if (B == 0 || H == 0) return 0;
    launch_gated_delta(S, q, k, v, beta, decay, B, H, o, (cudaStream_t)stream);
    CK(cudaGetLastError());
    return 0;
}

AB2_API int ab2_attn_decode(const float* proj, void* k_cache, void* v_cache, int64_t cap, const int32_t* pos, int B,
                            int Hq, int Hkv, int hd, int kv_bf16, const float* q_norm, const float* k_norm,
                            float rope_base, int rope_dims, int max_pos, float* out, void* stream) {
    if (!proj || !k_cache || !v_cache || !pos || !out) return seterr(AB2_ERR_ARG, "null argument");
    if (B < 1) return seterr(AB2_ERR_ARG, "B must be positive");
    if ((hd != 128 && hd != 256) || Hkv < 1 || Hq != 4 * Hkv) return seterr(AB2_ERR_SHAPE, "unsupported head configuration");
    if (rope_dims < 0 || rope_dims > hd || rope_dims % 2) return seterr(AB2_ERR_SHAPE, "bad rope_dims");
    if (max_pos < 0 || max_pos >= cap) return seterr(AB2_ERR_CAPACITY, "max_pos outside [0, cap)");
    int dev;
    CK(cudaGetDevice(&dev));
    int nsm = 148;
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    OpCache& oc = g_ops[dev & 63];
    std::lock_guard<std::mutex> lk(oc.mu);
    cudaStream_t st = (cudaStream_t)stream;
    const int rot = rope_dims ? rope_dims : hd;
    if (oc.rope_rows < cap || oc.rope_rot != rot || oc.rope_base != rope_base) {
        const int hr = rot / 2;
        std::vector<float2> tab((size_t)cap * hr);
        for (int j = 0; j < hr; j++) {
            const float freq = 1.0f / powf(rope_base, (float)(2 * j) / (float)rot);
            for (int64_t p = 0; p < cap; p++) {
                const float val = (float)p * freq;
                tab[(size_t)p * hr + j] = make_float2(cosf(val), sinf(val));
            }
        }
        CK(cudaStreamSynchronize(st));
        if (oc.rope) cudaFree(oc.rope);
        oc.rope = nullptr;
        CK(cudaMalloc(&oc.rope, tab.size() * sizeof(float2) + 16));
        CK(cudaMemcpy(oc.rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice));
        oc.rope_rows = cap;
        oc.rope_rot = rot;
        oc.rope_base = rope_base;
    }
    const int max_len = max_pos + 1;
    const int chunk = kv_bf16 ? attn_mma_chunk(B, Hkv, max_len, nsm) : attn_chunk(B, Hkv, max_len, nsm);
    // the tensor-core kernel lays partials out with a fixed split stride (its split bound)
    const int ws_splits = kv_bf16 ? attn_mma_nsplit_bound(B, Hkv, max_len, nsm) : attn_nsplit(max_len, chunk);
    RET(ensure(&oc.ws, &oc.ws_bytes, attn_ws_floats(B, Hkv, ws_splits, hd, Hq / Hkv) * 4));
    size_t errb = oc.err ? 16 : 0;
    RET(ensure((void**)&oc.err, &errb, 16));
    size_t tkb = oc.tk_n * 4;
    RET(ensure((void**)&oc.tk, &tkb, (size_t)B * Hkv * 4));
    oc.tk_n = tkb / 4;
    RET(ensure((void**)&oc.xf, &oc.xf_bytes, xfrag_bytes(Hq * hd, B)));
    if (kv_bf16) RET(ensure((void**)&oc.qp, &oc.qp_bytes, (size_t)B * Hq * hd * 4));
    AttnParams p;
    p.proj = proj;
    p.ldp = Hq * 2 * hd + 2 * Hkv * hd;
    p.q_norm = q_norm;
    p.k_norm = k_norm;
    p.rope = oc.rope;
    p.rot = rot;
    p.kc = k_cache;
    p.vc = v_cache;
    p.kv_slot_stride = (int64_t)Hkv * cap * hd;
    p.cap = (int)cap;
    p.pos = pos;
    p.max_pos = max_pos;
    p.Hq = Hq;
    p.Hkv = Hkv;
    p.chunk = chunk;
    p.ws = (float*)oc.ws;
    p.qprep = oc.qp;
    p.tickets = oc.tk;
    p.out = act_out(oc.xf, Hq * hd, B, false);
    p.o_out = out;
    p.err = oc.err;
    if (kv_bf16) {
        alignas(64) uint8_t tmk[128], tmv[128];
        const int64_t rows = (int64_t)B * Hkv * cap;
        if (make_kv_tensor_map(tmk, k_cache, rows, hd) || make_kv_tensor_map(tmv, v_cache, rows, hd))
            return seterr(AB2_ERR_ARG, "could not encode TMA tensor maps for the caches (alignment?)");
        if (launch_attention_mma(tmk, tmv, p, 0, B, hd, max_len, nsm, st))
            return seterr(AB2_ERR_SHAPE, "unsupported attention shape");
    } else if (launch_attention(p, B, hd, false, max_len, st)) {
        return seterr(AB2_ERR_SHAPE, "unsupported attention shape");
    }
    CK(cudaGetLastError());
    return 0;
}

// ===================================================================== allocation-free GEMV
// ab2_q8_gemv allocates its activation buffer, split-K workspace and tickets with
// cudaMalloc the first time a size is seen. Some callers cannot allow that: a host whose
// device memory is carved up by its own pool before it loads this library (cudaMalloc would
// fail or fragment it), and a caller on a latency-critical thread where cudaMalloc's implicit
// device synchronisation would stall the other streams. ab2_q8_gemv_noalloc runs the same
// mma.sync Q8_0 GEMM (batches 1..8) with all of its scratch in one fixed device array of
// this module, so it never allocates.
namespace {

// 4 MiB: tickets | activation fragments | split-K partials
constexpr size_t kNoAllocScratchBytes = 4u << 20;
constexpr size_t kNoAllocTicketBytes = 16u << 10;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};

// device address of g_noalloc_scratch on `dev` (the current device), looked up once
int noalloc_scratch(int dev, unsigned char** out) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return seterr(AB2_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed on device %d: %s", dev,
                          cudaGetErrorString(e));
        g_noalloc_ptr[dev] = p;
    }
    *out = (unsigned char*)g_noalloc_ptr[dev];
    return 0;
}

}  // namespace

AB2_API int ab2_q8_gemv_noalloc(ab2_q8* w, const float* xin, int batch, float* y, void* stream) {
    if (!w || !xin || !y) return seterr(AB2_ERR_ARG, "null argument");
    if (batch < 1 || batch >= kUmmaMinBatch)
        return seterr(AB2_ERR_CAPACITY, "ab2_q8_gemv_noalloc: batch %d outside [1, %d]", batch, kUmmaMinBatch - 1);
    if (w->device < 0 || w->device >= 64) return seterr(AB2_ERR_ARG, "device index out of range");
    const int gx = gemm_grid_x(w->w.M16);
    const size_t tk_bytes = (size_t)gx * 4;
    const size_t xf_bytes = (xfrag_bytes((int)w->n, batch) + 255) & ~(size_t)255;
    const size_t ws_bytes = gemm_ws_floats(w->w.M16, w->w.KB, batch, w->num_sms) * 4;
    if (tk_bytes > kNoAllocTicketBytes || kNoAllocTicketBytes + xf_bytes + ws_bytes > kNoAllocScratchBytes)
        return seterr(AB2_ERR_CAPACITY,
                      "ab2_q8_gemv_noalloc: %lld x %lld at batch %d needs %zu B of scratch (tickets %zu, "
                      "activations %zu, split-K %zu); the fixed scratch holds %zu B (tickets at most %zu)",
                      (long long)w->w.M, (long long)w->n, batch, kNoAllocTicketBytes + xf_bytes + ws_bytes,
                      tk_bytes, xf_bytes, ws_bytes, kNoAllocScratchBytes, kNoAllocTicketBytes);
    DeviceGuard dev_guard(w->device);
    CK(dev_guard.err);
    unsigned char* base = nullptr;
    RET(noalloc_scratch(w->device, &base));
    unsigned* tickets = (unsigned*)base;
    uint8_t* xf = base + kNoAllocTicketBytes;
    float* ws = (float*)(base + kNoAllocTicketBytes + xf_bytes);
    cudaStream_t st = (cudaStream_t)stream;
    // the split-K tickets must start at zero (the last CTA of each row group re-arms its
    // ticket, but a fresh device array or an earlier aborted call gives no such guarantee)
    CK(cudaMemsetAsync(tickets, 0, tk_bytes, st));
    const ActOut in = act_out(xf, (int)w->n, batch, false);
    launch_to_act(xin, (int)w->n, (int)w->n, batch, in, st);
    launch_q8_gemm(w->w, xf, batch, ws, tickets, epi_store(y, (int)w->w.M, w->w.M), w->num_sms, st);
    CK(cudaGetLastError());
    return 0;
}
