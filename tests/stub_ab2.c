/* stub_ab2.c -- test double of libab2.so for the command-line benchmark's CPU tests: the
 * entry points ab2_bench calls, with a deterministic stand-in for decoding (next token =
 * (7 * token + position + slot) mod vocab) and a call log written to $STUB_LOG. Built only
 * by tests/test_cli.py. */
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "ab2.h"

#define STUB_VOCAB 1000

struct ab2_ctx {
    int device, max_batch, max_ctx;
    long long pos[256];
};

static const char* g_msg = "";

/* one line per call, appended to $STUB_LOG (long long arguments) */
static void logf_(const char* fmt, ...) {
    const char* path = getenv("STUB_LOG");
    if (!path) return;
    FILE* f = fopen(path, "a");
    if (!f) return;
    va_list ap;
    va_start(ap, fmt);
    vfprintf(f, fmt, ap);
    va_end(ap);
    fputc('\n', f);
    fclose(f);
}

const char* ab2_last_error(void) { return g_msg; }

int ab2_gguf_inspect(const uint8_t* gguf, uint64_t len, ab2_config* out) {
    memset(out, 0, sizeof(*out));
    if (len < 4 || memcmp(gguf, "GGUF", 4) != 0) {
        g_msg = "stub: not a GGUF file";
        return AB2_ERR_FORMAT;
    }
    out->n_layers = 4;
    out->n_dn = 3;
    out->n_attn = 1;
    out->dim = 64;
    out->vocab = STUB_VOCAB;
    return 0;
}

int ab2_create(const uint8_t* gguf, uint64_t len, int device, int max_batch, int max_ctx,
               const ab2_options* opt, ab2_ctx** out) {
    (void)gguf;
    (void)len;
    logf_("create %lld %lld %lld %lld", (long long)device, (long long)max_batch, (long long)max_ctx,
          (long long)(opt ? opt->kv_bf16 : -1));
    const char* fail_dev = getenv("STUB_FAIL_CREATE_DEVICE");  /* only this device fails */
    if (getenv("STUB_FAIL_CREATE") || (fail_dev && atoi(fail_dev) == device)) {
        g_msg = "stub: no CUDA device available";
        return AB2_ERR_DEVICE;
    }
    const char* slow_dev = getenv("STUB_SLOW_CREATE_DEVICE");  /* this device uploads slowly */
    if (slow_dev && atoi(slow_dev) == device) usleep(400000);
    if (max_batch < 1 || max_batch > 256) {
        g_msg = "stub: bad max_batch";
        return AB2_ERR_ARG;
    }
    ab2_ctx* x = (ab2_ctx*)calloc(1, sizeof(ab2_ctx));
    x->device = device;
    x->max_batch = max_batch;
    x->max_ctx = max_ctx;
    *out = x;
    return 0;
}

void ab2_destroy(ab2_ctx* ctx) {
    logf_("destroy");
    free(ctx);
}

int ab2_step_graph(ab2_ctx* ctx, int enable) {
    (void)ctx;
    logf_("graph %lld 0 0 0", (long long)enable);
    return 0;
}

int ab2_seed_state(ab2_ctx* x, uint64_t seed, int n_slots, int64_t n_tokens, float dn_std, float conv_std,
                   float kv_std) {
    (void)dn_std;
    (void)conv_std;
    (void)kv_std;
    logf_("seed %lld %lld %lld 0 %lld", (long long)seed, (long long)n_slots, (long long)n_tokens,
          (long long)x->device);
    if (n_slots < 1 || n_slots > x->max_batch || n_tokens < 0 || n_tokens >= x->max_ctx) {
        g_msg = "stub: bad seed_state arguments";
        return AB2_ERR_ARG;
    }
    for (int b = 0; b < n_slots; b++) x->pos[b] = n_tokens;
    return 0;
}

/* the prompt of one slot: the decode stand-in applied token by token */
int ab2_prefill(ab2_ctx* x, int slot, const int32_t* tokens, int64_t n, float* logits, int32_t* next_token) {
    if (slot < 0 || slot >= x->max_batch || n < 1) {
        g_msg = "stub: bad prefill arguments";
        return AB2_ERR_ARG;
    }
    if (x->pos[slot] + n > x->max_ctx) {
        g_msg = "stub: prompt does not fit";
        return AB2_ERR_CAPACITY;
    }
    for (int64_t i = 0; i < n; i++)
        if (tokens[i] < 0 || tokens[i] >= STUB_VOCAB) {
            g_msg = "stub: token out of range";
            return AB2_ERR_ARG;
        }
    (void)logits;
    int32_t nx = 0;
    for (int64_t i = 0; i < n; i++) {
        nx = (int32_t)((7LL * tokens[i] + x->pos[slot] + slot) % STUB_VOCAB);
        x->pos[slot]++;
    }
    if (next_token) *next_token = nx;
    logf_("prefill %lld %lld %lld %lld %lld %lld", (long long)slot, (long long)n, (long long)tokens[0],
          (long long)tokens[n - 1], (long long)nx, (long long)x->device);
    return 0;
}

int ab2_decode_step(ab2_ctx* x, const int32_t* tokens, int batch, float* logits, int32_t* next) {
    if (batch < 1 || batch > x->max_batch) {
        g_msg = "stub: batch outside [1, max_batch]";
        return AB2_ERR_CAPACITY;
    }
    for (int b = 0; b < batch; b++) {
        if (x->pos[b] >= x->max_ctx) {
            g_msg = "stub: slot is full";
            return AB2_ERR_CAPACITY;
        }
        if (tokens[b] < 0 || tokens[b] >= STUB_VOCAB) {
            g_msg = "stub: token out of range";
            return AB2_ERR_ARG;
        }
    }
    (void)logits;
    int32_t n0 = 0;
    for (int b = 0; b < batch; b++) {
        const int32_t n = (int32_t)((7LL * tokens[b] + x->pos[b] + b) % STUB_VOCAB);
        if (next) next[b] = n;
        if (b == 0) n0 = n;
        x->pos[b]++;
    }
    logf_("step %lld %lld %lld %lld %lld", (long long)batch, (long long)tokens[0], (long long)n0,
          (long long)(batch > 1 ? tokens[batch - 1] : -1), (long long)x->device);
    return 0;
}
