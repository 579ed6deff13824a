// ab2_bench -- command-line decode benchmark over the C ABI of include/ab2.h.
//
// The B200 counterpart of the reference CLI's `bench` command (crates/cli/src/main.rs:251-508;
// its GPU section, :418-498, times encode_full_token_gpu one token at a time). It loads a
// qwen35 GGUF, runs a prompt of -pp tokens through the decode path, and then times -tg greedy
// tokens. Flags follow the reference (-m/--model, -pp/--prompt-tokens, -tg/--gen-tokens,
// defaults 128/128). The additions are the batch, the device, the KV cache type and the
// step-graph switch.
//
// Differences, since no tokenizer is part of this path:
// * Prompt ids are synthetic: a seeded hash of (seed, sequence, position) modulo the
//   vocabulary.
// * Generation does not stop at EOS.
// * With -b B, B independent sequences decode together; the reference decodes one.
//
// --ctx N seeds every sequence's state as N tokens already processed (ab2_seed_state: DeltaNet
// and conv state, KV cache), the prefilled workload of the backend's own benchmark (64
// sequences at ctx 8192 on the 2B shape). The prompt then continues from position N; with
// -pp 0 generation starts straight from a synthetic id.
//
// --gpus N runs the same workload on N GPUs at once, one host thread and context per GPU
// (sequence sharding: nothing is exchanged), with seeds offset per GPU; the rates are
// whole-job figures over the slowest GPU's time.
//
// The timing also follows the reference. The first generated token is a warm-up. Speed is
// (tokens - 1) / time over the rest, summed over the batch, and wall-clock timed around the
// synchronous ab2_decode_step calls (host buffers in and out).
//
// Output: the reference's human-readable lines on stderr, and one JSON line on stdout with
// the rates and sequence 0's prompt and generated ids (`prompt`, `tokens`). Exit
// status: 0 on success, 1 if a file or ab2 call fails (the ab2 message is printed), 2 on bad
// usage.
#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "ab2.h"

namespace {

struct Args {
    std::string model;
    long pp = 128, tg = 128, batch = 1, device = 0, graph = 1, ctx = 0, gpus = 1, prefill = 1;
    bool kv_bf16 = true;
    uint64_t seed = 0;
};

void usage(FILE* f) {
    std::fprintf(f,
                 "usage: ab2_bench -m MODEL.gguf [-pp N] [-tg N] [-b B] [-d DEVICE] [--gpus N]\n"
                 "                 [--kv bf16|f32] [--graph 0|1] [--prefill 0|1] [--ctx N] [--seed S]\n"
                 "  -m, --model          qwen35 GGUF with Q8_0 weights (required)\n"
                 "  -pp, --prompt-tokens prompt tokens per sequence (default 128; 0 allowed)\n"
                 "  -tg, --gen-tokens    greedy tokens per sequence (default 128)\n"
                 "  -b, --batch          sequences decoded together (default 1)\n"
                 "  -d, --device         first CUDA device (default 0)\n"
                 "  --gpus               GPUs from --device on, one host thread and context each,\n"
                 "                       -b sequences per GPU (default 1)\n"
                 "  --kv                 KV cache type (default bf16; f32 as the reference)\n"
                 "  --graph              replay each step as one CUDA graph (default 1)\n"
                 "  --prefill            1 (default): each sequence's prompt through ab2_prefill\n"
                 "                       (bf16 cache); 0: one decode step per prompt position\n"
                 "  --ctx                seed every sequence as N tokens already processed (default 0)\n"
                 "  --seed               seed of the synthetic prompt ids (default 0)\n");
}

bool parse_long(const char* s, long lo, long* out) {
    char* end = nullptr;
    const long v = std::strtol(s, &end, 10);
    if (!s[0] || *end || v < lo) return false;
    *out = v;
    return true;
}

// 0: parsed; 1: help was asked for; 2: bad usage (message printed)
int parse(int argc, char** argv, Args* a) {
    for (int i = 1; i < argc; i++) {
        const std::string k = argv[i];
        if (k == "-h" || k == "--help") return 1;
        if (i + 1 >= argc) {
            std::fprintf(stderr, "ab2_bench: %s needs a value\n", k.c_str());
            return 2;
        }
        const char* v = argv[++i];
        bool ok = true;
        if (k == "-m" || k == "--model") {
            a->model = v;
        } else if (k == "-pp" || k == "--prompt-tokens") {
            ok = parse_long(v, 0, &a->pp);
        } else if (k == "-tg" || k == "--gen-tokens") {
            ok = parse_long(v, 1, &a->tg);
        } else if (k == "-b" || k == "--batch") {
            ok = parse_long(v, 1, &a->batch);
        } else if (k == "-d" || k == "--device") {
            ok = parse_long(v, 0, &a->device);
        } else if (k == "--gpus") {
            ok = parse_long(v, 1, &a->gpus) && a->gpus <= 64;
        } else if (k == "--ctx") {
            ok = parse_long(v, 0, &a->ctx);
        } else if (k == "--prefill") {
            ok = parse_long(v, 0, &a->prefill) && a->prefill <= 1;
        } else if (k == "--graph") {
            ok = parse_long(v, 0, &a->graph) && a->graph <= 1;
        } else if (k == "--seed") {
            long s = 0;
            ok = parse_long(v, 0, &s);
            a->seed = (uint64_t)s;
        } else if (k == "--kv") {
            ok = !std::strcmp(v, "bf16") || !std::strcmp(v, "f32");
            a->kv_bf16 = !std::strcmp(v, "bf16");
        } else {
            std::fprintf(stderr, "ab2_bench: unknown option %s\n", k.c_str());
            return 2;
        }
        if (!ok) {
            std::fprintf(stderr, "ab2_bench: bad value for %s: %s\n", k.c_str(), v);
            return 2;
        }
    }
    if (a->model.empty()) {
        std::fprintf(stderr, "ab2_bench: -m MODEL.gguf is required\n");
        return 2;
    }
    return 0;
}

bool read_file(const std::string& path, std::vector<uint8_t>* out) {
    FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) return false;
    bool ok = std::fseek(f, 0, SEEK_END) == 0;
    const long n = ok ? std::ftell(f) : -1;
    ok = ok && n > 0 && std::fseek(f, 0, SEEK_SET) == 0;
    if (ok) {
        out->resize((size_t)n);
        ok = std::fread(out->data(), 1, (size_t)n, f) == (size_t)n;
    }
    std::fclose(f);
    return ok;
}

// splitmix64 finaliser
uint64_t mix(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

int fail(const char* what) {
    std::fprintf(stderr, "ab2_bench: %s failed: %s\n", what, ab2_last_error());
    return 1;
}

// a JSON string body: quotes, backslashes and control characters escaped
std::string json_escape(const std::string& s) {
    std::string o;
    for (const char c : s) {
        if (c == '"' || c == '\\') {
            o += '\\';
            o += c;
        } else if ((unsigned char)c < 0x20) {
            char buf[8];
            std::snprintf(buf, sizeof(buf), "\\u%04x", (unsigned)(unsigned char)c);
            o += buf;
        } else {
            o += c;
        }
    }
    return o;
}

// A rendezvous of the device threads (C++17 has no std::barrier): wait() returns once every
// thread still taking part has arrived; drop() leaves for good, so a thread whose device failed
// does not hold the others back.
class Gate {
public:
    explicit Gate(int n) : n_(n) {}
    void wait() {
        std::unique_lock<std::mutex> lk(mu_);
        const long gen = gen_;
        if (++arrived_ >= n_) {
            open_locked();
        } else {
            cv_.wait(lk, [&] { return gen_ != gen; });
        }
    }
    void drop() {
        std::lock_guard<std::mutex> lk(mu_);
        if (--n_ > 0 && arrived_ >= n_) open_locked();
    }

private:
    void open_locked() {
        arrived_ = 0;
        gen_++;
        cv_.notify_all();
    }
    std::mutex mu_;
    std::condition_variable cv_;
    int n_;
    int arrived_ = 0;
    long gen_ = 0;
};

using Clock = std::chrono::steady_clock;

// one device's run: its own context, prompt and generation
struct Run {
    int rc = 0;
    const char* what = "";
    std::string msg;  // ab2_last_error() of the failing call, read on this thread
    Clock::time_point pp0, pp1, tg0, tg1;  // the timed prompt and generation phases
    std::vector<int32_t> prompt0, gen0;    // sequence 0's prompt and generated ids
};

// Every device thread uploads and seeds its context, then all start the prompt together (one
// gate) and the timed generation together (a second gate, after each thread's warm-up token),
// so the whole-job rates are taken over the span from the first start to the last end.
void run_device(const Args& a, const std::vector<uint8_t>& gguf, const ab2_config& cfg, int device, uint64_t seed,
                int max_ctx, Gate* gate, Run* out) {
    const int B = (int)a.batch;
    auto failed = [&](const char* what) {
        out->rc = 1;
        out->what = what;
        out->msg = ab2_last_error();
        gate->drop();
    };
    ab2_options opt;
    std::memset(&opt, 0, sizeof(opt));
    opt.kv_bf16 = a.kv_bf16 ? 1 : 0;
    ab2_ctx* ctx = nullptr;
    if (ab2_create(gguf.data(), gguf.size(), device, B, max_ctx, &opt, &ctx)) return failed("ab2_create");
    std::vector<int32_t> tok((size_t)B), next((size_t)B);
    do {
        if (ab2_step_graph(ctx, (int)a.graph)) {
            failed("ab2_step_graph");
            break;
        }
        if (a.ctx > 0 && ab2_seed_state(ctx, seed, B, a.ctx, 0.1f, 1.0f, 1.0f)) {
            failed("ab2_seed_state");
            break;
        }
        // the id each sequence starts generating from when there is no prompt
        for (int b = 0; b < B; b++) next[b] = (int32_t)(mix(~seed ^ mix((uint64_t)b)) % cfg.vocab);
        // the prompt id of sequence b at position i
        auto prompt_id = [&](int b, long i) { return (int32_t)(mix(seed ^ mix(((uint64_t)b << 32) + i)) % cfg.vocab); };
        gate->wait();
        out->pp0 = Clock::now();
        if (a.prefill && a.kv_bf16) {
            // prompt: each sequence's tokens through one prefill call (steps of 128 on the GPU)
            std::vector<int32_t> ids((size_t)a.pp);
            for (int b = 0; b < B && a.pp > 0 && !out->rc; b++) {
                for (long i = 0; i < a.pp; i++) ids[(size_t)i] = prompt_id(b, i);
                if (b == 0) out->prompt0 = ids;
                if (ab2_prefill(ctx, b, ids.data(), a.pp, nullptr, &next[(size_t)b])) failed("ab2_prefill");
            }
        } else {
            // prompt: one decode step per position for all sequences
            for (long i = 0; i < a.pp && !out->rc; i++) {
                for (int b = 0; b < B; b++) tok[b] = prompt_id(b, i);
                out->prompt0.push_back(tok[0]);
                if (ab2_decode_step(ctx, tok.data(), B, nullptr, next.data())) failed("ab2_decode_step (prompt)");
            }
        }
        if (out->rc) break;
        out->pp1 = Clock::now();
        // generation: the first token is the warm-up, then (tg - 1) timed greedy steps
        for (long i = 0; i < a.tg && !out->rc; i++) {
            if (i == 1) {
                gate->wait();
                out->tg0 = Clock::now();
            }
            tok = next;
            out->gen0.push_back(tok[0]);
            if (ab2_decode_step(ctx, tok.data(), B, nullptr, next.data())) failed("ab2_decode_step");
        }
        if (out->rc) break;
        out->tg1 = Clock::now();
        if (a.tg <= 1) out->tg0 = out->tg1;
    } while (false);
    ab2_destroy(ctx);
}

}  // namespace

int main(int argc, char** argv) {
    Args a;
    const int pr = parse(argc, argv, &a);
    if (pr == 1) {
        usage(stdout);
        return 0;
    }
    if (pr) {
        usage(stderr);
        return 2;
    }
    std::vector<uint8_t> gguf;
    if (!read_file(a.model, &gguf)) {
        std::fprintf(stderr, "ab2_bench: cannot read %s\n", a.model.c_str());
        return 1;
    }
    ab2_config cfg;
    if (ab2_gguf_inspect(gguf.data(), gguf.size(), &cfg)) return fail("reading the GGUF");
    std::fprintf(stderr, "  Model: %lld layers (%lld DeltaNet, %lld attention), dim %lld, vocab %lld\n",
                 (long long)cfg.n_layers, (long long)cfg.n_dn, (long long)cfg.n_attn, (long long)cfg.dim,
                 (long long)cfg.vocab);

    const long max_ctx = a.ctx + a.pp + a.tg + 2;
    if (max_ctx > 0x7fffffffL) {
        std::fprintf(stderr, "ab2_bench: --ctx + -pp + -tg is too large\n");
        return 2;
    }
    // one host thread per GPU, each with its own context (contexts are per device and are
    // driven from separate threads), started together
    const int G = (int)a.gpus;
    std::vector<Run> runs((size_t)G);
    std::fprintf(stderr, "  Uploading model weights to %d GPU(s) from device %ld...\n", G, a.device);
    std::vector<std::thread> threads;
    Gate gate(G);
    for (int g = 0; g < G; g++)
        threads.emplace_back(run_device, std::cref(a), std::cref(gguf), std::cref(cfg), (int)a.device + g,
                             a.seed + (uint64_t)g, (int)max_ctx, &gate, &runs[(size_t)g]);
    for (auto& t : threads) t.join();
    int rc = 0;
    for (int g = 0; g < G; g++)
        if (runs[(size_t)g].rc) {
            std::fprintf(stderr, "ab2_bench: GPU %ld: %s failed: %s\n", a.device + g, runs[(size_t)g].what,
                         runs[(size_t)g].msg.c_str());
            rc = 1;
        }
    if (rc) return rc;

    // whole-job rates over the span from the first device's start to the last device's end
    const int B = (int)a.batch;
    Clock::time_point pp0 = runs[0].pp0, pp1 = runs[0].pp1, tg0 = runs[0].tg0, tg1 = runs[0].tg1;
    for (const Run& r : runs) {
        pp0 = std::min(pp0, r.pp0);
        pp1 = std::max(pp1, r.pp1);
        tg0 = std::min(tg0, r.tg0);
        tg1 = std::max(tg1, r.tg1);
    }
    const double pp_s = std::chrono::duration<double>(pp1 - pp0).count();
    const double tg_s = std::chrono::duration<double>(tg1 - tg0).count();
    const double pp_tps = pp_s > 0 ? (double)G * B * a.pp / pp_s : 0.0;
    const double tg_tps = tg_s > 0 ? (double)G * B * (a.tg - 1) / tg_s : 0.0;
    std::fprintf(stderr, "  Prompt: %ld tokens x %d sequences x %d GPU(s) in %.1fms (%.1f tok/s)\n", a.pp, B, G,
                 1e3 * pp_s, pp_tps);
    std::fprintf(stderr, "  Tokens: %ld\n", a.tg);
    std::fprintf(stderr, "  Time: %.1fms\n", 1e3 * tg_s);
    std::fprintf(stderr, "  Speed: %.1f tok/s (B200 tg%ld, %d sequences x %d GPU(s))\n", tg_tps, a.tg, B, G);
    const Run& r0 = runs[0];
    std::printf("{\"model\": \"%s\", \"gpus\": %d, \"batch\": %d, \"ctx\": %ld, \"prompt_tokens\": %ld, "
                "\"gen_tokens\": %ld, \"prompt_tok_s\": %.2f, \"gen_tok_s\": %.2f, \"gen_ms\": %.3f, \"kv\": \"%s\", "
                "\"graph\": %ld, \"gen_tok_s_per_gpu\": [",
                json_escape(a.model).c_str(), G, B, a.ctx, a.pp, a.tg, pp_tps, tg_tps, 1e3 * tg_s,
                a.kv_bf16 ? "bf16" : "f32", a.graph);
    for (int g = 0; g < G; g++) {
        const double t = std::chrono::duration<double>(runs[(size_t)g].tg1 - runs[(size_t)g].tg0).count();
        std::printf("%s%.2f", g ? ", " : "", t > 0 ? (double)B * (a.tg - 1) / t : 0.0);
    }
    std::printf("], \"prompt\": [");
    for (size_t i = 0; i < r0.prompt0.size(); i++) std::printf("%s%d", i ? ", " : "", r0.prompt0[i]);
    std::printf("], \"tokens\": [");
    for (size_t i = 0; i < r0.gen0.size(); i++) std::printf("%s%d", i ? ", " : "", r0.gen0[i]);
    std::printf("]}\n");
    return 0;
}
