// Engine harness: runs tiny-llm's own engine classes (TransformerLayer,
// InferenceEngine) on seeded synthetic weights and writes what they produce
// to a file, for tests/test_gpu_engine.py.
//
// TEST INFRASTRUCTURE ONLY. oracle/Makefile.engine compiles this file twice:
//   engine_ref     against the reference's sources as they are (its
//                  KVCacheManager and kernels::attention_decode/prefill);
//   engine_dropin  against the same sources with oracle/engine/drop_in.patch
//                  applied and this repository's include/tiny_llm/kv_cache.h
//                  in front (the paged cache through libtllm_kv.so), with
//                  TLLM_DROP_IN defined (batched modes).
//
// Modes (all sizes on the command line, everything else from the seed):
//   layer <hidden> <heads> <kv_heads> <head_dim> <inter> <group> <P> <seed> <out>
//       layer 0 of a model: forwardPrefill over P prompt rows, advance, then
//       forward of one decode row at position P (src/transformer.cpp:123-198;
//       the fixture of tests/test_integration.cu:208-269 with data checked).
//       Writes the weights, the inputs, both outputs and the decode row's
//       normed input and Q/K/V (and, drop-in, its attention) as probes.
//   batch <hidden> <heads> <kv_heads> <head_dim> <inter> <group> <seed> <out> <P_0> ... <P_B-1>
//       (drop-in only) every sequence prefilled, then ONE forwardBatch step
//       of all of them, and the same decode row of each through forward on a
//       second cache: writes the batched and the one-by-one outputs.
//   generate <layers> <hidden> <heads> <kv_heads> <head_dim> <inter> <vocab> <group> <max_seq>
//            <seed> <max_new> <out> <prompt tokens...>
//       InferenceEngine::generate, greedy: writes the model's weights and the
//       generated token ids.
//   generate_batch <same as generate> <prompt lengths ...> -- <all prompts' tokens...>
//       (drop-in only) InferenceEngine::generateBatch, and generate for each
//       prompt on the same engine: writes both.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "rmsnorm.cuh"
#include "tiny_llm/inference_engine.h"
#include "tiny_llm/transformer.h"
#include "w8a16_matmul.cuh"

using namespace tiny_llm;

namespace {

#define HCHECK(x)                                                                                 \
    do {                                                                                          \
        cudaError_t e_ = (x);                                                                     \
        if (e_ != cudaSuccess) {                                                                  \
            std::fprintf(stderr, "%s:%d: %s: %s\n", __FILE__, __LINE__, #x, cudaGetErrorString(e_)); \
            std::exit(3);                                                                         \
        }                                                                                         \
    } while (0)

// splitmix64 stream: uniform doubles in [0, 1) from (seed, stream id).
struct Rng {
    uint64_t s;
    Rng(uint64_t seed, uint64_t id) : s(seed * 0x9E3779B97F4A7C15ull + id * 0xD1B54A32D192ED03ull + 1) {}
    uint64_t next() {
        uint64_t z = (s += 0x9E3779B97F4A7C15ull);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    }
    double uniform() { return (double)(next() >> 11) * (1.0 / 9007199254740992.0); }
};

// Named host arrays written to the output file:
// [u32 name length][name][u8 kind: 'h' fp16, 'b' int8, 'i' int32][u64 count][data].
struct Dump {
    FILE *f;
    explicit Dump(const char *path) : f(std::fopen(path, "wb")) {
        if (!f) {
            std::perror(path);
            std::exit(2);
        }
    }
    ~Dump() { std::fclose(f); }
    void put(const std::string &name, char kind, const void *data, uint64_t count) {
        const uint32_t n = (uint32_t)name.size();
        const size_t esz = kind == 'h' ? 2 : (kind == 'b' ? 1 : 4);
        std::fwrite(&n, 4, 1, f);
        std::fwrite(name.data(), 1, n, f);
        std::fwrite(&kind, 1, 1, f);
        std::fwrite(&count, 8, 1, f);
        std::fwrite(data, esz, count, f);
    }
    template <typename T>
    void dev(const std::string &name, char kind, const T *d, uint64_t count) {
        std::vector<T> h(count);
        HCHECK(cudaMemcpy(h.data(), d, count * sizeof(T), cudaMemcpyDeviceToHost));
        put(name, kind, h.data(), count);
    }
};

template <typename T>
T *upload(const std::vector<T> &h) {
    T *d = nullptr;
    HCHECK(cudaMalloc(&d, h.size() * sizeof(T)));
    HCHECK(cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice));
    return d;
}

std::vector<half> random_half(size_t n, double lo, double hi, uint64_t seed, uint64_t id) {
    Rng r(seed, id);
    std::vector<half> v(n);
    for (auto &x : v) x = __float2half((float)(lo + (hi - lo) * r.uniform()));
    return v;
}

// int8 weights uniform in [-127, 127]; scales around 1 / (sqrt(rows) * 64)
// so each projection keeps activations of order one.
QuantizedWeight random_weight(int rows, int cols, int group, uint64_t seed, uint64_t id) {
    Rng r(seed, id);
    std::vector<int8_t> w((size_t)rows * cols);
    for (auto &x : w) x = (int8_t)((int)(r.uniform() * 255.0) - 127);
    const int srows = (rows + group - 1) / group;
    const double s0 = 1.0 / (std::sqrt((double)rows) * 64.0);
    std::vector<half> s((size_t)srows * cols);
    for (auto &x : s) x = __float2half((float)(s0 * (0.5 + r.uniform())));
    QuantizedWeight q;
    q.data = upload(w);
    q.scales = upload(s);
    q.rows = rows;
    q.cols = cols;
    q.group_size = group;
    return q;
}

void dump_weight(Dump &d, const std::string &name, const QuantizedWeight &q) {
    d.dev(name + ".w", 'b', q.data, q.weightElements());
    d.dev(name + ".s", 'h', q.scales, q.scaleElements());
}

TransformerWeights layer_weights(const ModelConfig &c, int group, uint64_t seed, int layer) {
    const int h = c.hidden_dim, qd = c.num_heads * c.head_dim, kvd = c.num_kv_heads * c.head_dim,
              f = c.intermediate_dim;
    const uint64_t base = 100 * (uint64_t)(layer + 1);
    TransformerWeights w;
    w.wq = random_weight(h, qd, group, seed, base + 1);
    w.wk = random_weight(h, kvd, group, seed, base + 2);
    w.wv = random_weight(h, kvd, group, seed, base + 3);
    w.wo = random_weight(qd, h, group, seed, base + 4);
    w.w1 = random_weight(h, f, group, seed, base + 5);
    w.w2 = random_weight(f, h, group, seed, base + 6);
    w.w3 = random_weight(h, f, group, seed, base + 7);
    w.rms_att_weight = upload(random_half(h, 0.8, 1.2, seed, base + 8));
    w.rms_ffn_weight = upload(random_half(h, 0.8, 1.2, seed, base + 9));
    return w;
}

void dump_layer(Dump &d, const TransformerWeights &w, int hidden) {
    dump_weight(d, "wq", w.wq);
    dump_weight(d, "wk", w.wk);
    dump_weight(d, "wv", w.wv);
    dump_weight(d, "wo", w.wo);
    dump_weight(d, "w1", w.w1);
    dump_weight(d, "w2", w.w2);
    dump_weight(d, "w3", w.w3);
    d.dev("rms_att", 'h', w.rms_att_weight, hidden);
    d.dev("rms_ffn", 'h', w.rms_ffn_weight, hidden);
}

ModelConfig model_config(int layers, int hidden, int heads, int kv_heads, int head_dim, int inter, int vocab,
                         int max_seq) {
    ModelConfig c;
    c.vocab_size = vocab;
    c.hidden_dim = hidden;
    c.num_layers = layers;
    c.num_heads = heads;
    c.num_kv_heads = kv_heads;
    c.head_dim = head_dim;
    c.intermediate_dim = inter;
    c.max_seq_len = max_seq;
    c.eos_token_id = -1;  // never produced: every run generates max_new tokens
    return c;
}

std::unique_ptr<KVCacheManager> make_cache(const ModelConfig &c, int layers, int batch) {
#ifdef TLLM_DROP_IN
    PagedKVCacheConfig kv;
    kv.num_q_heads = c.num_heads;
#else
    KVCacheConfig kv;
#endif
    kv.num_layers = layers;
    kv.num_heads = c.num_kv_heads;
    kv.head_dim = c.head_dim;
    kv.max_seq_len = c.max_seq_len;
    kv.max_batch_size = batch;
    auto r = KVCacheManager::create(kv);
    if (r.isErr()) {
        std::fprintf(stderr, "KVCacheManager::create: %s\n", r.error().c_str());
        std::exit(4);
    }
    return std::move(r.value());
}

int seq_of(KVCacheManager &cache, int max_len) {
    auto r = cache.allocateSequence(max_len);
    if (r.isErr()) {
        std::fprintf(stderr, "allocateSequence: %s\n", r.error().c_str());
        std::exit(4);
    }
    return r.value();
}

int run_layer(char **a) {
    const int hidden = std::atoi(a[0]), heads = std::atoi(a[1]), kv_heads = std::atoi(a[2]),
              head_dim = std::atoi(a[3]), inter = std::atoi(a[4]), group = std::atoi(a[5]), P = std::atoi(a[6]);
    const uint64_t seed = std::strtoull(a[7], nullptr, 10);
    Dump d(a[8]);
    const ModelConfig c = model_config(1, hidden, heads, kv_heads, head_dim, inter, 32, P + 8);
    TransformerWeights w = layer_weights(c, group, seed, 0);
    auto cache = make_cache(c, 1, 1);
    const int sid = seq_of(*cache, P + 1);
    TransformerLayer layer(0, w, c);

    auto xp_h = random_half((size_t)P * hidden, -1.0, 1.0, seed, 1);
    auto xd_h = random_half(hidden, -1.0, 1.0, seed, 2);
    half *xp = upload(xp_h), *xd = upload(xd_h);
    layer.forwardPrefill(xp, *cache, sid, P);
    HCHECK(cudaDeviceSynchronize());
    if (cache->advanceSeqLen(sid, P).isErr()) return 5;
    layer.forward(xd, *cache, sid, P);
    HCHECK(cudaDeviceSynchronize());

    dump_layer(d, w, hidden);
    d.put("x_prefill_in", 'h', xp_h.data(), xp_h.size());
    d.put("x_decode_in", 'h', xd_h.data(), xd_h.size());
    d.dev("x_prefill_out", 'h', xp, (size_t)P * hidden);
    d.dev("x_decode_out", 'h', xd, hidden);

    // the decode row's attention inputs, recomputed with the engine's own
    // kernels (RMSNorm, then the Q/K/V projections), and in the drop-in build
    // the attention of that query over the cache the forward calls left
    const int qd = heads * head_dim, kvd = kv_heads * head_dim;
    half *xin = upload(xd_h), *n = nullptr, *q = nullptr, *k = nullptr, *v = nullptr;
    HCHECK(cudaMalloc(&n, hidden * sizeof(half)));
    HCHECK(cudaMalloc(&q, qd * sizeof(half)));
    HCHECK(cudaMalloc(&k, kvd * sizeof(half)));
    HCHECK(cudaMalloc(&v, kvd * sizeof(half)));
    kernels::rmsnorm(xin, w.rms_att_weight, n, 1, hidden, c.rms_norm_eps);
    kernels::w8a16_matmul(n, w.wq.data, w.wq.scales, q, 1, qd, hidden, group);
    kernels::w8a16_matmul(n, w.wk.data, w.wk.scales, k, 1, kvd, hidden, group);
    kernels::w8a16_matmul(n, w.wv.data, w.wv.scales, v, 1, kvd, hidden, group);
    HCHECK(cudaDeviceSynchronize());
    d.dev("probe_norm", 'h', n, hidden);
    d.dev("probe_q", 'h', q, qd);
    d.dev("probe_k", 'h', k, kvd);
    d.dev("probe_v", 'h', v, kvd);
#ifdef TLLM_DROP_IN
    // (the decode token appended, not yet advanced)
    half *o = nullptr;
    HCHECK(cudaMalloc(&o, qd * sizeof(half)));
    if (cache->decodeAttention(0, q, o, {sid}).isErr()) return 7;
    HCHECK(cudaDeviceSynchronize());
    d.dev("probe_attn", 'h', o, qd);
#endif
    HCHECK(cudaFree(xp));
    HCHECK(cudaFree(xd));
    return 0;
}

#ifdef TLLM_DROP_IN
int run_batch(char **a, int nlens) {
    const int hidden = std::atoi(a[0]), heads = std::atoi(a[1]), kv_heads = std::atoi(a[2]),
              head_dim = std::atoi(a[3]), inter = std::atoi(a[4]), group = std::atoi(a[5]);
    const uint64_t seed = std::strtoull(a[6], nullptr, 10);
    Dump d(a[7]);
    std::vector<int> lens;
    int max_p = 0;
    for (int i = 0; i < nlens; ++i) {
        lens.push_back(std::atoi(a[8 + i]));
        max_p = std::max(max_p, lens.back());
    }
    const int B = nlens;
    const ModelConfig c = model_config(1, hidden, heads, kv_heads, head_dim, inter, 32, max_p + 8);
    TransformerWeights w = layer_weights(c, group, seed, 0);
    TransformerLayer layer(0, w, c);
    auto batched = make_cache(c, 1, B), single = make_cache(c, 1, B);
    std::vector<int> sb, ss;
    dump_layer(d, w, hidden);
    for (int i = 0; i < B; ++i) {
        const auto xh = random_half((size_t)lens[i] * hidden, -1.0, 1.0, seed, 10 + i);
        d.put("prompt" + std::to_string(i), 'h', xh.data(), xh.size());
        for (int pass = 0; pass < 2; ++pass) {
            KVCacheManager &cache = pass ? *single : *batched;
            const int sid = seq_of(cache, lens[i] + 1);
            (pass ? ss : sb).push_back(sid);
            half *x = upload(xh);
            layer.forwardPrefill(x, cache, sid, lens[i]);
            HCHECK(cudaDeviceSynchronize());
            HCHECK(cudaFree(x));
            if (cache.advanceSeqLen(sid, lens[i]).isErr()) return 5;
        }
    }
    const auto rows_h = random_half((size_t)B * hidden, -1.0, 1.0, seed, 3);
    d.put("rows_in", 'h', rows_h.data(), rows_h.size());
    half *rows = upload(rows_h);
    layer.forwardBatch(rows, *batched, sb);
    HCHECK(cudaDeviceSynchronize());
    d.dev("rows_batched", 'h', rows, (size_t)B * hidden);
    std::vector<half> one(hidden);
    std::vector<half> singles((size_t)B * hidden);
    for (int i = 0; i < B; ++i) {
        half *x = upload(std::vector<half>(rows_h.begin() + (size_t)i * hidden, rows_h.begin() + (size_t)(i + 1) * hidden));
        layer.forward(x, *single, ss[i], lens[i]);
        HCHECK(cudaDeviceSynchronize());
        HCHECK(cudaMemcpy(singles.data() + (size_t)i * hidden, x, hidden * sizeof(half), cudaMemcpyDeviceToHost));
        HCHECK(cudaFree(x));
    }
    d.put("rows_single", 'h', singles.data(), singles.size());
    HCHECK(cudaFree(rows));
    return 0;
}
#endif

// Seeded model; its weights are written to `d` (layer l's under "L<l>.").
std::unique_ptr<InferenceEngine> make_engine(const ModelConfig &c, int group, uint64_t seed, Dump *d) {
    ModelWeights mw;
    mw.token_embedding = upload(random_half((size_t)c.vocab_size * c.hidden_dim, -1.0, 1.0, seed, 7));
    for (int l = 0; l < c.num_layers; ++l) mw.layers.push_back(layer_weights(c, group, seed, l));
    mw.final_norm_weight = upload(random_half(c.hidden_dim, 0.8, 1.2, seed, 8));
    mw.lm_head = random_weight(c.hidden_dim, c.vocab_size, group, seed, 9);
    d->dev("embedding", 'h', mw.token_embedding, (size_t)c.vocab_size * c.hidden_dim);
    d->dev("final_norm", 'h', mw.final_norm_weight, c.hidden_dim);
    dump_weight(*d, "lm_head", mw.lm_head);
    for (int l = 0; l < c.num_layers; ++l) {
        const TransformerWeights &w = mw.layers[l];
        const std::string p = "L" + std::to_string(l) + ".";
        for (auto [name, q] : {std::pair<const char *, const QuantizedWeight *>{"wq", &w.wq}, {"wk", &w.wk},
                               {"wv", &w.wv}, {"wo", &w.wo}, {"w1", &w.w1}, {"w2", &w.w2}, {"w3", &w.w3}})
            dump_weight(*d, p + name, *q);
        d->dev(p + "rms_att", 'h', w.rms_att_weight, c.hidden_dim);
        d->dev(p + "rms_ffn", 'h', w.rms_ffn_weight, c.hidden_dim);
    }
    return std::make_unique<InferenceEngine>(c, std::move(mw));
}

GenerationConfig greedy(int max_new) {
    GenerationConfig g;
    g.max_new_tokens = max_new;
    g.do_sample = false;
    return g;
}

int run_generate(char **a, int argc_rest, bool batch) {
    const int layers = std::atoi(a[0]), hidden = std::atoi(a[1]), heads = std::atoi(a[2]),
              kv_heads = std::atoi(a[3]), head_dim = std::atoi(a[4]), inter = std::atoi(a[5]),
              vocab = std::atoi(a[6]), group = std::atoi(a[7]), max_seq = std::atoi(a[8]);
    const uint64_t seed = std::strtoull(a[9], nullptr, 10);
    const int max_new = std::atoi(a[10]);
    Dump d(a[11]);
    const ModelConfig c = model_config(layers, hidden, heads, kv_heads, head_dim, inter, vocab, max_seq);
    auto engine = make_engine(c, group, seed, &d);
    std::vector<std::vector<int>> prompts;
    int i = 12;
    if (!batch) {
        prompts.emplace_back();
        for (; i < 12 + argc_rest; ++i) prompts[0].push_back(std::atoi(a[i]));
    } else {
        std::vector<int> lens;
        for (; i < 12 + argc_rest && std::strcmp(a[i], "--") != 0; ++i) lens.push_back(std::atoi(a[i]));
        ++i;
        for (int n : lens) {
            prompts.emplace_back();
            for (int k = 0; k < n; ++k) prompts.back().push_back(std::atoi(a[i++]));
        }
    }
    for (size_t p = 0; p < prompts.size(); ++p) {
        auto r = engine->generate(prompts[p], greedy(max_new));
        if (r.isErr()) {
            std::fprintf(stderr, "generate: %s\n", r.error().c_str());
            return 6;
        }
        d.put("tokens" + std::to_string(p), 'i', r.value().data(), r.value().size());
    }
#ifdef TLLM_DROP_IN
    if (batch) {
        auto r = engine->generateBatch(prompts, greedy(max_new));
        if (r.isErr()) {
            std::fprintf(stderr, "generateBatch: %s\n", r.error().c_str());
            return 6;
        }
        for (size_t p = 0; p < prompts.size(); ++p)
            d.put("batch_tokens" + std::to_string(p), 'i', r.value()[p].data(), r.value()[p].size());
    }
#endif
    return 0;
}

}  // namespace

int main(int argc, char **argv) {
    if (argc < 2) {
        std::fprintf(stderr, "usage: %s layer|batch|generate|generate_batch ...\n", argv[0]);
        return 1;
    }
    const std::string mode = argv[1];
    if (mode == "layer" && argc == 11) return run_layer(argv + 2);
#ifdef TLLM_DROP_IN
    if (mode == "batch" && argc > 10) return run_batch(argv + 2, argc - 10);
    if (mode == "generate_batch" && argc > 14) return run_generate(argv + 2, argc - 14, true);
#endif
    if (mode == "generate" && argc > 14) return run_generate(argv + 2, argc - 14, false);
    std::fprintf(stderr, "bad arguments for mode %s (or mode not in this build)\n", mode.c_str());
    return 1;
}
