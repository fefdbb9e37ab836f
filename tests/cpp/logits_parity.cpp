// logits_parity.cpp -- final logits of s1-infer's own model code over a
// seeded random-weight model (test infrastructure).
//
// The reference's test tests/test_kv_cache_correctness.cpp:28-114 runs an
// 8-step cached greedy decode of the real superwhisper/s1-mini weights
// through model_forward (src/model/model.cpp:83-130, layer_forward
// src/nn/layer.cpp:5-111, self_attention src/nn/attention.cpp:241-291).
// Those weights are not available, so this program builds the same model
// shape (Qwen3-0.6B: 28 layers hard-wired in model_forward, hidden 1024,
// 16 query heads / 8 KV heads of 128, q/k RMSNorm, MLP 3072) with seeded
// random weights and runs the same loop: the prompt, then one token per
// step, the next token being the argmax of the last step's logits.
//
// oracle/Makefile links it twice, from the reference's sources where they
// lie: once with the reference's own KV path (KVBlockPool, apply_rope, the
// GQA functions -- all on the CPU), and once with those replaced by the
// B200 engine through the C++ shim (s1-infer_b200/shim).  The GPU test
// compares the two programs' logits.
//
//   logits_parity <f32|int8> <prompt_tokens> <steps> <vocab> <seed> <out.bin>
//
// f32 runs model_forward (pretransposed fp32 weights, contiguous
// GQA_attention over get_k/get_v); int8 runs model_forward_quantized
// (quantize_tensor of every projection and the LM head, as src/demo.cpp:48-52
// does, and GQA_attention_paged over the pool's block-table views).
//
// out.bin: int32 steps, int32 vocab, then per step int32 argmax and
// float32 logits[vocab].
#include <dlfcn.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "core/quantized_tensor.h"
#include "core/tensor.h"
#include "infer/kv_block_pool.h"
#include "model/model.h"

namespace {

constexpr size_t kLayers = 28, kHidden = 1024, kQDim = 16 * 128, kKVDim = 8 * 128, kMlp = 3072, kHeadDim = 128;

uint64_t splitmix64(uint64_t& s) {
    uint64_t z = (s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Uniform values of standard deviation `std` around `mean` (a uniform on
// [-a, a] has standard deviation a / sqrt(3)); one stream per tensor.
TensorPtr random_tensor(std::vector<size_t> shape, uint64_t seed, float mean, float std) {
    auto t = Tensor::create(shape);
    std::vector<scalar_t>& d = t->mutable_data();
    uint64_t s = seed * 0x2545F4914F6CDD1Dull + 1;
    const float a = std * 1.7320508f;
    for (size_t i = 0; i < d.size(); i++) {
        const float u = (float)((splitmix64(s) >> 40) * (1.0 / 16777216.0));  // [0, 1)
        d[i] = mean + a * (2.0f * u - 1.0f);
    }
    return t;
}

// HF layout ([out, in]) as load_safetensors returns it; pretranspose_weights
// (src/model/model.cpp:8-33) turns the projections and the LM head into
// [in, out].
std::map<std::string, TensorPtr> make_weights(size_t vocab, uint64_t seed) {
    std::map<std::string, TensorPtr> w;
    uint64_t id = seed * 1000;
    auto proj = [&](size_t out, size_t in) { return random_tensor({out, in}, ++id, 0.0f, 1.0f / std::sqrt((float)in)); };
    auto norm = [&](size_t n) { return random_tensor({n}, ++id, 1.0f, 0.1f); };
    w["model.embed_tokens.weight"] = random_tensor({vocab, kHidden}, ++id, 0.0f, 0.5f);
    for (size_t l = 0; l < kLayers; l++) {
        const std::string p = "model.layers." + std::to_string(l) + ".";
        w[p + "input_layernorm.weight"] = norm(kHidden);
        w[p + "self_attn.q_proj.weight"] = proj(kQDim, kHidden);
        w[p + "self_attn.k_proj.weight"] = proj(kKVDim, kHidden);
        w[p + "self_attn.v_proj.weight"] = proj(kKVDim, kHidden);
        w[p + "self_attn.o_proj.weight"] = proj(kHidden, kQDim);
        w[p + "self_attn.q_norm.weight"] = norm(kHeadDim);
        w[p + "self_attn.k_norm.weight"] = norm(kHeadDim);
        w[p + "post_attention_layernorm.weight"] = norm(kHidden);
        w[p + "mlp.gate_proj.weight"] = proj(kMlp, kHidden);
        w[p + "mlp.up_proj.weight"] = proj(kMlp, kHidden);
        w[p + "mlp.down_proj.weight"] = proj(kHidden, kMlp);
    }
    w["model.norm.weight"] = norm(kHidden);
    w["lm_head.weight"] = proj(vocab, kHidden);
    return pretranspose_weights(w);
}

int64_t engine_launches() {
    // present only when the engine is linked in (the shim build)
    using fn_t = int64_t (*)();
    auto fn = reinterpret_cast<fn_t>(dlsym(RTLD_DEFAULT, "s1kv_launch_count"));
    return fn ? fn() : -1;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc != 7) {
        std::fprintf(stderr, "usage: %s <f32|int8> <prompt_tokens> <steps> <vocab> <seed> <out.bin>\n", argv[0]);
        return 2;
    }
    const bool quant = std::strcmp(argv[1], "int8") == 0;
    const size_t prompt = std::strtoul(argv[2], nullptr, 10), steps = std::strtoul(argv[3], nullptr, 10);
    const size_t vocab = std::strtoul(argv[4], nullptr, 10);
    const uint64_t seed = std::strtoull(argv[5], nullptr, 10);
    auto weights = make_weights(vocab, seed);
    std::map<std::string, QuantizedTensor> qweights;
    if (quant) {
        for (const auto& [name, t] : weights)
            if (name == "lm_head.weight" || (t->shape().size() == 2 && name != "model.embed_tokens.weight"))
                qweights[name] = quantize_tensor(*t);
    }
    // the prompt: seeded token ids
    std::vector<int> ids(prompt);
    uint64_t s = seed + 77;
    for (auto& t : ids) t = (int)(splitmix64(s) % vocab);

    // the loop of tests/test_kv_cache_correctness.cpp:39-72
    std::vector<KVBlockPool> caches;
    caches.reserve(kLayers);
    for (size_t l = 0; l < kLayers; l++) caches.emplace_back(8, 128, /*max_blocks=*/128, /*block_size=*/16);
    const int64_t launches0 = engine_launches();
    FILE* f = std::fopen(argv[6], "wb");
    if (!f) return 3;
    const int32_t hdr[2] = {(int32_t)steps, (int32_t)vocab};
    std::fwrite(hdr, sizeof(int32_t), 2, f);
    std::vector<int> next = ids;
    for (size_t step = 0; step < steps; step++) {
        TensorPtr logits = quant ? model_forward_quantized(next, weights, qweights, caches, 0, true)
                                 : model_forward(next, weights, caches, 0, true);
        const std::vector<scalar_t>& d = logits->data();
        int32_t best = 0;
        for (size_t j = 1; j < vocab; j++)
            if (d[j] > d[best]) best = (int32_t)j;
        std::fwrite(&best, sizeof(int32_t), 1, f);
        std::fwrite(d.data(), sizeof(float), vocab, f);
        std::printf("step %zu: argmax %d logit %.6f\n", step, best, d[best]);
        next = {best};
    }
    std::fclose(f);
    const int64_t launches1 = engine_launches();
    std::printf("cache length %zu\n", caches[0].length(0));
    if (launches0 >= 0) std::printf("engine launches %lld\n", (long long)(launches1 - launches0));
    return 0;
}
