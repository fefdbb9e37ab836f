// test_shim.cpp -- the C++ reference-interface shim (KVBlockPool, KVView,
// GQA_attention(_paged), apply_rope, quantize_tensor / matmul_quantized) on
// the GPU, against the known answers of the reference's own tests:
// tests/test_kv_block_pool.cpp:6-207, tests/test_attention.cpp:5-120,
// tests/test_rope.cpp:5-34, tests/test_quantized_tensor.cpp:5-75.
// Exit status 0 when every check passes.
#include <cmath>
#include <cstdio>
#include <functional>
#include <memory>
#include <stdexcept>
#include <vector>

#include "core/quantized_tensor.h"
#include "infer/kv_block_pool.h"
#include "nn/RoPE.h"
#include "nn/attention.h"

static int g_checks = 0, g_failed = 0;

#define EXPECT(cond)                                                        \
    do {                                                                    \
        g_checks++;                                                         \
        if (!(cond)) {                                                      \
            g_failed++;                                                     \
            std::printf("FAILED %s:%d: %s\n", __FILE__, __LINE__, #cond);   \
        }                                                                   \
    } while (0)

static bool near(float a, float b, float rel = 1e-5f, float abs_tol = 1e-6f) {
    return std::fabs(a - b) <= abs_tol + rel * std::fmax(std::fabs(a), std::fabs(b));
}

static bool throws(const std::function<void()>& f) {
    try {
        f();
    } catch (const std::runtime_error&) {
        return true;
    }
    return false;
}

static TensorPtr col(std::vector<float> v) {
    size_t n = v.size();
    return std::make_shared<Tensor>(std::vector<size_t>{n, 1, 1}, std::move(v));
}

static void pool_cases() {
    {  // round trip inside one block
        KVBlockPool pool(1, 2, 4, 4);
        auto k = std::make_shared<Tensor>(std::vector<size_t>{3, 1, 2}, std::vector<float>{1, 2, 3, 4, 5, 6});
        auto v = std::make_shared<Tensor>(std::vector<size_t>{3, 1, 2}, std::vector<float>{10, 20, 30, 40, 50, 60});
        pool.append(0, k, v);
        auto ok = pool.get_k(0), ov = pool.get_v(0);
        EXPECT(ok->shape()[0] == 3 && ok->shape()[1] == 1 && ok->shape()[2] == 2);
        EXPECT(ok->at({0, 0, 0}) == 1.0f && ok->at({0, 0, 1}) == 2.0f && ok->at({2, 0, 0}) == 5.0f &&
               ok->at({2, 0, 1}) == 6.0f);
        EXPECT(ov->at({0, 0, 0}) == 10.0f && ov->at({2, 0, 1}) == 60.0f);
    }
    {  // 5 tokens over three blocks of 2
        KVBlockPool pool(1, 1, 4, 2);
        pool.append(0, col({1, 2, 3, 4, 5}), col({10, 20, 30, 40, 50}));
        auto ok = pool.get_k(0);
        EXPECT(ok->shape()[0] == 5);
        for (size_t i = 0; i < 5; i++) EXPECT(ok->at({i, 0, 0}) == (float)(i + 1));
    }
    {  // a partial block continues across calls
        KVBlockPool pool(1, 1, 4, 4);
        pool.append(0, col({1, 2, 3}), col({1, 2, 3}));
        pool.append(0, col({4, 5, 6}), col({4, 5, 6}));
        auto ok = pool.get_k(0);
        EXPECT(ok->shape()[0] == 6);
        for (size_t i = 0; i < 6; i++) EXPECT(ok->at({i, 0, 0}) == (float)(i + 1));
    }
    {  // remove frees for reuse; exhaustion throws
        KVBlockPool pool(1, 1, 1, 2);
        pool.append(0, col({1, 2}), col({1, 2}));
        EXPECT(throws([&] { pool.append(1, col({1, 2}), col({1, 2})); }));
        pool.remove(0);
        EXPECT(!throws([&] { pool.append(1, col({1, 2}), col({1, 2})); }));
        auto ok = pool.get_k(1);
        EXPECT(ok->at({0, 0, 0}) == 1.0f && ok->at({1, 0, 0}) == 2.0f);
        EXPECT(throws([&] { pool.get_k(0); }));
    }
    {  // unknown ids
        KVBlockPool pool(1, 1, 4, 2);
        EXPECT(throws([&] { pool.get_k(99); }));
        EXPECT(pool.length(0) == 0);
        pool.append(0, col({1, 2, 3}), col({1, 2, 3}));
        EXPECT(pool.length(0) == 3);
    }
    {  // truncate mid-block, then append
        KVBlockPool pool(1, 1, 4, 4);
        std::vector<float> vals;
        for (int i = 1; i <= 10; i++) vals.push_back((float)i);
        pool.append(0, col(vals), col(vals));
        pool.truncate(0, 5);
        EXPECT(pool.length(0) == 5);
        pool.append(0, col({100, 101}), col({100, 101}));
        auto ok = pool.get_k(0);
        EXPECT(ok->shape()[0] == 7 && ok->at({5, 0, 0}) == 100.0f && ok->at({6, 0, 0}) == 101.0f &&
               ok->at({4, 0, 0}) == 5.0f);
    }
    {  // truncate at a block multiple frees exactly one block
        KVBlockPool pool(1, 1, 4, 4);
        std::vector<float> vals;
        for (int i = 1; i <= 10; i++) vals.push_back((float)i);
        pool.append(0, col(vals), col(vals));
        pool.truncate(0, 8);
        EXPECT(pool.length(0) == 8);
        EXPECT(!throws([&] { pool.append(1, col({1, 2, 3, 4, 5}), col({1, 2, 3, 4, 5})); }));
    }
    {  // truncate no-op and truncate to 0
        KVBlockPool pool(1, 1, 4, 4);
        pool.append(0, col({1, 2, 3}), col({1, 2, 3}));
        pool.truncate(0, 10);
        pool.truncate(0, 3);
        EXPECT(pool.length(0) == 3);
        pool.truncate(0, 0);
        EXPECT(pool.length(0) == 0);
        EXPECT(!throws([&] { pool.append(1, col(std::vector<float>(13, 9.0f)), col(std::vector<float>(13, 9.0f))); }));
    }
}

static void attention_cases() {
    {  // reshape_to_heads keeps values
        auto flat = std::make_shared<Tensor>(std::vector<size_t>{2, 4}, std::vector<float>{1, 2, 3, 4, 5, 6, 7, 8});
        auto h = reshape_to_heads(flat, 2, 2);
        EXPECT(h->shape()[0] == 2 && h->shape()[1] == 2 && h->shape()[2] == 2);
        EXPECT(h->at({0, 1, 0}) == 3.0f && h->at({1, 1, 1}) == 8.0f);
    }
    {  // causal mask: token 0 sees itself, token 1 averages tied scores
        auto Q = std::make_shared<Tensor>(std::vector<size_t>{2, 2, 2}, std::vector<float>(8, 1.0f));
        auto K = std::make_shared<Tensor>(std::vector<size_t>{2, 1, 2}, std::vector<float>{1, 0, 1, 0});
        auto V = std::make_shared<Tensor>(std::vector<size_t>{2, 1, 2}, std::vector<float>{2, 4, 6, 8});
        auto out = GQA_attention(Q, K, V, 2, 1, 2);
        EXPECT(near(out->at({0, 0, 0}), 2) && near(out->at({0, 1, 1}), 4));
        EXPECT(near(out->at({1, 0, 0}), 4) && near(out->at({1, 1, 1}), 6));
    }
    {  // paged == contiguous on scattered blocks [3, 1, 0]
        KVBlockPool pool(1, 2, 4, 2);
        auto filler = std::make_shared<Tensor>(std::vector<size_t>{2, 1, 2}, std::vector<float>(4, 0.0f));
        pool.append(1, filler, filler);
        pool.append(2, filler, filler);
        pool.remove(1);
        auto K = std::make_shared<Tensor>(std::vector<size_t>{5, 1, 2},
                                          std::vector<float>{1, -1, 2, -2, 3, -3, 4, -4, 5, -5});
        auto V = std::make_shared<Tensor>(std::vector<size_t>{5, 1, 2},
                                          std::vector<float>{10, 100, 20, 200, 30, 300, 40, 400, 50, 500});
        pool.append(0, K, V);
        KVView kv = pool.get_k_view(0), vv = pool.get_v_view(0);
        EXPECT(kv.block_table->size() == 3 && (*kv.block_table)[0] == 3 && (*kv.block_table)[1] == 1 &&
               (*kv.block_table)[2] == 0);
        std::vector<float> q;
        for (int i = 1; i <= 20; i++) q.push_back(0.1f * i);
        auto Q = std::make_shared<Tensor>(std::vector<size_t>{5, 2, 2}, q);
        auto expected = GQA_attention(Q, pool.get_k(0), pool.get_v(0), 2, 1, 2);
        auto actual = GQA_attention_paged(Q, kv, vv, 2, 1, 2);
        EXPECT(actual->shape() == expected->shape());
        for (size_t i = 0; i < 5; i++)
            for (size_t h = 0; h < 2; h++)
                for (size_t d = 0; d < 2; d++) EXPECT(near(actual->at({i, h, d}), expected->at({i, h, d}), 2e-5f));
    }
}

static void rope_cases() {
    auto x = std::make_shared<Tensor>(std::vector<size_t>{1, 4}, std::vector<float>{1, 2, 3, 4});
    auto y = apply_rope(x, 0);
    for (size_t j = 0; j < 4; j++) EXPECT(y->at({0, j}) == x->at({0, j}));
    auto x1 = std::make_shared<Tensor>(std::vector<size_t>{1, 4}, std::vector<float>{1, 0, 1, 0});
    auto y1 = apply_rope(x1, 1);
    EXPECT(near(y1->at({0, 0}), -0.30117f, 1e-3f) && near(y1->at({0, 2}), 1.38177f, 1e-3f));
    EXPECT(std::fabs(y1->at({0, 1})) < 1e-3f && std::fabs(y1->at({0, 3})) < 1e-3f);
}

static void quantized_cases() {
    // tests/test_quantized_tensor.cpp:5-23: recovered within 2% of each value
    {
        Tensor t(std::vector<size_t>{2, 3}, std::vector<float>{1.0f, -2.0f, 0.5f, 10.0f, -20.0f, 5.0f});
        QuantizedTensor qt = quantize_tensor(t);
        EXPECT(qt.rows == 2 && qt.cols == 3);
        for (size_t r = 0; r < 2; r++)
            for (size_t c = 0; c < 3; c++) EXPECT(near(dequantize(qt, r, c), t.at({r, c}), 0.02f));
    }
    // :25-39: each row its own scale
    {
        auto t = std::make_shared<Tensor>(std::vector<size_t>{2, 2}, std::vector<float>{0.01f, 0.02f, 1.0f, 2.0f});
        QuantizedTensor qt = quantize_tensor(*t);
        EXPECT(!near(qt.scales[0], qt.scales[1], 1e-3f));
        EXPECT(near(dequantize(qt, 0, 0), 0.01f, 0.02f) && near(dequantize(qt, 0, 1), 0.02f, 0.02f));
    }
    // :41-49: an all-zero row gives zeros, not NaN
    {
        auto t = std::make_shared<Tensor>(std::vector<size_t>{1, 2}, std::vector<float>{0.0f, 0.0f});
        QuantizedTensor qt = quantize_tensor(*t);
        EXPECT(dequantize(qt, 0, 0) == 0.0f && dequantize(qt, 0, 1) == 0.0f);
    }
    // :51-75: blocked product close to the float product (5% of max), with a
    // tail that is not a multiple of 8 (index expressions signed here, so all
    // values stay O(1)); here on a column range as well
    {
        const size_t M = 2, K = 80, N = 88;
        std::vector<float> a(M * K), b(K * N);
        for (size_t i = 0; i < M * K; i++) a[i] = 0.01f * (float)((int)((i * 13) % 200) - 100);
        for (size_t i = 0; i < K * N; i++) b[i] = 0.01f * (float)((int)((i * 7) % 200) - 100);
        auto bt = std::make_shared<Tensor>(std::vector<size_t>{K, N}, b);
        QuantizedTensor qb = quantize_tensor(*bt);
        std::vector<double> ref(M * N, 0.0);
        double mx = 0;
        for (size_t i = 0; i < M; i++)
            for (size_t j = 0; j < N; j++) {
                for (size_t k = 0; k < K; k++) ref[i * N + j] += (double)a[i * K + k] * b[k * N + j];
                mx = std::fmax(mx, std::fabs(ref[i * N + j]));
            }
        std::vector<float> out(M * N, -1.0f);
        matmul_quantized_range_blocked(a.data(), qb, out.data(), M, K, N, 0, N);
        for (size_t i = 0; i < M * N; i++) EXPECT(std::fabs(out[i] - ref[i]) < 0.05 * mx);
        std::vector<float> part(M * N, -7.0f);
        matmul_quantized_range_blocked(a.data(), qb, part.data(), M, K, N, 40, 88);
        for (size_t i = 0; i < M; i++)
            for (size_t j = 0; j < N; j++) EXPECT(j < 40 ? part[i * N + j] == -7.0f : part[i * N + j] == out[i * N + j]);
        auto x = std::make_shared<Tensor>(std::vector<size_t>{M, K}, a);
        auto y = matmul_quantized(x, qb);
        EXPECT(y->shape() == (std::vector<size_t>{M, N}));
        for (size_t i = 0; i < M * N; i++) EXPECT(y->data()[i] == out[i]);
    }
}

int main() {
    pool_cases();
    attention_cases();
    rope_cases();
    quantized_cases();
    std::printf("%d checks, %d failed\n", g_checks, g_failed);
    return g_failed ? 1 : 0;
}
