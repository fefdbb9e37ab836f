// rope_host.cpp -- the device RoPE cos/sin table, filled on the host.
//
// The appended K bytes must equal the reference's bit for bit, and the
// reference rotates with the host C library's powf/cosf/sinf
// (src/nn/RoPE.cpp:22-24); the device's transcendental functions round
// differently.  So the (cos, sin) pair of every (position, pair index) is
// computed here with exactly the reference's float expression and uploaded
// once per (device, head_dim, base); the table grows by doubling when a
// longer position is needed.  Compiled with -ffp-contract=off.
#include <cmath>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "internal.h"

namespace s1kv {

namespace {

struct RopeKey {
    int device, D;
    uint32_t base_bits;
    bool operator==(const RopeKey& o) const { return device == o.device && D == o.D && base_bits == o.base_bits; }
};

struct RopeKeyHash {
    size_t operator()(const RopeKey& k) const {
        return (size_t)k.device * 1000003u ^ (size_t)k.D * 131u ^ (size_t)k.base_bits;
    }
};

struct RopeTable {
    float2* d = nullptr;
    int64_t cap = 0;
};

// theta = (float)pos / powf(base, (float)(2j) / (float)D); then cosf / sinf
// of theta (src/nn/RoPE.cpp:22-24, std::pow/cos/sin on float arguments).
void fill_rows(float2* h, int64_t p0, int64_t p1, int D, float base) {
    const int half = D / 2;
    std::vector<float> denom(half);
    for (int j = 0; j < half; j++) denom[j] = std::pow(base, static_cast<float>(2 * j) / static_cast<float>(D));
    for (int64_t pos = p0; pos < p1; pos++) {
        for (int j = 0; j < half; j++) {
            float theta = static_cast<float>(pos) / denom[j];
            h[(pos - p0) * half + j] = make_float2(std::cos(theta), std::sin(theta));
        }
    }
}

}  // namespace

const float2* rope_table(int device, int D, float base, int64_t min_positions, int64_t* cap, cudaStream_t stream,
                         int* status) {
    (void)stream;
    static std::mutex mu;
    static std::unordered_map<RopeKey, RopeTable, RopeKeyHash> tables;
    std::lock_guard<std::mutex> g(mu);
    uint32_t bits;
    std::memcpy(&bits, &base, 4);
    RopeTable& t = tables[RopeKey{device, D, bits}];
    *status = S1KV_OK;
    if (t.d && t.cap >= min_positions) {
        *cap = t.cap;
        return t.d;
    }
    int64_t ncap = std::max<int64_t>(std::max<int64_t>(min_positions, 2 * t.cap), 4096);
    const int half = D / 2;
    std::vector<float2> h((size_t)(ncap - t.cap) * half);
    fill_rows(h.data(), t.cap, ncap, D, base);
    float2* nd = nullptr;
    // Growth is rare (doubling); synchronising keeps every in-flight kernel
    // off the old table before it is freed.
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMalloc(&nd, (size_t)ncap * half * sizeof(float2));
    if (e == cudaSuccess && t.d)
        e = cudaMemcpy(nd, t.d, (size_t)t.cap * half * sizeof(float2), cudaMemcpyDeviceToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy(nd + (size_t)t.cap * half, h.data(), h.size() * sizeof(float2), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        if (nd) cudaFree(nd);
        *status = cuda_error(e, "s1kv: RoPE table upload");
        return nullptr;
    }
    if (t.d) cudaFree(t.d);
    t.d = nd;
    t.cap = ncap;
    *cap = ncap;
    return t.d;
}

}  // namespace s1kv
