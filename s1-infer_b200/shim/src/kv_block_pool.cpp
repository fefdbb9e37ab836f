// kv_block_pool.cpp -- KVBlockPool of s1-infer on the B200 engine.
//
// Each method maps to the reference method of the same name
// (src/infer/kv_block_pool.cpp) through the C ABI: bookkeeping on the host,
// K/V bytes in device memory.  Calls are synchronous on the legacy default
// stream, like the reference's.
#include "infer/kv_block_pool.h"

#include <cuda_runtime.h>

#include <mutex>
#include <stdexcept>
#include <string>

#include "s1kv.h"
#include "shim_internal.h"

namespace s1kv_shim {

[[noreturn]] void raise(int status, const char* what) {
    std::string msg = s1kv_last_error();
    if (msg.empty()) msg = what;
    throw std::runtime_error(msg);
}

void check(int status, const char* what) {
    if (status != S1KV_OK) raise(status, what);
}

void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// Views carry the device storage address; GQA_attention_paged maps it back
// to the owning pool.
static std::mutex g_mu;
static std::unordered_map<const void*, const KVBlockPool*> g_views;

void register_pool(const void* base, const KVBlockPool* pool) {
    std::lock_guard<std::mutex> g(g_mu);
    if (pool) g_views[base] = pool;
    else g_views.erase(base);
}

const KVBlockPool* pool_of(const void* base) {
    std::lock_guard<std::mutex> g(g_mu);
    auto it = g_views.find(base);
    return it == g_views.end() ? nullptr : it->second;
}

DeviceBuffer::~DeviceBuffer() {
    if (p) cudaFree(p);
}

void* DeviceBuffer::get(size_t bytes) {
    if (bytes > cap) {
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
        cuda_check(cudaMalloc(&p, bytes), "cudaMalloc");
        cap = bytes;
    }
    return p;
}

}  // namespace s1kv_shim

using namespace s1kv_shim;

KVBlockPool::KVBlockPool(size_t num_heads, size_t head_dim, size_t max_blocks, size_t block_size)
    : num_heads_(num_heads), head_dim_(head_dim), block_size_(block_size) {
    s1kv_pool_desc d{};
    d.num_layers = 1;
    d.num_kv_heads = (int32_t)num_heads;
    d.head_dim = (int32_t)head_dim;
    d.block_size = (int32_t)block_size;
    d.max_blocks = (int64_t)max_blocks;
    d.dtype = S1KV_DTYPE_F32;
    int dev = 0;
    cudaGetDevice(&dev);
    check(s1kv_pool_create(&d, dev, &pool_), "KVBlockPool: pool creation failed");
    void *k = nullptr, *v = nullptr;
    check(s1kv_pool_storage(pool_, 0, &k, &v), "KVBlockPool: storage");
    register_pool(k, this);
    register_pool(v, this);
}

KVBlockPool::KVBlockPool(KVBlockPool&& o) noexcept
    : pool_(o.pool_), num_heads_(o.num_heads_), head_dim_(o.head_dim_), block_size_(o.block_size_),
      tables_(std::move(o.tables_)) {
    o.pool_ = nullptr;
    void *k = nullptr, *v = nullptr;
    if (pool_ && s1kv_pool_storage(pool_, 0, &k, &v) == S1KV_OK) {
        register_pool(k, this);
        register_pool(v, this);
    }
}

KVBlockPool::~KVBlockPool() {
    if (!pool_) return;
    void *k = nullptr, *v = nullptr;
    if (s1kv_pool_storage(pool_, 0, &k, &v) == S1KV_OK) {
        register_pool(k, nullptr);
        register_pool(v, nullptr);
    }
    s1kv_pool_destroy(pool_);
}

void KVBlockPool::refresh(size_t seq) const {
    if (!s1kv_seq_exists(pool_, seq)) {
        tables_.erase(seq);
        return;
    }
    int64_t n = 0;
    check(s1kv_block_table(pool_, seq, nullptr, 0, &n), "KVBlockPool: block table");
    std::vector<int32_t> t((size_t)n);
    check(s1kv_block_table(pool_, seq, t.data(), n, &n), "KVBlockPool: block table");
    auto& mirror = tables_[seq];
    mirror.assign(t.begin(), t.end());
}

// KVBlockPool::append (kv_block_pool.cpp:20-65): slots are reserved on the
// host; the tokens that fit are copied into the device pool; exhaustion
// throws afterwards, as the reference does.
void KVBlockPool::append(size_t seq, const TensorPtr& k, const TensorPtr& v) {
    const size_t T = k->shape()[0];
    const size_t row = num_heads_ * head_dim_;
    auto kc = k->is_contiguous() ? k : k->contiguous();
    auto vc = v->is_contiguous() ? v : v->contiguous();
    std::vector<int32_t> slots(T);
    int64_t done = 0;
    int st = s1kv_seq_reserve(pool_, seq, (int64_t)T, slots.data(), &done);
    refresh(seq);
    if (done > 0) {
        thread_local DeviceBuffer buf;
        const size_t bytes = (size_t)done * row * sizeof(float);
        char* d = (char*)buf.get(2 * bytes + (size_t)done * sizeof(int32_t) + 64);
        float* dk = (float*)d;
        float* dv = (float*)(d + bytes);
        int32_t* ds = (int32_t*)(d + 2 * bytes);
        cuda_check(cudaMemcpy(dk, kc->data().data() + kc->offset(), bytes, cudaMemcpyHostToDevice), "append");
        cuda_check(cudaMemcpy(dv, vc->data().data() + vc->offset(), bytes, cudaMemcpyHostToDevice), "append");
        cuda_check(cudaMemcpy(ds, slots.data(), (size_t)done * sizeof(int32_t), cudaMemcpyHostToDevice), "append");
        check(s1kv_append(pool_, 0, dk, dv, ds, done, nullptr), "KVBlockPool: append");
        cuda_check(cudaDeviceSynchronize(), "append");
    }
    if (st != S1KV_OK) raise(st, "KVBlockPool: No free blocks available");
}

TensorPtr KVBlockPool::gather(size_t seq, int which) const {
    if (!s1kv_seq_exists(pool_, seq)) throw std::runtime_error("KVBlockPool: Sequence ID not found");
    const size_t len = (size_t)s1kv_seq_length(pool_, seq);
    auto out = Tensor::create({len, num_heads_, head_dim_});
    if (len) {
        thread_local DeviceBuffer buf;
        const size_t bytes = out->numel() * sizeof(float);
        float* d = (float*)buf.get(bytes);
        check(s1kv_gather(pool_, 0, seq, which, d, nullptr), "KVBlockPool: gather");
        cuda_check(cudaMemcpy(out->mutable_data().data(), d, bytes, cudaMemcpyDeviceToHost), "gather");
    }
    return out;
}

TensorPtr KVBlockPool::get_k(size_t seq) const { return gather(seq, S1KV_K); }
TensorPtr KVBlockPool::get_v(size_t seq) const { return gather(seq, S1KV_V); }

size_t KVBlockPool::length(size_t seq) const { return (size_t)s1kv_seq_length(pool_, seq); }

void KVBlockPool::remove(size_t seq) {
    check(s1kv_seq_remove(pool_, seq), "KVBlockPool: Sequence ID not found");
    tables_.erase(seq);
}

void KVBlockPool::truncate(size_t seq, size_t keep) {
    check(s1kv_seq_truncate(pool_, seq, (int64_t)keep), "KVBlockPool: Sequence ID not found");
    refresh(seq);
}

KVView KVBlockPool::view(size_t seq, int which) const {
    if (!s1kv_seq_exists(pool_, seq)) throw std::runtime_error("Sequence ID not found");
    refresh(seq);
    void *k = nullptr, *v = nullptr;
    check(s1kv_pool_storage(pool_, 0, &k, &v), "KVBlockPool: storage");
    return KVView{(const scalar_t*)(which == S1KV_K ? k : v), &tables_.at(seq), block_size_,
                  (size_t)s1kv_seq_length(pool_, seq)};
}

KVView KVBlockPool::get_k_view(size_t seq) const { return view(seq, S1KV_K); }
KVView KVBlockPool::get_v_view(size_t seq) const { return view(seq, S1KV_V); }

bool KVBlockPool::sequence_of(const std::vector<size_t>* table, size_t* seq) const {
    for (const auto& kv : tables_) {
        if (&kv.second == table) {
            *seq = kv.first;
            return true;
        }
    }
    return false;
}
