// pool.cpp -- host bookkeeping of the device-resident block pool and the
// C-ABI entry points for pool lifecycle, sequences and the prefix cache.
//
// Bookkeeping follows src/infer/kv_block_pool.cpp of s1-infer: a LIFO free
// list seeded 0..max_blocks-1 (ctor :6-18), block allocation when a table is
// empty or its last block is full (append :35-42), remove releasing blocks
// in table order (:148-161), truncate releasing tail blocks last-first
// (:163-190).  Block sharing (refcounts, fork, copy-on-write of a partial
// tail, prefix cache with LRU eviction) has no reference counterpart; its
// rules are stated at each function.  Every mutation that a kernel must see
// (block-table entries, copy-on-write copies) is queued here and applied on
// the device by s1kv_flush, which every kernel entry point runs first.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "internal.h"

namespace s1kv {

static thread_local std::string g_err;
std::atomic<int64_t> g_launches{0};

int set_error(int status, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return status;
}

int cuda_error(cudaError_t e, const char* what) {
    return set_error(e == cudaErrorMemoryAllocation ? S1KV_ENOMEM : S1KV_ECUDA, "%s: %s", what,
                     cudaGetErrorString(e));
}

namespace {
std::mutex g_word_mu;
std::unordered_map<int, int*> g_words;
}  // namespace

int* device_error_word(int device) {
    std::lock_guard<std::mutex> g(g_word_mu);
    auto it = g_words.find(device);
    if (it != g_words.end()) return it->second;
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
    cudaMemset(p, 0, sizeof(int));
    cudaDeviceSynchronize();
    g_words[device] = p;
    return p;
}

// The word of `device` if some call already created it, else NULL (no
// allocation).
static int* existing_error_word(int device) {
    std::lock_guard<std::mutex> g(g_word_mu);
    auto it = g_words.find(device);
    return it == g_words.end() ? nullptr : it->second;
}

// ---------------------------------------------------------------- stager --
int Stager::acquire(size_t bytes, StageSeg** out) {
    int pick = -1;
    for (int i = 0; i < kSegs && pick < 0; i++)
        if (!seg[(next + i) % kSegs].in_use) pick = (next + i) % kSegs;
    if (pick < 0) return set_error(S1KV_EINVAL, "s1kv: more than %d batches alive at once", kSegs - 1);
    StageSeg& s = seg[pick];
    next = (pick + 1) % kSegs;
    if (s.ev == nullptr) S1KV_CUDA(cudaEventCreateWithFlags(&s.ev, cudaEventDisableTiming));
    if (s.pending) {
        S1KV_CUDA(cudaEventSynchronize(s.ev));
        s.pending = false;
    }
    if (s.cap < bytes) {
        size_t cap = std::max<size_t>({bytes, 2 * s.cap, 64 << 10});
        if (s.h) cudaFreeHost(s.h);
        if (s.d) cudaFree(s.d);
        s.h = nullptr;
        s.d = nullptr;
        s.cap = 0;
        S1KV_CUDA(cudaHostAlloc((void**)&s.h, cap, cudaHostAllocDefault));
        S1KV_CUDA(cudaMalloc((void**)&s.d, cap));
        s.cap = cap;
    }
    s.in_use = true;
    *out = &s;
    return S1KV_OK;
}

int Stager::reserve(size_t bytes) {
    for (auto& s : seg) {
        if (s.h || s.d) continue;  // a fresh stager's segments only (pool creation)
        if (s.ev == nullptr) S1KV_CUDA(cudaEventCreateWithFlags(&s.ev, cudaEventDisableTiming));
        S1KV_CUDA(cudaHostAlloc((void**)&s.h, bytes, cudaHostAllocDefault));
        S1KV_CUDA(cudaMalloc((void**)&s.d, bytes));
        s.cap = bytes;
    }
    return S1KV_OK;
}

int Stager::release(StageSeg* s, cudaStream_t stream) {
    s->in_use = false;
    S1KV_CUDA(cudaEventRecord(s->ev, stream));
    s->pending = true;
    return S1KV_OK;
}

void Stager::destroy() {
    for (auto& s : seg) {
        if (s.pending && s.ev) cudaEventSynchronize(s.ev);
        if (s.h) cudaFreeHost(s.h);
        if (s.d) cudaFree(s.d);
        if (s.ev) cudaEventDestroy(s.ev);
        s = StageSeg{};
    }
}

// Grows geometrically (at least 2x, at least 16 MB) so that a workload whose
// size creeps up step by step reallocates a handful of times, not per step.
int DevBuf::ensure(size_t bytes) {
    if (cap >= bytes) return S1KV_OK;
    S1KV_CUDA(cudaDeviceSynchronize());
    if (p) cudaFree(p);
    p = nullptr;
    size_t c = std::max<size_t>({bytes + bytes / 4, 2 * cap, size_t(16) << 20});
    cap = 0;
    S1KV_CUDA(cudaMalloc(&p, c));
    cap = c;
    return S1KV_OK;
}

void DevBuf::destroy() {
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
}

// ------------------------------------------------------ block primitives --
static Seq* find_seq(s1kv_pool* p, uint64_t id) {
    auto it = p->seqs.find(id);
    return it == p->seqs.end() ? nullptr : &it->second;
}

static const Seq* find_seq(const s1kv_pool* p, uint64_t id) {
    auto it = p->seqs.find(id);
    return it == p->seqs.end() ? nullptr : &it->second;
}

static int64_t seq_len(const s1kv_pool* p, const Seq* s) {
    if (!s || s->table.empty()) return 0;
    return (int64_t)(s->table.size() - 1) * p->desc.block_size + s->tokens_in_last;
}

static void mark_dirty(s1kv_pool* p, uint64_t id, Seq* s, int64_t from) {
    if (s->synced > from) s->synced = from;
    p->dirty.push_back(id);
}

// sequences_[id] creates an empty entry on first use (kv_block_pool.cpp:28).
static int get_or_create(s1kv_pool* p, uint64_t id, Seq** out) {
    auto it = p->seqs.find(id);
    if (it != p->seqs.end()) {
        *out = &it->second;
        return S1KV_OK;
    }
    if (p->free_rows.empty())
        return set_error(S1KV_EINVAL, "s1kv: more than max_seqs=%d live sequences", p->desc.max_seqs);
    Seq s;
    s.row = p->free_rows.back();
    p->free_rows.pop_back();
    *out = &p->seqs.emplace(id, std::move(s)).first->second;
    return S1KV_OK;
}

static void cache_unregister(s1kv_pool* p, int32_t b) {
    if (!p->cached[b]) return;
    auto range = p->cache_map.equal_range(p->cache_entry[b].hash);
    for (auto it = range.first; it != range.second; ++it) {
        if (it->second == b) {
            p->cache_map.erase(it);
            break;
        }
    }
    p->cache_entry[b] = CacheEntry{};
    p->cached[b] = 0;
    p->num_cached--;
}

// Top of the LIFO free list (kv_block_pool.cpp:40-41); when it is empty,
// the least recently released zero-refcount cached block is evicted.
static int32_t alloc_block(s1kv_pool* p) {
    int32_t b;
    if (!p->free_list.empty()) {
        b = p->free_list.back();
        p->free_list.pop_back();
    } else if (!p->lru.empty()) {
        b = p->lru.front();
        p->lru.pop_front();
        p->in_lru[b] = 0;
        cache_unregister(p, b);
        p->evictions++;
    } else {
        return -1;
    }
    p->rc[b] = 1;
    return b;
}

// Drops a reference; at zero a cached block joins the LRU tail and any
// other block goes back on top of the free list.
static void release_block(s1kv_pool* p, int32_t b) {
    if (--p->rc[b] > 0) return;
    if (p->cached[b]) {
        p->lru.push_back(b);
        p->lru_pos[b] = std::prev(p->lru.end());
        p->in_lru[b] = 1;
    } else {
        p->free_list.push_back(b);
    }
}

// Allocation half of KVBlockPool::append (kv_block_pool.cpp:20-65).
static int reserve(s1kv_pool* p, uint64_t id, int64_t n, int32_t* slots, int64_t* n_done) {
    if (n_done) *n_done = 0;
    if (n < 0) return set_error(S1KV_EINVAL, "s1kv_seq_reserve: negative token count");
    Seq* s = nullptr;
    int st = get_or_create(p, id, &s);
    if (st) return st;
    const int64_t bs = p->desc.block_size;
    // Copy-on-write: a partially filled last block that another table shares
    // or the prefix cache holds is replaced by a private copy before any
    // token lands in it.
    if (n > 0 && !s->table.empty() && s->tokens_in_last < bs) {
        int32_t last = s->table.back();
        if (p->rc[last] > 1 || p->cached[last]) {
            int32_t nb = alloc_block(p);
            if (nb < 0) return set_error(S1KV_ENOBLOCKS, "KVBlockPool: No free blocks available");
            p->pend_cow_src.push_back(last);
            p->pend_cow_dst.push_back(nb);
            p->cow_copies++;
            release_block(p, last);
            s->table.back() = nb;
            mark_dirty(p, id, s, (int64_t)s->table.size() - 1);
        }
    }
    int64_t i = 0;
    bool grew = false;
    int64_t first_new = (int64_t)s->table.size();
    while (i < n) {
        int32_t b;
        if (s->tokens_in_last == bs || s->table.empty()) {
            const bool exhausted = p->free_list.empty() && p->lru.empty();
            if (exhausted || (int64_t)s->table.size() >= p->max_bps) {
                if (grew) mark_dirty(p, id, s, first_new);
                p->max_len_seen = std::max(p->max_len_seen, seq_len(p, s));
                if (exhausted) return set_error(S1KV_ENOBLOCKS, "KVBlockPool: No free blocks available");
                return set_error(S1KV_EINVAL, "s1kv: sequence exceeds max_seq_len (%lld blocks)",
                                 (long long)p->max_bps);
            }
            b = alloc_block(p);
            s->table.push_back(b);
            s->tokens_in_last = 0;
            grew = true;
        } else {
            b = s->table.back();
        }
        int64_t take = std::min<int64_t>(bs - s->tokens_in_last, n - i);
        if (slots)
            for (int64_t t = 0; t < take; t++) slots[i + t] = (int32_t)(b * bs + s->tokens_in_last + t);
        s->tokens_in_last += take;
        i += take;
        if (n_done) *n_done = i;
    }
    if (grew) mark_dirty(p, id, s, first_new);
    p->max_len_seen = std::max(p->max_len_seen, seq_len(p, s));
    return S1KV_OK;
}

// Builds the list of device table entries the queued mutations need.
static void collect_table_updates(s1kv_pool* p, std::vector<TableUpdate>& upd) {
    std::sort(p->dirty.begin(), p->dirty.end());
    p->dirty.erase(std::unique(p->dirty.begin(), p->dirty.end()), p->dirty.end());
    for (uint64_t id : p->dirty) {
        Seq* s = find_seq(p, id);
        if (!s) continue;
        for (int64_t c = s->synced; c < (int64_t)s->table.size(); c++) upd.push_back({s->row, (int32_t)c, s->table[c]});
        s->synced = (int64_t)s->table.size();
    }
    p->dirty.clear();
}

int flush(s1kv_pool* p, cudaStream_t stream) {
    if (p->host_only) return set_error(S1KV_EINVAL, "s1kv: host-only pool has no device storage");
    std::vector<TableUpdate> upd;
    collect_table_updates(p, upd);
    int64_t n_cow = (int64_t)p->pend_cow_src.size();
    if (upd.empty() && n_cow == 0) return S1KV_OK;
    size_t bytes = upd.size() * sizeof(TableUpdate) + 2 * n_cow * sizeof(int32_t) + 64;
    StageSeg* seg = nullptr;
    int st = p->stager.acquire(bytes, &seg);
    if (st) return st;
    size_t off = 0;
    std::memcpy(seg->h, upd.data(), upd.size() * sizeof(TableUpdate));
    off += upd.size() * sizeof(TableUpdate);
    off = (off + 15) & ~size_t(15);
    size_t cow_off = off;
    std::memcpy(seg->h + off, p->pend_cow_src.data(), n_cow * sizeof(int32_t));
    off += n_cow * sizeof(int32_t);
    std::memcpy(seg->h + off, p->pend_cow_dst.data(), n_cow * sizeof(int32_t));
    off += n_cow * sizeof(int32_t);
    S1KV_CUDA(cudaMemcpyAsync(seg->d, seg->h, off, cudaMemcpyHostToDevice, stream));
    if (!upd.empty()) {
        st = launch_table_update((const TableUpdate*)seg->d, (int64_t)upd.size(), p->d_table, p->max_bps, stream);
        if (st) return st;
    }
    if (n_cow) {
        st = launch_cow(p, (const int32_t*)(seg->d + cow_off), (const int32_t*)(seg->d + cow_off + n_cow * 4), n_cow,
                        stream);
        if (st) return st;
    }
    p->pend_cow_src.clear();
    p->pend_cow_dst.clear();
    return p->stager.release(seg, stream);
}

// Device table row / length of a sequence for the kernels.
int seq_row(const s1kv_pool* p, uint64_t id, int32_t* row, int64_t* len) {
    const Seq* s = find_seq(p, id);
    if (!s) return set_error(S1KV_ENOSEQ, "KVBlockPool: Sequence ID not found");
    *row = s->row;
    *len = seq_len(p, s);
    return S1KV_OK;
}

int reserve_internal(s1kv_pool* p, uint64_t id, int64_t n, int32_t* slots, int64_t* n_done) {
    return reserve(p, id, n, slots, n_done);
}

// ------------------------------------------------------------ prefix hash --
static uint64_t block_hash(uint64_t parent, const int32_t* tokens, int64_t n) {
    uint64_t h = 0xcbf29ce484222325ull;
    for (int i = 0; i < 8; i++) {
        h ^= (parent >> (8 * i)) & 0xFF;
        h *= 0x100000001b3ull;
    }
    for (int64_t t = 0; t < n; t++) {
        uint32_t x = (uint32_t)tokens[t];
        for (int i = 0; i < 4; i++) {
            h ^= (x >> (8 * i)) & 0xFF;
            h *= 0x100000001b3ull;
        }
    }
    h ^= h >> 30;
    h *= 0xbf58476d1ce4e5b9ull;
    h ^= h >> 27;
    h *= 0x94d049bb133111ebull;
    h ^= h >> 31;
    return h;
}

static int32_t cache_find(const s1kv_pool* p, uint64_t h, uint64_t parent, const int32_t* tokens) {
    auto range = p->cache_map.equal_range(h);
    const size_t bs = (size_t)p->desc.block_size;
    for (auto it = range.first; it != range.second; ++it) {
        const CacheEntry& e = p->cache_entry[it->second];
        if (e.parent == parent && std::memcmp(e.tokens.data(), tokens, bs * sizeof(int32_t)) == 0) return it->second;
    }
    return -1;
}

}  // namespace s1kv

using namespace s1kv;

// ====================================================================== ABI

extern "C" {

const char* s1kv_last_error(void) { return g_err.c_str(); }

const char* s1kv_status_str(int status) {
    switch (status) {
        case S1KV_OK: return "ok";
        case S1KV_ENOBLOCKS: return "no free blocks";
        case S1KV_ENOSEQ: return "unknown sequence";
        case S1KV_EINVAL: return "invalid argument";
        case S1KV_ECUDA: return "CUDA error";
        case S1KV_ETIMEOUT: return "device wait timed out";
        case S1KV_ENOMEM: return "out of memory";
        case S1KV_EDEVICE: return "device bounds check failed";
        default: return "unknown status";
    }
}

int64_t s1kv_launch_count(void) { return g_launches.load(); }

int s1kv_pool_create(const s1kv_pool_desc* d, int device, s1kv_pool** out) {
    if (!d || !out) return set_error(S1KV_EINVAL, "s1kv_pool_create: null argument");
    *out = nullptr;
    if (d->num_layers < 1 || d->num_kv_heads < 1 || d->head_dim < 1 || d->block_size < 1 || d->max_blocks < 1 ||
        d->max_blocks > INT32_MAX / 2 || (d->dtype != S1KV_DTYPE_F32 && d->dtype != S1KV_DTYPE_BF16))
        return set_error(S1KV_EINVAL, "s1kv_pool_create: bad descriptor");
    int64_t slots = d->max_blocks * (int64_t)d->block_size;
    if (slots > INT32_MAX) return set_error(S1KV_EINVAL, "s1kv_pool_create: more than 2^31 slots per layer");
    auto* p = new s1kv_pool();
    p->desc = *d;
    p->desc.initial_free_list = nullptr;
    if (p->desc.max_seqs <= 0) p->desc.max_seqs = 1024;
    if (p->desc.max_seq_len <= 0) p->desc.max_seq_len = slots;
    if (p->desc.rope_theta == 0.0f) p->desc.rope_theta = 1.0e6f;
    p->device = device;
    p->host_only = (d->flags & S1KV_POOL_HOST_ONLY) != 0;
    p->elem = d->dtype == S1KV_DTYPE_F32 ? 4 : 2;
    p->num_slots = slots;
    p->max_bps = (int32_t)std::min<int64_t>((p->desc.max_seq_len + d->block_size - 1) / d->block_size,
                                            d->max_blocks);
    p->layer_bytes = (size_t)slots * d->num_kv_heads * d->head_dim * p->elem;
    // Free list bottom .. top; the reference pushes 0..max_blocks-1 in order.
    p->free_list.resize(d->max_blocks);
    if (d->initial_free_list) {
        std::vector<uint8_t> seen(d->max_blocks, 0);
        for (int64_t i = 0; i < d->max_blocks; i++) {
            int32_t b = d->initial_free_list[i];
            if (b < 0 || b >= d->max_blocks || seen[b]) {
                delete p;
                return set_error(S1KV_EINVAL, "s1kv_pool_create: initial_free_list is not a permutation");
            }
            seen[b] = 1;
            p->free_list[i] = b;
        }
    } else {
        for (int64_t i = 0; i < d->max_blocks; i++) p->free_list[i] = (int32_t)i;
    }
    p->rc.assign(d->max_blocks, 0);
    p->cached.assign(d->max_blocks, 0);
    p->in_lru.assign(d->max_blocks, 0);
    p->lru_pos.resize(d->max_blocks);
    p->cache_entry.resize(d->max_blocks);
    for (int32_t r = p->desc.max_seqs - 1; r >= 0; r--) p->free_rows.push_back(r);

    if (!p->host_only) {
        DeviceGuard guard(device);
        cudaError_t e = guard.err;
        size_t total = p->layer_bytes * d->num_layers;
        if (e == cudaSuccess) e = cudaMalloc((void**)&p->k, total);
        if (e == cudaSuccess) e = cudaMalloc((void**)&p->v, total);
        // The reference zero-fills its storage (kv_block_pool.cpp:12-13).
        if (e == cudaSuccess) e = cudaMemset(p->k, 0, total);
        if (e == cudaSuccess) e = cudaMemset(p->v, 0, total);
        if (e == cudaSuccess)
            e = cudaMalloc((void**)&p->d_table, (size_t)p->desc.max_seqs * p->max_bps * sizeof(int32_t));
        if (e == cudaSuccess)
            e = cudaMemset(p->d_table, 0, (size_t)p->desc.max_seqs * p->max_bps * sizeof(int32_t));
        if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->copy_stream, cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->d2h_stream, cudaStreamNonBlocking);
        for (int i = 0; i < 6 && e == cudaSuccess; i++)
            e = cudaEventCreateWithFlags(&p->io_ev[i], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess) {
            int st = cuda_error(e, "s1kv_pool_create: device allocation");
            s1kv_pool_destroy(p);
            return st;
        }
        p->d_err = device_error_word(device);
        if (!p->d_err) {
            s1kv_pool_destroy(p);
            return set_error(S1KV_ENOMEM, "s1kv_pool_create: error word allocation failed");
        }
        int st = make_tensor_maps(p);
        if (!st) st = p->stager.reserve(Stager::kInitialBytes);
        if (st) {
            s1kv_pool_destroy(p);
            return st;
        }
        // The RoPE table is computed on the host (bit-exact cos/sin) and
        // growing it synchronises the device, so it is built here for every
        // position the pool can hold (up to 2^18), not in the middle of a
        // decode loop when a sequence first crosses a power of two.
        int64_t rope_cap = 0;
        rope_table(device, d->head_dim, p->desc.rope_theta, std::min<int64_t>(p->desc.max_seq_len, int64_t(1) << 18),
                   &rope_cap, nullptr, &st);
        if (st) {
            s1kv_pool_destroy(p);
            return st;
        }
    }
    *out = p;
    return S1KV_OK;
}

int s1kv_pool_destroy(s1kv_pool* p) {
    if (!p) return S1KV_OK;
    if (!p->host_only) {
        DeviceGuard guard(p->device);
        cudaDeviceSynchronize();
        p->stager.destroy();
        p->scratch.destroy();
        p->counters.destroy();
        p->late_meta.destroy();
        p->io.destroy();
        if (p->k) cudaFree(p->k);
        if (p->v) cudaFree(p->v);
        if (p->d_table) cudaFree(p->d_table);
        for (auto& e : p->io_ev)
            if (e) cudaEventDestroy(e);
        if (p->copy_stream) cudaStreamDestroy(p->copy_stream);
        if (p->d2h_stream) cudaStreamDestroy(p->d2h_stream);
    }
    delete p;
    return S1KV_OK;
}

int s1kv_pool_get_desc(const s1kv_pool* p, s1kv_pool_desc* out) {
    if (!p || !out) return set_error(S1KV_EINVAL, "null argument");
    *out = p->desc;
    return S1KV_OK;
}

int s1kv_pool_stats_get(const s1kv_pool* p, s1kv_pool_stats* out) {
    if (!p || !out) return set_error(S1KV_EINVAL, "null argument");
    out->num_free = (int64_t)p->free_list.size();
    out->num_lru = (int64_t)p->lru.size();
    out->num_cached = p->num_cached;
    out->num_seqs = (int64_t)p->seqs.size();
    out->cow_copies = p->cow_copies;
    out->evictions = p->evictions;
    out->device_bytes = p->host_only ? 0
                                     : (int64_t)(2 * p->layer_bytes * p->desc.num_layers +
                                                 (size_t)p->desc.max_seqs * p->max_bps * 4 + p->scratch.cap +
                                                 p->io.cap);
    return S1KV_OK;
}

int s1kv_pool_storage(const s1kv_pool* p, int32_t layer, void** k, void** v) {
    if (!p || layer < 0 || layer >= p->desc.num_layers) return set_error(S1KV_EINVAL, "s1kv_pool_storage: bad layer");
    if (p->host_only) return set_error(S1KV_EINVAL, "s1kv: host-only pool has no device storage");
    if (k) *k = p->k + (size_t)layer * p->layer_bytes;
    if (v) *v = p->v + (size_t)layer * p->layer_bytes;
    return S1KV_OK;
}

int s1kv_pool_check(s1kv_pool* p, int32_t* flags_out) {
    if (!p || p->host_only) return set_error(S1KV_EINVAL, "s1kv_pool_check: no device pool");
    return s1kv_device_check(p->device, flags_out);
}

int s1kv_device_check(int device, int32_t* flags_out) {
    S1KV_ON_DEVICE(device);
    S1KV_CUDA(cudaDeviceSynchronize());
    int h = 0;
    // the word shared by pools and single calls (created by the first of
    // them), then the no-allocation decode's own word in its fixed array;
    // reading allocates nothing
    if (int* word = existing_error_word(device)) {
        S1KV_CUDA(cudaMemcpy(&h, word, sizeof(int), cudaMemcpyDeviceToHost));
        if (h) S1KV_CUDA(cudaMemset(word, 0, sizeof(int)));
    }
    int na = 0;
    const int st = noalloc_take_error(device, &na);
    if (st) return st;
    h |= na;
    if (flags_out) *flags_out = h;
    if (h & kErrTimeout) return set_error(S1KV_ETIMEOUT, "s1kv: a bounded device wait timed out");
    if (h & kErrBounds) return set_error(S1KV_EDEVICE, "s1kv: a kernel saw an out-of-range slot or block");
    return S1KV_OK;
}

// ------------------------------------------------------------- sequences --

int s1kv_seq_reserve(s1kv_pool* p, uint64_t seq, int64_t n, int32_t* slots_out, int64_t* n_done) {
    if (!p) return set_error(S1KV_EINVAL, "null pool");
    return reserve(p, seq, n, slots_out, n_done);
}

int64_t s1kv_seq_length(const s1kv_pool* p, uint64_t seq) { return p ? seq_len(p, find_seq(p, seq)) : 0; }

int s1kv_seq_exists(const s1kv_pool* p, uint64_t seq) { return p && find_seq(p, seq) ? 1 : 0; }

int s1kv_seq_remove(s1kv_pool* p, uint64_t seq) {
    Seq* s = p ? find_seq(p, seq) : nullptr;
    if (!s) return set_error(S1KV_ENOSEQ, "KVBlockPool: Sequence ID not found");
    for (int32_t b : s->table) release_block(p, b);
    p->free_rows.push_back(s->row);
    p->seqs.erase(seq);
    return S1KV_OK;
}

int s1kv_seq_truncate(s1kv_pool* p, uint64_t seq, int64_t keep) {
    Seq* s = p ? find_seq(p, seq) : nullptr;
    if (!s) return set_error(S1KV_ENOSEQ, "KVBlockPool: Sequence ID not found");
    if (keep < 0) return set_error(S1KV_EINVAL, "s1kv_seq_truncate: negative length");
    if (keep >= seq_len(p, s)) return S1KV_OK;
    const int64_t bs = p->desc.block_size;
    int64_t keep_blocks = 0, in_last = 0;
    if (keep > 0) {
        keep_blocks = (keep - 1) / bs + 1;
        in_last = keep - (keep_blocks - 1) * bs;
    }
    while ((int64_t)s->table.size() > keep_blocks) {
        release_block(p, s->table.back());
        s->table.pop_back();
    }
    s->tokens_in_last = in_last;
    if (s->synced > (int64_t)s->table.size()) s->synced = (int64_t)s->table.size();
    return S1KV_OK;
}

int s1kv_seq_fork(s1kv_pool* p, uint64_t src, uint64_t dst, int64_t n) {
    Seq* s = p ? find_seq(p, src) : nullptr;
    if (!s) return set_error(S1KV_ENOSEQ, "KVBlockPool: Sequence ID not found");
    if (find_seq(p, dst)) return set_error(S1KV_EINVAL, "s1kv_seq_fork: destination sequence exists");
    if (n < 0 || n > seq_len(p, s)) return set_error(S1KV_EINVAL, "s1kv_seq_fork: prefix longer than source");
    const int64_t bs = p->desc.block_size;
    int64_t nb = n > 0 ? (n - 1) / bs + 1 : 0;
    std::vector<int32_t> shared(s->table.begin(), s->table.begin() + nb);
    Seq* d = nullptr;
    int st = get_or_create(p, dst, &d);
    if (st) return st;
    for (int32_t b : shared) {
        d->table.push_back(b);
        p->rc[b]++;
    }
    d->tokens_in_last = nb > 0 ? n - (nb - 1) * bs : 0;
    if (nb) mark_dirty(p, dst, d, 0);
    return S1KV_OK;
}

int s1kv_block_table(const s1kv_pool* p, uint64_t seq, int32_t* out, int64_t cap, int64_t* n_out) {
    const Seq* s = p ? find_seq(p, seq) : nullptr;
    if (!s) return set_error(S1KV_ENOSEQ, "KVBlockPool: Sequence ID not found");
    int64_t n = (int64_t)s->table.size();
    if (out)
        for (int64_t i = 0; i < n && i < cap; i++) out[i] = s->table[i];
    if (n_out) *n_out = n;
    return S1KV_OK;
}

int s1kv_block_refcount(const s1kv_pool* p, int32_t block, int32_t* rc_out) {
    if (!p || block < 0 || block >= p->desc.max_blocks) return set_error(S1KV_EINVAL, "s1kv: block id out of range");
    *rc_out = p->rc[block];
    return S1KV_OK;
}

int s1kv_free_list(const s1kv_pool* p, int32_t* out, int64_t cap, int64_t* n_out) {
    if (!p) return set_error(S1KV_EINVAL, "null pool");
    int64_t n = (int64_t)p->free_list.size();
    if (out)
        for (int64_t i = 0; i < n && i < cap; i++) out[i] = p->free_list[i];
    if (n_out) *n_out = n;
    return S1KV_OK;
}

int s1kv_lru_list(const s1kv_pool* p, int32_t* out, int64_t cap, int64_t* n_out) {
    if (!p) return set_error(S1KV_EINVAL, "null pool");
    int64_t i = 0;
    for (int32_t b : p->lru) {
        if (out && i < cap) out[i] = b;
        i++;
    }
    if (n_out) *n_out = i;
    return S1KV_OK;
}

// ---------------------------------------------------------- prefix cache --

uint64_t s1kv_block_hash(uint64_t parent, const int32_t* tokens, int64_t n) { return block_hash(parent, tokens, n); }

int s1kv_prefix_insert(s1kv_pool* p, uint64_t seq, const int32_t* tokens, int64_t n, int64_t* n_added) {
    Seq* s = p ? find_seq(p, seq) : nullptr;
    if (!s) return set_error(S1KV_ENOSEQ, "KVBlockPool: Sequence ID not found");
    if (n < 0 || n > seq_len(p, s) || (n > 0 && !tokens))
        return set_error(S1KV_EINVAL, "s1kv_prefix_insert: more tokens than the sequence holds");
    const int64_t bs = p->desc.block_size;
    int64_t nb = n / bs, added = 0;
    uint64_t parent = 0;
    for (int64_t i = 0; i < nb; i++) {
        const int32_t* tk = tokens + i * bs;
        uint64_t h = block_hash(parent, tk, bs);
        int32_t b = s->table[i];
        if (cache_find(p, h, parent, tk) < 0 && !p->cached[b]) {
            CacheEntry& e = p->cache_entry[b];
            e.hash = h;
            e.parent = parent;
            e.tokens.assign(tk, tk + bs);
            p->cache_map.emplace(h, b);
            p->cached[b] = 1;
            p->num_cached++;
            added++;
        }
        parent = h;
    }
    if (n_added) *n_added = added;
    return S1KV_OK;
}

int s1kv_prefix_match(s1kv_pool* p, uint64_t dst, const int32_t* tokens, int64_t n, int64_t* n_hit) {
    if (!p || (n > 0 && !tokens)) return set_error(S1KV_EINVAL, "null argument");
    if (find_seq(p, dst)) return set_error(S1KV_EINVAL, "s1kv_prefix_match: destination sequence exists");
    Seq* d = nullptr;
    int st = get_or_create(p, dst, &d);
    if (st) return st;
    const int64_t bs = p->desc.block_size;
    int64_t nb = std::min<int64_t>(n / bs, p->max_bps), hit = 0;
    uint64_t parent = 0;
    for (int64_t i = 0; i < nb; i++) {
        const int32_t* tk = tokens + i * bs;
        uint64_t h = block_hash(parent, tk, bs);
        int32_t b = cache_find(p, h, parent, tk);
        if (b < 0) break;
        if (p->rc[b] == 0 && p->in_lru[b]) {
            p->lru.erase(p->lru_pos[b]);
            p->in_lru[b] = 0;
        }
        p->rc[b]++;
        d->table.push_back(b);
        hit++;
        parent = h;
    }
    d->tokens_in_last = hit > 0 ? bs : 0;
    if (hit) mark_dirty(p, dst, d, 0);
    p->max_len_seen = std::max(p->max_len_seen, hit * bs);
    if (n_hit) *n_hit = hit * bs;
    return S1KV_OK;
}

int s1kv_flush(s1kv_pool* p, void* stream) {
    if (!p) return set_error(S1KV_EINVAL, "null pool");
    if (p->host_only) return set_error(S1KV_EINVAL, "s1kv: host-only pool has no device storage");
    S1KV_ON_DEVICE(p->device);
    return flush(p, (cudaStream_t)stream);
}

}  // extern "C"
