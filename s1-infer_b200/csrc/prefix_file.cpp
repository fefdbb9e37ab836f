// prefix_file.cpp -- the versioned prefix-cache file (format 1).
//
// The reference keeps one prefix on disk as raw fp32 K then V per layer
// with nothing else (src/demo.cpp:10-41; s1kv_prefix_save/load write and
// read that layout unchanged).  A raw dump cannot tell a file made for a
// different model shape, a truncated copy or a flipped byte from a good
// one, and it does not carry the token ids the hashed prefix cache needs.
// Format 1 (little-endian):
//
//   offset  size  field
//        0     8  magic "S1KVPFX\0"
//        8     4  version = 1
//       12     4  header bytes = 64
//       16     4  num_layers
//       20     4  num_kv_heads
//       24     4  head_dim
//       28     4  block_size of the writing pool (informational)
//       32     4  dtype of the payload (S1KV_DTYPE_F32 or S1KV_DTYPE_BF16)
//       36     4  flags (bit 0: token ids present)
//       40     8  n_tokens
//       48     4  rope_theta (float)
//       52     4  reserved (0)
//       56     8  FNV-1a 64 of every byte after the header
//       64        int32 token_ids[n_tokens] if flag bit 0
//                 then per layer: K [n_tokens][num_kv_heads][head_dim],
//                 V the same, in the payload dtype (bf16 stays 2 bytes)
#include <cstdio>
#include <cstring>
#include <vector>

#include "internal.h"

namespace s1kv {
namespace {

constexpr char kMagic[8] = {'S', '1', 'K', 'V', 'P', 'F', 'X', '\0'};
constexpr uint32_t kVersion = 1, kHeaderBytes = 64, kHasTokens = 1;

struct FileHeader {
    char magic[8];
    uint32_t version, header_bytes, num_layers, num_kv_heads, head_dim, block_size, dtype, flags;
    int64_t n_tokens;
    float rope_theta;
    uint32_t reserved;
    uint64_t checksum;
};
static_assert(sizeof(FileHeader) == kHeaderBytes, "prefix file header is 64 bytes");

struct Fnv {
    uint64_t h = 1469598103934665603ull;
    void add(const void* p, size_t n) {
        const unsigned char* c = static_cast<const unsigned char*>(p);
        for (size_t i = 0; i < n; i++) h = (h ^ c[i]) * 1099511628211ull;
    }
};

uint16_t to_bf16(float f) {  // round to nearest even (the append kernels' rule)
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}
float from_bf16(uint16_t b) {
    const uint32_t u = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// Reads and checks a whole file: header, token ids, payload as fp32.
int read_file(const char* path, FileHeader* hd, std::vector<int32_t>* tokens, std::vector<float>* payload) {
    FILE* f = std::fopen(path, "rb");
    if (!f) return set_error(S1KV_EINVAL, "prefix file: cannot open %s", path);
    std::vector<unsigned char> all;
    unsigned char buf[1 << 16];
    size_t got;
    while ((got = std::fread(buf, 1, sizeof(buf), f)) > 0) all.insert(all.end(), buf, buf + got);
    std::fclose(f);
    if (all.size() < kHeaderBytes) return set_error(S1KV_EINVAL, "prefix file %s: shorter than its header", path);
    std::memcpy(hd, all.data(), kHeaderBytes);
    if (std::memcmp(hd->magic, kMagic, 8) != 0)
        return set_error(S1KV_EINVAL, "prefix file %s: not a format-1 prefix file (bad magic)", path);
    if (hd->version != kVersion || hd->header_bytes != kHeaderBytes)
        return set_error(S1KV_EINVAL, "prefix file %s: version %u / header %u not supported", path, hd->version,
                         hd->header_bytes);
    if ((hd->dtype != S1KV_DTYPE_F32 && hd->dtype != S1KV_DTYPE_BF16) || hd->n_tokens < 0 || hd->head_dim == 0 ||
        hd->num_kv_heads == 0 || hd->num_layers == 0)
        return set_error(S1KV_EINVAL, "prefix file %s: bad header fields", path);
    const uint64_t e = hd->dtype == S1KV_DTYPE_F32 ? 4 : 2;
    const uint64_t row = (uint64_t)hd->num_kv_heads * hd->head_dim;
    const uint64_t tok_bytes = (hd->flags & kHasTokens) ? (uint64_t)hd->n_tokens * 4 : 0;
    const uint64_t body = tok_bytes + 2ull * hd->num_layers * (uint64_t)hd->n_tokens * row * e;
    if (all.size() - kHeaderBytes != body)
        return set_error(S1KV_EINVAL, "prefix file %s: %llu payload bytes, header says %llu", path,
                         (unsigned long long)(all.size() - kHeaderBytes), (unsigned long long)body);
    Fnv fnv;
    fnv.add(all.data() + kHeaderBytes, body);
    if (fnv.h != hd->checksum) return set_error(S1KV_EINVAL, "prefix file %s: checksum mismatch", path);
    const unsigned char* p = all.data() + kHeaderBytes;
    if (tokens) {
        tokens->resize(tok_bytes / 4);
        if (tok_bytes) std::memcpy(tokens->data(), p, tok_bytes);
    }
    p += tok_bytes;
    if (payload) {
        const uint64_t n = 2ull * hd->num_layers * (uint64_t)hd->n_tokens * row;
        payload->resize(n);
        if (e == 4) {
            std::memcpy(payload->data(), p, n * 4);
        } else {
            for (uint64_t i = 0; i < n; i++) {
                uint16_t b;
                std::memcpy(&b, p + 2 * i, 2);
                (*payload)[i] = from_bf16(b);
            }
        }
    }
    return S1KV_OK;
}

}  // namespace
}  // namespace s1kv

using namespace s1kv;

extern "C" {

int s1kv_prefix_save_v1(s1kv_pool* p, uint64_t seq, const int32_t* token_ids, const char* path) {
    if (!p || !path) return set_error(S1KV_EINVAL, "s1kv_prefix_save_v1: null argument");
    if (p->host_only) return set_error(S1KV_EINVAL, "s1kv: host-only pool has no device storage");
    const int64_t len = s1kv_seq_length(p, seq);
    if (!s1kv_seq_exists(p, seq)) return set_error(S1KV_ENOSEQ, "s1kv_prefix_save_v1: unknown sequence");
    const size_t row = (size_t)p->desc.num_kv_heads * p->desc.head_dim, n = (size_t)len * row;
    FileHeader hd{};
    std::memcpy(hd.magic, kMagic, 8);
    hd.version = kVersion;
    hd.header_bytes = kHeaderBytes;
    hd.num_layers = (uint32_t)p->desc.num_layers;
    hd.num_kv_heads = (uint32_t)p->desc.num_kv_heads;
    hd.head_dim = (uint32_t)p->desc.head_dim;
    hd.block_size = (uint32_t)p->desc.block_size;
    hd.dtype = (uint32_t)p->desc.dtype;
    hd.flags = token_ids ? kHasTokens : 0;
    hd.n_tokens = len;
    hd.rope_theta = p->desc.rope_theta;
    // body: token ids, then K and V of every layer in the pool dtype
    std::vector<unsigned char> body;
    if (token_ids) body.insert(body.end(), (const unsigned char*)token_ids, (const unsigned char*)(token_ids + len));
    std::vector<float> h(n);
    float* d = nullptr;
    cudaError_t e = cudaMalloc(&d, std::max<size_t>(n, 1) * sizeof(float));
    int st = S1KV_OK;
    for (int32_t l = 0; l < p->desc.num_layers && e == cudaSuccess && st == S1KV_OK; l++) {
        for (int which = 0; which < 2 && st == S1KV_OK; which++) {
            st = s1kv_gather(p, l, seq, which, d, nullptr);
            if (st) break;
            e = cudaMemcpy(h.data(), d, n * sizeof(float), cudaMemcpyDeviceToHost);
            if (e != cudaSuccess) break;
            if (p->desc.dtype == S1KV_DTYPE_F32) {
                body.insert(body.end(), (const unsigned char*)h.data(), (const unsigned char*)(h.data() + n));
            } else {
                for (size_t i = 0; i < n; i++) {  // gather widened exact bf16 values: narrowing is exact
                    const uint16_t b = to_bf16(h[i]);
                    body.push_back((unsigned char)(b & 0xff));
                    body.push_back((unsigned char)(b >> 8));
                }
            }
        }
    }
    if (d) cudaFree(d);
    if (e != cudaSuccess) return cuda_error(e, "s1kv_prefix_save_v1");
    if (st) return st;
    Fnv fnv;
    fnv.add(body.data(), body.size());
    hd.checksum = fnv.h;
    FILE* f = std::fopen(path, "wb");
    if (!f) return set_error(S1KV_EINVAL, "s1kv_prefix_save_v1: cannot open %s", path);
    const bool ok = std::fwrite(&hd, kHeaderBytes, 1, f) == 1 &&
                    (body.empty() || std::fwrite(body.data(), 1, body.size(), f) == body.size());
    std::fclose(f);
    return ok ? S1KV_OK : set_error(S1KV_EINVAL, "s1kv_prefix_save_v1: short write to %s", path);
}

int s1kv_prefix_file_info(const char* path, s1kv_prefix_info* info) {
    if (!path || !info) return set_error(S1KV_EINVAL, "s1kv_prefix_file_info: null argument");
    FileHeader hd{};
    int st = read_file(path, &hd, nullptr, nullptr);
    if (st) return st;
    info->version = (int32_t)hd.version;
    info->num_layers = (int32_t)hd.num_layers;
    info->num_kv_heads = (int32_t)hd.num_kv_heads;
    info->head_dim = (int32_t)hd.head_dim;
    info->block_size = (int32_t)hd.block_size;
    info->dtype = (int32_t)hd.dtype;
    info->has_tokens = (hd.flags & kHasTokens) ? 1 : 0;
    info->n_tokens = hd.n_tokens;
    info->rope_theta = hd.rope_theta;
    return S1KV_OK;
}

int s1kv_prefix_load_v1(s1kv_pool* p, uint64_t seq, const char* path, int32_t register_blocks, int64_t* n_tokens_out) {
    if (!p || !path) return set_error(S1KV_EINVAL, "s1kv_prefix_load_v1: null argument");
    if (p->host_only) return set_error(S1KV_EINVAL, "s1kv: host-only pool has no device storage");
    FileHeader hd{};
    std::vector<int32_t> tokens;
    std::vector<float> payload;
    int st = read_file(path, &hd, &tokens, &payload);
    if (st) return st;
    if ((int32_t)hd.num_layers != p->desc.num_layers || (int32_t)hd.num_kv_heads != p->desc.num_kv_heads ||
        (int32_t)hd.head_dim != p->desc.head_dim)
        return set_error(S1KV_EINVAL, "prefix file %s: shape %ux%ux%u does not match the pool's %dx%dx%d", path,
                         hd.num_layers, hd.num_kv_heads, hd.head_dim, p->desc.num_layers, p->desc.num_kv_heads,
                         p->desc.head_dim);
    if (hd.rope_theta != p->desc.rope_theta)
        return set_error(S1KV_EINVAL, "prefix file %s: keys rotated with theta %g, pool uses %g", path,
                         (double)hd.rope_theta, (double)p->desc.rope_theta);
    if (register_blocks && !(hd.flags & kHasTokens))
        return set_error(S1KV_EINVAL, "prefix file %s: no token ids to register", path);
    if (s1kv_seq_exists(p, seq)) return set_error(S1KV_EINVAL, "s1kv_prefix_load_v1: sequence exists");
    const int64_t n_tok = hd.n_tokens;
    const size_t n = (size_t)n_tok * p->desc.num_kv_heads * p->desc.head_dim;
    s1kv_batch* b = nullptr;
    const int32_t na = (int32_t)n_tok, ql = 0;
    st = s1kv_batch_begin(p, &seq, &na, &ql, 1, nullptr, &b);
    if (st) return st;
    float* d = nullptr;
    cudaError_t e = cudaMalloc(&d, std::max<size_t>(2 * n, 1) * sizeof(float));
    for (int32_t l = 0; l < p->desc.num_layers && e == cudaSuccess && st == S1KV_OK; l++) {
        e = cudaMemcpy(d, payload.data() + 2 * n * l, 2 * n * sizeof(float), cudaMemcpyHostToDevice);
        if (e == cudaSuccess) st = s1kv_batch_append(b, l, d, d + n, nullptr);
        if (e == cudaSuccess && st == S1KV_OK) e = cudaDeviceSynchronize();
    }
    const int st2 = s1kv_batch_end(b, nullptr);
    if (d) cudaFree(d);
    if (e != cudaSuccess) return cuda_error(e, "s1kv_prefix_load_v1");
    if (st || st2) return st ? st : st2;
    if (register_blocks) {
        int64_t added = 0;
        st = s1kv_prefix_insert(p, seq, tokens.data(), n_tok, &added);
        if (st) return st;
    }
    if (n_tokens_out) *n_tokens_out = n_tok;
    return S1KV_OK;
}

}  // extern "C"
