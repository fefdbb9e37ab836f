// noalloc.cu -- paged decode attention that allocates nothing.
//
// s1kv_decode_attention_noalloc runs the same split-K decode kernel as
// s1kv_batch_attention, but every buffer the kernel needs beyond the
// caller's inputs and outputs (the split-K partial results, the per-row
// metadata and the work list) lives in one file-scope device array of fixed
// size, and the work list is planned on the device from the caller's
// sequence lengths.  So the call issues no cudaMalloc / cudaFree, no pinned
// host allocation and no host-to-device copy of metadata.
//
// It is for callers that cannot allocate device memory at the point where
// attention runs: a plugin invoked from an inference server's execution
// step, which owns all device memory and forbids allocation there; a
// latency-critical decode loop that must not block on (or fail in) the
// allocator; or code whose memory budget is fixed up front.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <mutex>

#include "internal.h"

namespace s1kv {
namespace {

// The scratch array.  Every GPU that loads the library holds it until the
// process exits.  Layout per call: [error word | pad to 256 B][rows][items]
// [partial max/sum][partial o].
constexpr size_t kScratchBytes = size_t(8) << 20;  // 8 MiB
__device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices] = {};

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// One thread per work-item slot (n_seqs * max_splits) plus one per row
// (n_seqs + 1).  Sequence s owns item slots [s*max_splits, (s+1)*max_splits);
// slots past its splits point at the last, empty row (kv_len 0, two
// "splits"), whose CTAs do no loads and only write an empty partial.
__global__ void noalloc_plan_kernel(const int32_t* __restrict__ seq_lens, int32_t n_seqs, int32_t max_seq_len,
                                    int32_t split_tokens, int32_t max_splits, RowMeta* __restrict__ rows,
                                    WorkItem* __restrict__ items, int* __restrict__ err) {
    const int64_t n_items = (int64_t)n_seqs * max_splits;
    const int64_t total = n_items + n_seqs + 1;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const bool is_item = i < n_items;
        const int32_t s = is_item ? (int32_t)(i / max_splits) : (int32_t)(i - n_items);
        if (s == n_seqs) {  // the empty row
            rows[s] = RowMeta{0, 0, 2, n_seqs * max_splits};
            continue;
        }
        int32_t len = seq_lens[s];
        if (len < 1 || len > max_seq_len) {
            if (!is_item) atomicOr(err, kErrBounds);
            len = len < 1 ? 0 : max_seq_len;
        }
        const int32_t n_split = (len + split_tokens - 1) / split_tokens;
        if (is_item) {
            const int32_t j = (int32_t)(i % max_splits);
            items[i] = j < n_split ? WorkItem{s, j, s, len} : WorkItem{n_seqs, 0, 0, 0};
        } else {
            rows[s] = RowMeta{s, len, n_split, s * max_splits};
        }
    }
}

}  // namespace

// Reads and clears the error word of the array on `device` (the current
// device), if a no-allocation call ever ran there: synchronous symbol
// copies, no allocation.  *flags gets the word (0 when never set up).
int noalloc_take_error(int device, int* flags) {
    *flags = 0;
    if (device < 0 || device >= kMaxDevices) return S1KV_OK;
    {
        std::lock_guard<std::mutex> g(g_mu);
        if (!g_addr[device]) return S1KV_OK;
    }
    int h = 0;
    S1KV_CUDA(cudaMemcpyFromSymbol(&h, g_noalloc_scratch, sizeof(int), 0, cudaMemcpyDeviceToHost));
    if (h) {
        const int zero = 0;
        S1KV_CUDA(cudaMemcpyToSymbol(g_noalloc_scratch, &zero, sizeof(int), 0, cudaMemcpyHostToDevice));
    }
    *flags = h;
    return S1KV_OK;
}

}  // namespace s1kv

using namespace s1kv;

extern "C" int s1kv_decode_attention_noalloc(const void* k_cache, const void* v_cache, int32_t dtype,
                                             int64_t num_slots, int32_t num_kv_heads, int32_t head_dim,
                                             int32_t block_size, const int32_t* block_tables,
                                             int32_t max_blocks_per_seq, const int32_t* seq_lens, int32_t n_seqs,
                                             int32_t max_seq_len, const float* q, float* out, int32_t n_q_heads,
                                             void* stream_) {
    cudaStream_t stream = (cudaStream_t)stream_;
    if (n_seqs < 0 || num_kv_heads <= 0 || n_q_heads <= 0 || n_q_heads % num_kv_heads || num_slots <= 0 ||
        max_seq_len < 1 || max_blocks_per_seq < 1 || (int64_t)max_seq_len > (int64_t)max_blocks_per_seq * block_size)
        return set_error(S1KV_EINVAL, "s1kv_decode_attention_noalloc: bad sizes");
    if (dtype != S1KV_DTYPE_F32 && dtype != S1KV_DTYPE_BF16)
        return set_error(S1KV_EINVAL, "s1kv_decode_attention_noalloc: bad dtype");
    const int G = n_q_heads / num_kv_heads;
    if (!tma_attention_supported(dtype, head_dim, G, block_size))
        return set_error(S1KV_EINVAL,
                         "s1kv_decode_attention_noalloc: needs block_size 16, head_dim 64 or 128 and 1/2/4/7/8 "
                         "query heads per KV head");
    if (((uintptr_t)k_cache | (uintptr_t)v_cache) & 15)
        return set_error(S1KV_EINVAL, "s1kv_decode_attention_noalloc: K/V storage must be 16-byte aligned");
    if (n_seqs == 0) return S1KV_OK;
    if (!block_tables || !seq_lens || !q || !out)
        return set_error(S1KV_EINVAL, "s1kv_decode_attention_noalloc: null pointer");

    // Split plan from the length bound: about 8 waves of CTAs over the 148
    // SMs, 4 to 128 tiles of 16 tokens per split.
    const int nw = tma_warps_per_cta(dtype, head_dim);
    const int64_t tiles_per_seq = (max_seq_len + 15) / 16;
    int64_t split_tiles = ((int64_t)n_seqs * tiles_per_seq * num_kv_heads + 148 * 8 - 1) / (148 * 8);
    split_tiles = std::min<int64_t>(std::max<int64_t>(split_tiles, nw), 32 * nw);
    const int32_t split_tokens = (int32_t)(split_tiles * 16);
    const int32_t max_splits = (max_seq_len + split_tokens - 1) / split_tokens;

    // Scratch layout and its limit.
    const int64_t n_items = (int64_t)n_seqs * max_splits;
    const int64_t n_part = n_items + 1;
    const size_t o_rows = 256;
    const size_t o_items = align_up(o_rows + (size_t)(n_seqs + 1) * sizeof(RowMeta), 256);
    const size_t o_ml = align_up(o_items + (size_t)n_items * sizeof(WorkItem), 256);
    const size_t o_o = align_up(o_ml + (size_t)n_part * num_kv_heads * G * 2 * sizeof(float), 256);
    const size_t need = o_o + (size_t)n_part * num_kv_heads * G * head_dim * sizeof(float);
    if (need > kScratchBytes || n_items > INT32_MAX)
        return set_error(S1KV_EINVAL,
                         "s1kv_decode_attention_noalloc: %lld sequences x %d splits need %zu bytes of scratch; the "
                         "fixed limit is %zu (8 MiB)",
                         (long long)n_seqs, max_splits, need, kScratchBytes);

    // Set-up, once per device: the device address of the array.  In host
    // code g_noalloc_scratch names a host-side stand-in, not device memory.
    // The error word is cleared on the caller's stream, ahead of this
    // call's kernels (device globals also start at zero when the module
    // loads).
    int dev = 0;
    S1KV_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return set_error(S1KV_EINVAL, "s1kv_decode_attention_noalloc: device id");
    unsigned char* base = nullptr;
    {
        std::lock_guard<std::mutex> g(g_mu);
        if (!g_addr[dev]) {
            void* p = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
            if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
            e = cudaMemsetAsync(p, 0, 256, stream);
            if (e != cudaSuccess) return cuda_error(e, "cudaMemsetAsync(error word)");
            g_addr[dev] = p;
        }
        base = (unsigned char*)g_addr[dev];
    }
    int* err = (int*)base;
    RowMeta* rows = (RowMeta*)(base + o_rows);
    WorkItem* items = (WorkItem*)(base + o_items);

    const int64_t plan_threads = n_items + n_seqs + 1;
    const int plan_grid = (int)std::min<int64_t>((plan_threads + 255) / 256, 148 * 8);
    noalloc_plan_kernel<<<plan_grid, 256, 0, stream>>>(seq_lens, n_seqs, max_seq_len, split_tokens, max_splits, rows,
                                                       items, err);
    g_launches++;
    S1KV_CUDA(cudaGetLastError());

    CUtensorMap tk, tv;
    int st = encode_kv_maps(k_cache, v_cache, dtype, num_kv_heads, head_dim, num_slots, &tk, &tv);
    if (st) return st;
    AttnParams ap{};
    ap.q = q;
    ap.out = out;
    ap.part_ml = (float*)(base + o_ml);
    ap.part_o = (float*)(base + o_o);
    ap.table = block_tables;
    ap.rows = rows;
    ap.items = items;
    ap.kbase = k_cache;
    ap.vbase = v_cache;
    ap.num_slots = num_slots;
    ap.max_bps = max_blocks_per_seq;
    ap.max_blocks = (int32_t)std::min<int64_t>(num_slots / block_size, INT32_MAX);
    ap.n_rows = n_seqs;
    ap.n_items = (int32_t)n_items;
    ap.split_tokens = split_tokens;
    ap.block_size = block_size;
    ap.Hq = n_q_heads;
    ap.Hkv = num_kv_heads;
    ap.D = head_dim;
    ap.layer = 0;
    ap.scale_log2 = 1.4426950408889634f / std::sqrt((float)head_dim);
    ap.err = err;
    return launch_decode_with_maps(ap, tk, tv, dtype, stream);
}
