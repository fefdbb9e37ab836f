// internal.h -- shared declarations of libs1kv (host bookkeeping + kernels).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <utility>
#include <cstdint>
#include <list>
#include <string>
#include <unordered_map>
#include <vector>

#include "s1kv.h"

namespace s1kv {

// ---------------------------------------------------------------- errors --
int set_error(int status, const char* fmt, ...);
int cuda_error(cudaError_t e, const char* what);
#define S1KV_CUDA(call)                                           \
    do {                                                          \
        cudaError_t e_ = (call);                                  \
        if (e_ != cudaSuccess) return ::s1kv::cuda_error(e_, #call); \
    } while (0)

extern std::atomic<int64_t> g_launches;

// Makes `device` current for the enclosing scope and restores the caller's
// device on exit: entry points never change the calling thread's current
// CUDA device (a process that drives one GPU per rank relies on it).
struct DeviceGuard {
    int prev = -1;
    cudaError_t err = cudaSuccess;
    explicit DeviceGuard(int device) {
        int cur = 0;
        err = cudaGetDevice(&cur);
        if (err == cudaSuccess && cur != device) {
            err = cudaSetDevice(device);
            if (err == cudaSuccess) prev = cur;
        }
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
    DeviceGuard(const DeviceGuard&) = delete;
    DeviceGuard& operator=(const DeviceGuard&) = delete;
};
// Kernel attributes (dynamic shared memory, cluster size) belong to one
// device's context: a process that drives several GPUs sets them on each.
// `mask` holds one bit per device already set (devices 0-63); setting an
// attribute twice from racing threads is harmless, the mask is atomic.
template <typename F>
inline int once_per_device(std::atomic<uint64_t>& mask, F&& set) {
    int dev = 0;
    const cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
    const uint64_t bit = dev < 64 ? (uint64_t)1 << dev : 0;
    if (bit && (mask.load(std::memory_order_acquire) & bit)) return 0;
    const int st = set();
    if (st == 0) mask.fetch_or(bit, std::memory_order_acq_rel);
    return st;
}

// Programmatic dependent launch of the step's chain of kernels (RoPE +
// append, decode attention): a kernel launched with launch_pdl may become
// resident while the previous kernel of the stream finishes; pdl_enter at
// its very top lets the next kernel do the same and then waits for the
// previous grid to complete (its memory visible) before this one reads
// anything.  Without the launch attribute the wait returns at once.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
#ifdef __CUDACC__
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
#endif

#define S1KV_ON_DEVICE(dev)                                            \
    ::s1kv::DeviceGuard s1kv_device_guard_(dev);                       \
    if (s1kv_device_guard_.err != cudaSuccess) return ::s1kv::cuda_error(s1kv_device_guard_.err, "cudaSetDevice")

// Device error word bits (one word per device, shared by every kernel).
constexpr int kErrBounds = 1;
constexpr int kErrTimeout = 2;
int* device_error_word(int device);
// Reads and clears the no-allocation decode's error word on `device`
// (noalloc.cu); *flags = 0 if that entry point never ran there.
int noalloc_take_error(int device, int* flags);

// Split-K merging (combine.cuh): rows of up to kMergeGroup splits are
// merged by one CTA; longer rows in two levels (groups of kMergeGroup
// splits, then the groups).  A row has at most kMaxSplitsPerRow splits, so
// its (row, KV head) owns kCounterStride arrival counters: the row's, then
// one per group.
constexpr int kMergeGroup = 16;
constexpr int kMaxSplitsPerRow = 64;
constexpr int kCounterStride = 1 + (kMaxSplitsPerRow + kMergeGroup - 1) / kMergeGroup;

// -------------------------------------------------------- device structs --
// One query row of attention: its sequence's block-table row, the number
// of tokens it attends to (causal limit + 1), how many split-K items cover
// it and where its partial results start.
struct RowMeta {
    int32_t table_row;
    int32_t kv_len;
    int32_t n_split;
    int32_t part_off;
};

// One split-K work item: query row and split index, with the row's block
// table row and context length copied in, so a decode CTA can address its
// first K/V tiles without first loading the row's RowMeta.
struct WorkItem {
    int32_t row;
    int32_t split;
    int32_t table_row;
    int32_t kv_len;
};

struct AttnParams {
    const float* q;        // [rows][Hq][D] fp32, post-RoPE
    float* out;            // [rows][Hq][D] fp32
    float* part_o;         // [n_part][Hkv][G][D]
    float* part_ml;        // [n_part][Hkv][G][2]  (max in log2 domain, sum)
    const int32_t* table;  // [max_seqs][max_bps], NULL = contiguous K/V
    const RowMeta* rows;
    const WorkItem* items;
    const void* kbase;     // layer base of K storage (pool dtype)
    const void* vbase;
    int64_t num_slots;     // rows in one layer's storage (bounds)
    int32_t max_bps;
    int32_t max_blocks;
    int32_t n_rows;
    int32_t n_items;
    int32_t split_tokens;
    int32_t block_size;
    int32_t Hq, Hkv, D;
    int32_t layer;
    float scale_log2;      // log2(e) / sqrt(D)
    int* err;
    int32_t* counters;     // [n_rows][Hkv][kCounterStride] arrivals of split CTAs, zero between launches;
                           // NULL = partials are merged by a separate combine launch
    // Output placement and the optional exchange of finished rows with peer
    // GPUs (KV-head sharding): row r, local head j is element
    // (r * out_stride + out_head0 + j) * D + d (out_stride 0 = Hq) of out,
    // or, when xout is set, of xout and of every xpeer buffer as one 64-bit
    // word (epoch << 32 | float bits) that a reader polls.
    int32_t out_stride, out_head0;
    int32_t n_peers;
    uint64_t* xout;
    uint64_t* xpeer[7];
    uint32_t epoch;
    // Copies issued before the wait for the previous kernel (decode rows of
    // a batch): when prewait is set, a tile whose tokens all lie below
    // kv_len - prewait_margin (the tokens appended by this batch are the
    // last prewait_margin of each sequence) is requested before
    // griddepcontrol.wait.  See split_k_attention for why that is safe.
    int32_t prewait;
    int32_t prewait_margin;
};

// One sequence of a prefill batch (tensor-core prefill kernel).
struct PrefillSeq {
    int32_t table_row;
    int32_t kv_len;
    int32_t q_len;
    int32_t q_start;  // first row of this sequence in q / out
};

struct PrefillParams {
    const float* q;          // [rows][Hq][D] fp32, post-RoPE
    float* out;
    const int32_t* table;    // [max_seqs][max_bps]
    const PrefillSeq* seqs;
    int32_t n_seqs;
    int32_t max_chunks;      // grid.x = n_seqs * max_chunks
    int32_t max_bps;
    int32_t max_blocks;
    int32_t Hq, Hkv;
    int32_t layer;
    float scale_log2;
    int64_t n_rows;          // rows of q / out (tensor-map extent)
    int* err;
};

struct AppendParams {
    const float* k;        // [n][Hkv][D]
    const float* v;
    const float* q_in;     // [n][Hq][D] or NULL
    float* q_out;
    const int32_t* slots;  // [n]
    const int32_t* pos;    // [n] (RoPE only)
    void* kpool;           // layer base (pool dtype)
    void* vpool;
    const float2* rope;    // [rope_cap][D/2] (cos, sin)
    int64_t rope_cap;
    int64_t num_slots;
    int64_t n;
    int32_t Hkv, Hq, D;
    int* err;
};

// ------------------------------------------------------------ RoPE table --
// cos/sin of every (position, pair) computed on the host with the exact
// float expression of src/nn/RoPE.cpp:22-24 and uploaded once; device
// transcendental functions do not round like the host C library, and the
// appended K bytes must match the reference bit for bit.
const float2* rope_table(int device, int D, float theta, int64_t min_positions, int64_t* cap, cudaStream_t stream,
                         int* status);

// ------------------------------------------------------------- staging --
// Pinned host + device buffer pairs reused round-robin for per-step
// metadata uploads.  A segment is reused only after the event recorded at
// its release has completed.
struct StageSeg {
    char* h = nullptr;
    char* d = nullptr;
    size_t cap = 0;
    cudaEvent_t ev = nullptr;
    bool pending = false;  // an event recorded at release guards reuse
    bool in_use = false;   // held by a live batch or an in-progress flush
};

struct Stager {
    static constexpr int kSegs = 6;
    // Capacity every segment gets when the pool is created: growing one
    // later allocates pinned memory and frees device memory (which
    // synchronises the device) in the middle of a step.  1 MB holds the
    // metadata of a step of about 100K appended tokens.
    static constexpr size_t kInitialBytes = size_t(1) << 20;
    StageSeg seg[kSegs];
    int next = 0;
    int reserve(size_t bytes);
    int acquire(size_t bytes, StageSeg** out);
    int release(StageSeg* s, cudaStream_t stream);
    void destroy();
};

// Growable device buffer; growth synchronises the device first.
struct DevBuf {
    void* p = nullptr;
    size_t cap = 0;
    int ensure(size_t bytes);
    void destroy();
};

// ---------------------------------------------------------------- pool --
struct Seq {
    std::vector<int32_t> table;
    int64_t tokens_in_last = 0;
    int32_t row = -1;         // device block-table row
    int64_t synced = 0;       // table entries [0, synced) mirrored on the device
};

struct CacheEntry {
    uint64_t hash = 0;
    uint64_t parent = 0;
    std::vector<int32_t> tokens;
};

struct TableUpdate {
    int32_t row, col, block;
};

}  // namespace s1kv

struct s1kv_pool {
    s1kv_pool_desc desc{};
    int device = 0;
    bool host_only = false;
    // device storage
    char* k = nullptr;
    char* v = nullptr;
    size_t elem = 4;
    size_t layer_bytes = 0;   // bytes of one layer of K (or V)
    int64_t num_slots = 0;    // max_blocks * block_size
    int32_t* d_table = nullptr;
    int32_t max_bps = 0;
    int* d_err = nullptr;
    CUtensorMap tmap_k{};
    CUtensorMap tmap_v{};
    bool tmap_ok = false;
    CUtensorMap tmap_k_sw{};  // 128B-swizzled 64-element boxes (tensor-core prefill)
    CUtensorMap tmap_v_sw{};
    CUtensorMap tmap_k_blk{}; // one KV head of one block in one box, both 128B-swizzled halves (bf16 decode)
    CUtensorMap tmap_v_blk{};
    bool tmap_sw_ok = false;
    // host bookkeeping
    std::vector<int32_t> free_list;   // LIFO, back() allocated first
    std::vector<int32_t> rc;
    std::vector<int32_t> cached;      // 1 if the prefix cache holds the block
    std::list<int32_t> lru;           // zero-refcount cached blocks, oldest first
    std::vector<std::list<int32_t>::iterator> lru_pos;
    std::vector<uint8_t> in_lru;
    std::unordered_map<uint64_t, s1kv::Seq> seqs;
    std::vector<int32_t> free_rows;
    std::unordered_multimap<uint64_t, int32_t> cache_map;  // hash -> block
    std::vector<s1kv::CacheEntry> cache_entry;             // per block
    int64_t num_cached = 0;
    int64_t max_len_seen = 0;
    // pending device work
    std::vector<int32_t> pend_cow_src, pend_cow_dst;
    std::vector<uint64_t> dirty;      // sequences whose device table row is stale
    std::vector<s1kv::TableUpdate> pend_rows_cleared;
    // stats
    int64_t cow_copies = 0;
    int64_t evictions = 0;
    // device helpers
    s1kv::Stager stager;
    s1kv::DevBuf scratch;             // split-K partials
    s1kv::DevBuf counters;            // split-K arrival counters (kept at zero)
    s1kv::DevBuf late_meta;           // rows + work list planned after batch_begin
    s1kv::DevBuf io;                  // host-pointer step buffers: two slots
    // s1kv_batch_layer_host: inputs go up on copy_stream and outputs come back
    // on d2h_stream, overlapped with the kernels of neighbouring calls.
    // io_ev: [0,1] inputs of slot s landed, [2,3] slot s's kernels done,
    // [4,5] slot s's output copied back.
    cudaStream_t copy_stream = nullptr;
    cudaStream_t d2h_stream = nullptr;
    cudaEvent_t io_ev[6] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
    bool io_slot_used[2] = {false, false};
    size_t io_slot_bytes = 0;          // slot size of the last call (slots move when it changes)
};

// Peer exchange of attention outputs for KV-head sharding (exchange.cu).
struct s1kv_exchange {
    int device = 0, rank = 0, world = 1;
    int64_t slot_floats = 0;          // elements of one layer's gathered output [B][Hq_total][D]
    char* base = nullptr;             // [2 slots][slot_floats] 64-bit words (epoch << 32 | float bits)
    int64_t used[2] = {};             // words the last attention of each slot parity wrote (rows x heads x D)
    uint32_t used_epoch[2] = {};      // and its epoch
    char* peer_base[8] = {};          // other ranks' bases, NULL for self
    bool peer_ipc[8] = {};            // opened from a CUDA IPC handle (closed on destroy)
    bool opened = false;
    int* d_err = nullptr;
};

struct s1kv_batch {
    s1kv_pool* pool = nullptr;
    s1kv::StageSeg* seg = nullptr;
    int64_t n_tokens = 0;     // appended tokens
    int64_t n_rows = 0;       // attention query rows
    int64_t n_items = 0;      // split-K work items
    int64_t n_part = 0;       // partial-result slots
    int32_t split_tokens = 0;
    int64_t max_pos = 0;      // largest position appended + 1
    bool decode_rows = true;  // every row has q_len 1 for its sequence
    bool rows_are_tokens = true;  // q_len == n_append for every sequence: query row i is appended token i
    int32_t max_append = 0;   // the most tokens any sequence appends in this batch
    const int32_t* d_qpos = nullptr;  // position of each query row (kv_len - 1), when rows are not the tokens
    // device views into seg->d
    const int32_t* d_slots = nullptr;
    const int32_t* d_pos = nullptr;
    const s1kv::RowMeta* d_rows = nullptr;
    const s1kv::WorkItem* d_items = nullptr;
    const s1kv::PrefillSeq* d_pseqs = nullptr;
    int32_t n_seqs = 0;
    int32_t max_qlen = 0;
    std::vector<s1kv::RowMeta> rows;  // host copy (for dispatch decisions)
    std::vector<s1kv::WorkItem> items;  // split-K work list (host copy)
    bool items_planned = false;       // rows' split fields and items computed
    bool items_uploaded = false;      // d_rows / d_items carry them
    int32_t io_calls = 0;             // s1kv_batch_layer_host calls (slot = calls & 1)
};

namespace s1kv {

// --------------------------------------------------------------- kernels --
int launch_table_update(const TableUpdate* d_upd, int64_t n, int32_t* table, int32_t max_bps, cudaStream_t stream);
int launch_cow(s1kv_pool* pool, const int32_t* d_src, const int32_t* d_dst, int64_t n, cudaStream_t stream);
// pdl: launched as a programmatic dependent launch (the batch's appends);
// the single-call entry points launch plainly, so that a kernel after them
// never starts before their writes are complete.
int launch_append(const AppendParams& p, int dtype, bool rope, cudaStream_t stream, bool pdl);
// q/k RMSNorm + RoPE + append (k, v to slots; q rows at qpos to q_out).
int launch_norm_rope_append(const AppendParams& p, int dtype, const float* qw, const float* kw, float eps,
                            const int32_t* qpos, int64_t n_q_rows, cudaStream_t stream);
// Rotates n rows of H heads: row i at position pos[i], or start_pos + i
// when pos is NULL.
int launch_rope(const float* x, float* out, const float2* table, int64_t table_cap, int64_t start_pos, int64_t n,
                int32_t H, int32_t D, int* err, cudaStream_t stream, const int32_t* pos = nullptr);
int launch_gather(s1kv_pool* pool, int32_t layer, int32_t row, int64_t len, int which, float* out,
                  cudaStream_t stream);
// Paged attention over a prepared work list; picks the TMA split-K decode
// kernel when the shape allows it and the generic kernel otherwise.
int launch_attention(s1kv_pool* pool, const AttnParams& p, int dtype, cudaStream_t stream);
int launch_attention_generic(const AttnParams& p, int dtype, cudaStream_t stream);
bool tma_attention_supported(int dtype, int D, int G, int block_size);
int tma_warps_per_cta(int dtype, int D);
int make_tensor_maps(s1kv_pool* pool);

}  // namespace s1kv

namespace s1kv {
// Caller-supplied-storage variants (no pool): used by the no-allocation
// entry point.
int decode_tile_rows(int dtype, int D);
int encode_kv_maps(const void* k, const void* v, int dtype, int Hkv, int D, int64_t num_slots, CUtensorMap* tk,
                   CUtensorMap* tv);
int launch_decode_with_maps(const AttnParams& p, const CUtensorMap& tk, const CUtensorMap& tv, int dtype,
                            cudaStream_t stream);

// Tensor-core (mma.sync) decode over bf16 K/V, head_dim 128 (decode_mma.cu):
// partials in the same format as the CUDA-core decode kernel.
bool decode_mma_supported(int dtype, int D, int G, int block_size);
int launch_decode_mma(const AttnParams& p, const CUtensorMap& tk_sw, const CUtensorMap& tv_sw, cudaStream_t stream);

// Exchange fields of a decode launch that publishes its rows (exchange.cu).
int exchange_params(const s1kv_exchange* ex, uint32_t epoch, int32_t head0, int32_t heads_total, AttnParams* ap);
void exchange_record(s1kv_exchange* ex, uint32_t epoch, int64_t words);

// Tensor-core prefix-hit prefill (prefill_tc.cu).
bool prefill_tc_supported(int dtype, int D, int G, int block_size);
int prefill_queries_per_cta(int G);
int launch_prefill_tc(const PrefillParams& p, const CUtensorMap& tk, const CUtensorMap& tv, cudaStream_t stream);
}  // namespace s1kv
