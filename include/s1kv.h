/*
 * s1kv.h -- C ABI of the B200 paged KV-cache engine (libs1kv.so).
 *
 * The engine replaces the KV-cache hot path of liamma06/s1-infer:
 *   KVBlockPool            include/infer/kv_block_pool.h:13-45
 *   KVView                 include/infer/kv_block_pool.h:6-11
 *   apply_rope             include/nn/RoPE.h:4
 *   GQA_attention(_paged)  include/nn/attention.h:8-10
 * Reference paths above are relative to the s1-infer project root.
 *
 * Conventions
 *   - Every call returns an int status (S1KV_OK on success).  The message of
 *     the last failure on the calling thread is s1kv_last_error().
 *   - Host bookkeeping (free list, block tables, refcounts, prefix cache) is
 *     single-threaded per pool: drive one pool from one host thread.
 *   - Kernel calls are asynchronous and stream-ordered on the caller's CUDA
 *     stream (passed as void*, NULL = legacy default stream).  Device
 *     pointers passed in are borrowed until the stream work completes.
 *   - Unless a call says otherwise, data pointers are DEVICE pointers.
 *   - A pool holds num_layers layers that share one block table per
 *     sequence.  The reference keeps one KVBlockPool per layer and drives
 *     every layer with the same append/truncate/remove sequence
 *     (src/model/model.cpp:144-162, :297-298), so its per-layer tables are
 *     identical; a pool with num_layers = 1 is exactly one KVBlockPool.
 *   - Pool storage per layer is [max_blocks * block_size][num_kv_heads]
 *     [head_dim] in the pool dtype, the reference layout
 *     (src/infer/kv_block_pool.cpp:12-13); token i of a sequence lives at
 *     slot table[i / block_size] * block_size + i % block_size.
 */
#ifndef S1KV_H
#define S1KV_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define S1KV_OK 0
#define S1KV_ENOBLOCKS 1 /* free list (and LRU) exhausted; ref throws runtime_error (kv_block_pool.cpp:36-38) */
#define S1KV_ENOSEQ 2    /* unknown sequence id; ref throws runtime_error (kv_block_pool.cpp:70,151,166,195) */
#define S1KV_EINVAL 3    /* bad argument or shape */
#define S1KV_ECUDA 4     /* a CUDA runtime call failed */
#define S1KV_ETIMEOUT 5  /* a bounded device-side wait ran out */
#define S1KV_ENOMEM 6    /* device or host allocation failed */
#define S1KV_EDEVICE 7   /* a kernel's bounds check recorded a bad slot/block */

/* ---- storage dtypes ---- */
#define S1KV_DTYPE_F32 0  /* the reference's storage type (include/core/tensor.h:5) */
#define S1KV_DTYPE_BF16 1 /* round-to-nearest-even narrowed on append; widened like
                             bf16_to_float (include/io/safetensors.h:156-161) */

/* ---- pool flags ---- */
#define S1KV_POOL_HOST_ONLY 1 /* bookkeeping only: no device memory; kernel calls fail */

/* ---- which tensor ---- */
#define S1KV_K 0
#define S1KV_V 1

typedef struct s1kv_pool s1kv_pool;
typedef struct s1kv_batch s1kv_batch;

typedef struct s1kv_pool_desc {
    int32_t num_layers;   /* layers sharing one block table (>= 1) */
    int32_t num_kv_heads; /* KVBlockPool num_heads (kv_block_pool.h:32) */
    int32_t head_dim;     /* KVBlockPool head_dim */
    int32_t block_size;   /* KVBlockPool block_size (default 16) */
    int64_t max_blocks;   /* KVBlockPool max_blocks: physical blocks per layer */
    int32_t dtype;        /* S1KV_DTYPE_* */
    int32_t max_seqs;     /* rows of the device block table (0 = 1024) */
    int64_t max_seq_len;  /* tokens per sequence the device table can map (0 = max_blocks * block_size) */
    float rope_theta;     /* RoPE base; 0 = 1e6 (src/nn/RoPE.cpp:22) */
    int32_t flags;        /* S1KV_POOL_* */
    /* Optional initial free list, bottom .. top (the top is allocated
     * first).  NULL = 0 .. max_blocks-1 pushed in order, so the first
     * allocation returns max_blocks-1 (kv_block_pool.cpp:15-17).  Must be a
     * permutation of 0 .. max_blocks-1. */
    const int32_t* initial_free_list;
} s1kv_pool_desc;

/* Per-pool counters, for the tests and the bench. */
typedef struct s1kv_pool_stats {
    int64_t num_free;        /* blocks on the free list */
    int64_t num_lru;         /* zero-refcount cached blocks (evictable) */
    int64_t num_cached;      /* blocks registered in the prefix cache */
    int64_t num_seqs;        /* live sequences */
    int64_t cow_copies;      /* copy-on-write block copies queued so far */
    int64_t evictions;       /* LRU evictions so far */
    int64_t device_bytes;    /* device memory held by the pool */
} s1kv_pool_stats;

/* ======================== errors ======================== */

const char* s1kv_last_error(void);
const char* s1kv_status_str(int status);

/* ======================== lifecycle ======================== */

/* KVBlockPool::KVBlockPool (kv_block_pool.cpp:6-18).  Allocates and
 * zero-fills K/V storage for every layer on `device`. */
int s1kv_pool_create(const s1kv_pool_desc* desc, int device, s1kv_pool** out);
int s1kv_pool_destroy(s1kv_pool* pool);
int s1kv_pool_get_desc(const s1kv_pool* pool, s1kv_pool_desc* out);
int s1kv_pool_stats_get(const s1kv_pool* pool, s1kv_pool_stats* out);

/* Device base pointers of one layer's K and V storage (the KVView::base of
 * get_k_view/get_v_view, kv_block_pool.cpp:192-223). */
int s1kv_pool_storage(const s1kv_pool* pool, int32_t layer, void** k_base, void** v_base);

/* Synchronous copy of the raw bytes of storage slots [slot0, slot0 +
 * n_slots) of one layer's K (which = S1KV_K) or V into host memory
 * (n_slots * num_kv_heads * head_dim elements of the pool dtype). */
int s1kv_pool_read(s1kv_pool* pool, int32_t layer, int32_t which, int64_t slot0, int64_t n_slots, void* host_out);

/* s1kv_pool_check for the device error word of CUDA device `device`
 * (shared by every pool and call on that device), OR-ed with the error word
 * of s1kv_decode_attention_noalloc's fixed array on that device; both are
 * cleared.  Allocates nothing. */
int s1kv_device_check(int device, int32_t* flags_out);

/* Reads and clears the device error word (synchronises the device).  Bit 0:
 * a kernel saw a slot or block id out of range; bit 1: a bounded wait timed
 * out.  Returns S1KV_EDEVICE / S1KV_ETIMEOUT when a bit was set. */
int s1kv_pool_check(s1kv_pool* pool, int32_t* flags_out);

/* ======================== sequence bookkeeping (host) ======================== */

/* Allocation half of KVBlockPool::append (kv_block_pool.cpp:20-65): places
 * n_tokens new tokens at the end of `seq` (created if absent, like
 * sequences_[id]) and writes their slots to slots_out (host, may be NULL).
 * On exhaustion returns S1KV_ENOBLOCKS with the tokens placed so far kept
 * (*n_done), as the reference throws after partial progress.  If the last
 * block is partially filled and shared (refcount > 1) or held by the prefix
 * cache, it is first replaced by a private copy (copy-on-write); the copy is
 * queued and runs on the device at the next kernel call or s1kv_flush. */
int s1kv_seq_reserve(s1kv_pool* pool, uint64_t seq, int64_t n_tokens, int32_t* slots_out, int64_t* n_done);

/* KVBlockPool::length (kv_block_pool.cpp:134-146); 0 for an unknown id. */
int64_t s1kv_seq_length(const s1kv_pool* pool, uint64_t seq);
int s1kv_seq_exists(const s1kv_pool* pool, uint64_t seq);

/* KVBlockPool::remove (kv_block_pool.cpp:148-161).  Blocks are released in
 * table order; a block returns to the free list when its refcount hits 0
 * (to the LRU instead if the prefix cache holds it). */
int s1kv_seq_remove(s1kv_pool* pool, uint64_t seq);

/* KVBlockPool::truncate (kv_block_pool.cpp:163-190).  No-op when
 * keep >= length; tail blocks are released last-first. */
int s1kv_seq_truncate(s1kv_pool* pool, uint64_t seq, int64_t keep);

/* Block sharing (no reference counterpart): dst (must not exist) starts as
 * the first n_tokens of src, sharing its blocks with refcount + 1.  A shared
 * partial tail is copied on the first append by either side. */
int s1kv_seq_fork(s1kv_pool* pool, uint64_t src, uint64_t dst, int64_t n_tokens);

/* Physical block ids of `seq` (the KVView::block_table).  *n_out = table
 * length even when cap is smaller. */
int s1kv_block_table(const s1kv_pool* pool, uint64_t seq, int32_t* out, int64_t cap, int64_t* n_out);
int s1kv_block_refcount(const s1kv_pool* pool, int32_t block, int32_t* rc_out);
/* Free list bottom .. top and the LRU list oldest .. newest (host arrays). */
int s1kv_free_list(const s1kv_pool* pool, int32_t* out, int64_t cap, int64_t* n_out);
int s1kv_lru_list(const s1kv_pool* pool, int32_t* out, int64_t cap, int64_t* n_out);

/* ======================== prefix cache (host) ======================== */
/* Replaces the reference's single-sequence disk prefix and its truncate
 * rewind (src/demo.cpp:10-41, src/model/model.cpp:239-240). */

/* Registers the full blocks of `seq` covering tokens[0:n_tokens) (host
 * int32 token ids) under chained block hashes.  *n_added = blocks newly
 * registered. */
int s1kv_prefix_insert(s1kv_pool* pool, uint64_t seq, const int32_t* tokens, int64_t n_tokens, int64_t* n_added);

/* Creates `dst` from the longest registered chain matching tokens[0:n):
 * matching blocks gain a reference (leaving the LRU).  *n_hit = tokens
 * covered, a multiple of block_size. */
int s1kv_prefix_match(s1kv_pool* pool, uint64_t dst, const int32_t* tokens, int64_t n_tokens, int64_t* n_hit);

/* Chained hash of one block of ids (for host-side tooling and tests). */
uint64_t s1kv_block_hash(uint64_t parent, const int32_t* tokens, int64_t n);

/* save_prefix_cache (src/demo.cpp:33-41): for every layer in order, writes
 * seq's K then V as raw fp32 [length][num_kv_heads][head_dim]. */
int s1kv_prefix_save(s1kv_pool* pool, uint64_t seq, const char* path);
/* load_prefix_cache (src/demo.cpp:10-31): reads n_tokens tokens of that
 * layout and appends them to seq in every layer.  S1KV_EINVAL if the file
 * is missing or short (the reference returns false). */
int s1kv_prefix_load(s1kv_pool* pool, uint64_t seq, int64_t n_tokens, const char* path);

/* Versioned prefix file (format 1; no reference counterpart): supersedes
 * the raw dump above with a 64-byte header (magic "S1KVPFX", version, shape,
 * payload dtype, token count, RoPE theta, FNV-1a 64 checksum of the body),
 * optional token ids, then K and V of every layer in the pool dtype.  The
 * layout is documented in s1-infer_b200/csrc/prefix_file.cpp. */
typedef struct s1kv_prefix_info {
    int32_t version, num_layers, num_kv_heads, head_dim, block_size, dtype, has_tokens;
    int64_t n_tokens;
    float rope_theta;
} s1kv_prefix_info;
/* Writes seq's K/V of every layer; token_ids (host, length = seq length)
 * may be NULL. */
int s1kv_prefix_save_v1(s1kv_pool* pool, uint64_t seq, const int32_t* token_ids, const char* path);
/* Reads and verifies a file's header and checksum (host only, no device). */
int s1kv_prefix_file_info(const char* path, s1kv_prefix_info* info);
/* Creates seq (must not exist) from a file: S1KV_EINVAL on a bad magic,
 * version, size, checksum, shape or RoPE theta mismatch.  register_blocks:
 * also enter its full blocks into the hashed prefix cache under the stored
 * token ids, so later prompts share them.  *n_tokens_out may be NULL. */
int s1kv_prefix_load_v1(s1kv_pool* pool, uint64_t seq, const char* path, int32_t register_blocks,
                        int64_t* n_tokens_out);

/* ============ KV-head sharding: output exchange between GPUs ============ */
/* No reference counterpart (s1-infer is single-process).  One process per
 * GPU; rank r keeps KV heads [r*Hkv/N, (r+1)*Hkv/N) and their query heads.
 * Each rank creates an exchange holding two layer slots of the token-major
 * output [rows][all query heads][head_dim] (slot_floats elements each;
 * layers alternate by epoch parity), exports its CUDA IPC handle (64 bytes),
 * and opens every peer's from the array of all ranks' handles (world x 64
 * bytes, in rank order).  An element is one 64-bit word: the epoch that
 * wrote it in the high 32 bits, the fp32 value's bits in the low 32.
 * s1kv_batch_attention_exchange runs a decode batch's attention for this
 * rank's heads and stores each finished element, tagged with `epoch`, into
 * its place in every rank's slot over NVLink (no fence or flag: a 64-bit
 * store is seen whole or not at all); s1kv_exchange_wait (device, bounded:
 * sets the timeout bit of the error word after about a second) makes the
 * stream wait until every word that the epoch's attention fills, on all
 * ranks, carries the epoch; it is a programmatic dependent launch that
 * polls while this rank's decode kernel still finishes (the words carry
 * their epoch), so dst of s1kv_exchange_wait_copy must not be read by the
 * attention call of the same epoch.  Epochs start at 1 and increase by one per layer step;
 * every rank waits for each epoch (s1kv_exchange_wait or _wait_copy) on the
 * stream of its attention before its attention of the next epoch -- that
 * wait on all ranks' words is what makes reusing a slot two epochs later
 * safe. */
typedef struct s1kv_exchange s1kv_exchange;
int s1kv_exchange_create(int device, int32_t rank, int32_t world, int64_t slot_floats, s1kv_exchange** out);
int s1kv_exchange_handle(const s1kv_exchange* ex, void* handle64);
int s1kv_exchange_open(s1kv_exchange* ex, const void* handles);
/* For ranks that live in ONE process (one host thread per GPU, or several
 * ranks' exchanges on one GPU): bases[world] holds every rank's
 * s1kv_exchange_base() in rank order, device memory that this exchange's
 * GPU can reach (the same GPU, or a peer GPU: peer access is enabled here).
 * Replaces the IPC handle exchange of s1kv_exchange_open. */
void* s1kv_exchange_base(const s1kv_exchange* ex);
int s1kv_exchange_open_local(s1kv_exchange* ex, void* const* bases);
/* Device address of the slot `epoch` uses: [rows][heads_total][head_dim]
 * 64-bit words (epoch << 32 | float bits; on a little-endian GPU the float
 * is the first 4 bytes of each word). */
void* s1kv_exchange_buffer(const s1kv_exchange* ex, uint32_t epoch);
/* Waits for the words this rank's s1kv_batch_attention_exchange of `epoch`
 * filled (the whole slot if it issued none). */
int s1kv_exchange_wait(s1kv_exchange* ex, uint32_t epoch, void* stream);
/* s1kv_exchange_wait, then (in the same kernel) a copy of heads [head0,
 * head0 + n_heads) of every row of the epoch's slot, laid out [rows]
 * [heads_total][head_dim] as s1kv_batch_attention_exchange wrote it (rows x
 * heads_total x head_dim equal to what it wrote), into dst [rows][n_heads]
 * [head_dim] fp32 (device).  For a consumer that wants one contiguous head
 * range of the gathered output, e.g. the query heads a rank feeds to its
 * next layer.  On a timeout dst is incomplete (and the timeout bit set). */
int s1kv_exchange_wait_copy(s1kv_exchange* ex, uint32_t epoch, int32_t rows, int32_t heads_total, int32_t head_dim,
                            int32_t head0, int32_t n_heads, float* dst, void* stream);
int s1kv_exchange_destroy(s1kv_exchange* ex);
/* Decode attention of this rank's n_q_heads query heads (first global head
 * head0 of heads_total), output published through the exchange. */
int s1kv_batch_attention_exchange(s1kv_batch* batch, int32_t layer, const float* q, int32_t n_q_heads,
                                  s1kv_exchange* ex, int32_t head0, int32_t heads_total, uint32_t epoch,
                                  void* stream);

/* ======================== kernels (device, async) ======================== */

/* Runs queued copy-on-write block copies and device block-table updates. */
int s1kv_flush(s1kv_pool* pool, void* stream);

/* Data half of KVBlockPool::append: k, v [n][num_kv_heads][head_dim] fp32
 * are stored at slots[n] (device int32) of `layer`, narrowed to the pool
 * dtype (kv_block_pool.cpp:53-59). */
int s1kv_append(s1kv_pool* pool, int32_t layer, const float* k, const float* v, const int32_t* slots, int64_t n,
                void* stream);

/* Fused RoPE + append.  k is rotated at pos[t] (apply_rope, RoPE.cpp:6-39)
 * and stored with v at slots[t].  When q_in is non-NULL, q_in [n][n_q_heads]
 * [head_dim] is rotated at the same positions into q_out.  max_pos is an
 * exclusive bound on the pos values (0 = the longest sequence in the pool);
 * a position beyond it is skipped and flagged in the device error word. */
int s1kv_rope_append(s1kv_pool* pool, int32_t layer, const float* q_in, float* q_out, int32_t n_q_heads,
                     const float* k, const float* v, const int32_t* slots, const int32_t* pos, int64_t n,
                     int64_t max_pos, void* stream);

/* apply_rope(input, start_pos) (RoPE.cpp:6-39) of x [n][n_heads][head_dim]
 * on the current CUDA device: token t rotates at start_pos + t.  theta 0 =
 * 1e6.  x and out may alias. */
int s1kv_apply_rope(const float* x, float* out, int64_t start_pos, int64_t n, int32_t n_heads, int32_t head_dim,
                    float theta, void* stream);

/* KVBlockPool::get_k / get_v (kv_block_pool.cpp:67-132): gathers `seq`'s
 * tokens of one layer into out [length][num_kv_heads][head_dim] fp32. */
int s1kv_gather(s1kv_pool* pool, int32_t layer, uint64_t seq, int32_t which, float* out, void* stream);

/* Copies whole blocks src[i] -> dst[i] (device int32 ids) in every layer,
 * K and V: the copy-on-write kernel. */
int s1kv_cow_copy(s1kv_pool* pool, const int32_t* src, const int32_t* dst, int64_t n, void* stream);

/* GQA_attention_paged (attention.cpp:128-239) for sequences of one layer.
 * q [sum q_lens][n_q_heads][head_dim] fp32 holds each sequence's q_len
 * query rows back to back; row i of a sequence of length L attends to
 * tokens 0 .. (L - q_len) + i.  out has q's shape.  seqs / q_lens are host
 * arrays. */
int s1kv_attention(s1kv_pool* pool, int32_t layer, const uint64_t* seqs, const int32_t* q_lens, int32_t n_seqs,
                   const float* q, float* out, int32_t n_q_heads, void* stream);

/* Decode attention that allocates nothing.  No counterpart in the reference:
 * this is an extra entry point of this library.
 *
 * For callers that cannot allocate device memory where attention runs -- a
 * plugin called from an inference server's execution step (the server owns
 * all device memory and forbids allocation there), a latency-critical decode
 * loop that must not block on or fail in the allocator, code with a memory
 * budget fixed up front.  It computes what s1kv_batch_attention computes for
 * q_len 1 per sequence, from caller-owned buffers only:
 *   k_cache, v_cache  one layer's storage [num_slots][num_kv_heads][head_dim]
 *                     in `dtype` (e.g. from s1kv_pool_storage), 16-byte aligned
 *   block_tables      device int32 [n_seqs][max_blocks_per_seq]: physical
 *                     block ids of sequence i in row i
 *   seq_lens          device int32 [n_seqs], each in [1, max_seq_len]
 *   q, out            device fp32 [n_seqs][n_q_heads][head_dim]
 * block_size must be 16, head_dim 64 or 128, n_q_heads / num_kv_heads one of
 * 1, 2, 4, 7, 8, and max_seq_len <= max_blocks_per_seq * 16.
 *
 * Its scratch (split-K partial results, row metadata, work list) is one
 * fixed 8 MiB array in device memory that every GPU which loads this
 * library holds until the process exits; the work list is planned on the
 * device.  The call issues no cudaMalloc, cudaFree or other allocating
 * routine.  A call whose sizes need more than 8 MiB (about n_seqs x
 * ceil(max_seq_len / split) x num_kv_heads x (n_q_heads / num_kv_heads) x
 * (head_dim + 2) x 4 bytes) returns S1KV_EINVAL with the sizes in
 * s1kv_last_error().  The first call on a device does a one-time set-up
 * (looks up the array's device address and clears its error word on
 * `stream`), so make that first call before any stream capture.  Every
 * call reuses the same array, which keeps the last call's contents: calls
 * that overlap on the GPU (other streams, other host threads) race and must
 * be serialised by the caller.  The set-up is cached per device ordinal for the life of the
 * process: cudaDeviceReset after the first call is not supported.
 * Sequence lengths outside [1, max_seq_len] (bit 0) and a timed-out copy
 * wait (bit 1) set the array's error word, and the affected output rows are
 * unspecified; s1kv_device_check(device) reads and clears that word, with
 * no allocation. */
int s1kv_decode_attention_noalloc(const void* k_cache, const void* v_cache, int32_t dtype, int64_t num_slots,
                                  int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                  const int32_t* block_tables, int32_t max_blocks_per_seq, const int32_t* seq_lens,
                                  int32_t n_seqs, int32_t max_seq_len, const float* q, float* out,
                                  int32_t n_q_heads, void* stream);

/* GQA_attention (attention.cpp:13-126) over contiguous device K/V
 * [kv_len][n_kv_heads][head_dim] fp32. */
int s1kv_attention_contig(const float* q, const float* k, const float* v, int64_t q_len, int64_t kv_len,
                          int32_t n_q_heads, int32_t n_kv_heads, int32_t head_dim, float* out, void* stream);

/* ======================== batched step (device, async) ======================== */
/* One decode or prefill step of many sequences, amortising the host
 * bookkeeping over all layers: begin reserves n_append[i] slots for each
 * sequence and uploads the step's slots, positions, block tables and work
 * lists once; then per layer rope_append and attention run on that upload.
 * q_len[i] = rows of attention queries for sequence i (NULL = n_append).
 * A decode step is n_append = q_len = 1 for every sequence. */
int s1kv_batch_begin(s1kv_pool* pool, const uint64_t* seqs, const int32_t* n_append, const int32_t* q_lens,
                     int32_t n_seqs, void* stream, s1kv_batch** out);
/* Total appended tokens and query rows of the batch. */
int s1kv_batch_sizes(const s1kv_batch* batch, int64_t* n_tokens, int64_t* n_rows);
/* RoPE + append of this step's k, v [n_tokens][num_kv_heads][head_dim]; q
 * [n_rows][n_q_heads][head_dim] rotated into q_out when q_in is non-NULL,
 * each query row at its own position (the last q_len positions of its
 * sequence), so a step may mix prompts appended without queries and
 * decode rows. */
int s1kv_batch_rope_append(s1kv_batch* batch, int32_t layer, const float* q_in, float* q_out, int32_t n_q_heads,
                           const float* k, const float* v, void* stream);
/* The same step from the raw projection outputs (src/nn/attention.cpp:
 * 316-322): q [n_rows][n_q_heads][head_dim] and k [n_tokens][num_kv_heads]
 * [head_dim] are RMS-normalised per head with q_norm_weight / k_norm_weight
 * (device fp32 [head_dim]; src/nn/rmsnorm.cpp:4-33, bit-exact) and rotated;
 * k and v go to their slots, q to q_out.  One kernel for rmsnorm(Q),
 * rmsnorm(K), apply_rope(Q), apply_rope(K) and KVBlockPool::append.
 * head_dim 64 or 128; pointers 16-byte aligned. */
int s1kv_batch_norm_rope_append(s1kv_batch* batch, int32_t layer, const float* q_in, float* q_out, int32_t n_q_heads,
                                const float* q_norm_weight, const float* k, const float* v, const float* k_norm_weight,
                                float eps, void* stream);

/* Self-check of the division the fused norm kernel uses (no reference
 * counterpart; test support): adds to *mismatch (device, unsigned long long)
 * the number of (x, d) pairs, x from xs[nx] and d from ds[nd] (device
 * arrays), on which it differs from the correctly rounded x / d. */
int s1kv_debug_div_check(const float* xs, int64_t nx, const float* ds, int64_t nd, unsigned long long* mismatch,
                         void* stream);
/* Append without RoPE (KVBlockPool::append data movement). */
int s1kv_batch_append(s1kv_batch* batch, int32_t layer, const float* k, const float* v, void* stream);
/* Paged GQA attention of the batch's query rows (post-RoPE q).  For decode
 * batches (at most one query row per sequence) the kernel is a programmatic
 * dependent launch that may request the K/V of tokens this batch did not
 * append while the previous kernel of the stream is still running; every
 * kernel of this library that writes the pool elsewhere completes before a
 * later kernel starts.  A caller's own programmatic-dependent kernel that
 * writes the pool must therefore not come directly before this call. */
int s1kv_batch_attention(s1kv_batch* batch, int32_t layer, const float* q, float* out, int32_t n_q_heads,
                         void* stream);
/* End-to-end layer step with HOST buffers (pinned for full speed): copies
 * q, k, v in, runs RoPE+append and attention on `stream`, copies out back.
 * Shapes as above.  The copies run on the pool's own copy streams, two
 * buffer slots alternating between calls, so one call's inputs go up while
 * the previous call's kernels run and its output comes back during the
 * next call's.  h_q/h_k/h_v may be reused once the stream has passed the
 * call; h_out of every call of the batch is complete once the stream has
 * passed s1kv_batch_end (synchronise then). */
int s1kv_batch_layer_host(s1kv_batch* batch, int32_t layer, const float* h_q, const float* h_k, const float* h_v,
                          float* h_out, int32_t n_q_heads, void* stream);
int s1kv_batch_end(s1kv_batch* batch, void* stream);

/* ============ int8 projections either side of the KV path ============ */
/* The reference quantizes every pre-transposed [K, N] weight (the q/k/v
 * projections whose outputs the append consumes, o_proj after the attention,
 * the MLP and the LM head) and multiplies with it on the CPU
 * (src/quantized_tensor.cpp; weights pre-transposed by
 * src/model/model.cpp:8-33).  Device pointers; asynchronous on `stream`. */

/* quantize_tensor (src/quantized_tensor.cpp:9-47, include/core/
 * quantized_tensor.h:13): w [rows][cols] fp32 -> q [rows][cols] int8 and
 * one scale per row, scale = max|w[row,:]| / 127 (1 for an all-zero row),
 * q = round(w / scale) with ties away from zero.  Bit-exact with the
 * reference. */
int s1kv_quantize_rows(const float* w, int64_t rows, int64_t cols, int8_t* q, float* scales, void* stream);

/* matmul_quantized (src/quantized_tensor.cpp:102-122, kernel
 * matmul_quantized_range_blocked :60-100; include/core/quantized_tensor.h:
 * 17-23): out [M][N] = x [M][K] * (q [K][N] scaled by scales[k] per row k),
 * fp32.  Sums over k in a fixed tree order (the same on every run), within
 * 2e-5 of the output scale of the reference's sequential sum.  K <= 8192;
 * M any (rows of x are taken 8 at a time). */
int s1kv_matmul_int8(const float* x, int64_t M, int64_t K, const int8_t* q, const float* scales, int64_t N,
                     float* out, void* stream);
/* Up to 4 products sharing x and K in one launch (the q/k/v projections of
 * self_attention_quantized, src/nn/attention.cpp:307-309; gate/up of the
 * MLP, src/nn/mlp.cpp:81-82): out[i] [M][N[i]] = x * (q[i], scales[i]).
 * The same results as n_mats separate s1kv_matmul_int8 calls; the arrays
 * (host memory) hold device pointers. */
int s1kv_matmul_int8_group(const float* x, int64_t M, int64_t K, int32_t n_mats, const int8_t* const* q,
                           const float* const* scales, const int64_t* N, float* const* out, void* stream);

/* ======================== introspection ======================== */

/* Number of kernel launches this library issued on the calling process
 * (all pools), for launch accounting. */
int64_t s1kv_launch_count(void);
/* Split size (tokens per work item) the last s1kv_batch_begin chose, and
 * the number of attention work items. */
int s1kv_batch_plan(const s1kv_batch* batch, int32_t* split_tokens, int64_t* n_items);

#ifdef __cplusplus
}
#endif

#endif /* S1KV_H */
