/*
 * kvoracle.c -- CPU oracle for the paged KV-cache path.  TEST INFRASTRUCTURE
 * ONLY: the parity tests, the smoke check and the bench's CPU-baseline leg
 * compare the library's results with it.  Nothing in the product library
 * links or calls it.
 *
 * A plain-C restatement of liamma06/s1-infer's KV-cache hot path:
 *   - KVBlockPool bookkeeping and storage   src/infer/kv_block_pool.cpp:6-223
 *   - apply_rope                             src/nn/RoPE.cpp:6-39
 *   - GQA_attention / GQA_attention_paged    src/nn/attention.cpp:13-239
 * plus the block-sharing semantics that the reference does not have
 * (refcounts, fork, copy-on-write of a partial tail block, a hashed prefix
 * cache with LRU eviction of zero-refcount blocks).  Those follow the
 * written specification in the repository's design notes; the product's
 * host bookkeeping implements the same specification independently.
 *
 * Build with -O2 -ffp-contract=off and without -ffast-math so every float
 * operation is the plain IEEE mul/add/div the reference executes.  The
 * fp32 restatement is pinned bit-for-bit against the reference compiled
 * from its own sources (oracle/_ref) and against committed golden vectors.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define KVO_OK 0
#define KVO_ENOBLOCKS 1
#define KVO_ENOSEQ 2
#define KVO_EINVAL 3

/* ------------------------------------------------------------------ */
/* bf16 narrowing / widening                                           */
/* ------------------------------------------------------------------ */

/* Round-to-nearest-even narrowing of an IEEE float to bfloat16. NaN maps to
 * the quiet NaN 0x7FC0 with the input's sign. */
uint16_t kvo_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu) != 0)
        return (uint16_t)(((u >> 16) & 0x8000u) | 0x7FC0u);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

/* Widening puts the 16 bits in the top half of a float
 * (include/io/safetensors.h:156-161). */
float kvo_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

void kvo_bf16_round_array(const float* in, float* out, int64_t n) {
    for (int64_t i = 0; i < n; i++) out[i] = kvo_bf16_to_f32(kvo_f32_to_bf16(in[i]));
}

void kvo_to_bf16_array(const float* in, uint16_t* out, int64_t n) {
    for (int64_t i = 0; i < n; i++) out[i] = kvo_f32_to_bf16(in[i]);
}

/* ------------------------------------------------------------------ */
/* RoPE (src/nn/RoPE.cpp:6-39)                                         */
/* ------------------------------------------------------------------ */

/* Rotate-half RoPE of one [H, D] token at position pos.  theta for pair j
 * is (float)pos / powf(base, (float)(2j) / (float)D) (RoPE.cpp:22), then
 * out[j] = x1*c - x2*s and out[j+D/2] = x2*c + x1*s (RoPE.cpp:32-33). */
static void rope_token(const float* x, float* out, int64_t H, int64_t D, int64_t pos, float base) {
    int64_t half = D / 2;
    for (int64_t h = 0; h < H; h++) {
        for (int64_t j = 0; j < half; j++) {
            float theta = (float)pos / powf(base, (float)(2 * j) / (float)D);
            float c = cosf(theta);
            float s = sinf(theta);
            float x1 = x[h * D + j];
            float x2 = x[h * D + j + half];
            out[h * D + j] = x1 * c - x2 * s;
            out[h * D + j + half] = x2 * c + x1 * s;
        }
    }
}

/* apply_rope(input [T, H, D], start_pos): token i rotates at start_pos + i. */
void kvo_apply_rope(const float* x, int64_t T, int64_t H, int64_t D, int64_t start_pos, float base,
                    float* out) {
    for (int64_t i = 0; i < T; i++)
        rope_token(x + i * H * D, out + i * H * D, H, D, start_pos + i, base);
}

/* Same rotation with an explicit position per token. */
void kvo_apply_rope_pos(const float* x, int64_t T, int64_t H, int64_t D, const int32_t* pos, float base,
                        float* out) {
    for (int64_t i = 0; i < T; i++) rope_token(x + i * H * D, out + i * H * D, H, D, pos[i], base);
}

/* rmsnorm(input [rows, D], weight [D], eps) (src/nn/rmsnorm.cpp:4-33): per
 * row, the squares summed in order, rms = sqrt(sum / D + eps), then
 * (x / rms) * w. */
void kvo_rmsnorm(const float* x, int64_t rows, int64_t D, const float* w, float eps, float* out) {
    for (int64_t r = 0; r < rows; r++) {
        const float* xr = x + r * D;
        float sum = 0.0f;
        for (int64_t j = 0; j < D; j++) sum += xr[j] * xr[j];
        float rms = sqrtf(sum / (float)D + eps);
        for (int64_t j = 0; j < D; j++) out[r * D + j] = (xr[j] / rms) * w[j];
    }
}

/* The cos/sin pair the rotation uses for (pos, j), for table checks. */
void kvo_rope_cs(int64_t pos, int64_t j, int64_t D, float base, float* c, float* s) {
    float theta = (float)pos / powf(base, (float)(2 * j) / (float)D);
    *c = cosf(theta);
    *s = sinf(theta);
}

/* ------------------------------------------------------------------ */
/* Attention (src/nn/attention.cpp:13-239)                             */
/* ------------------------------------------------------------------ */

/* Shared core: K/V row j of kv head kvh is fetched by a callback-free
 * address rule.  Per q head h (kv_head = h / group, attention.cpp:155):
 * scores = dot / sqrtf(D) over j <= (kv_len - q_len) + i (:181, :190),
 * softmax as max / expf(s - max) / sum / divide (:196-218), then PV summed
 * in increasing j (:220-235).  Everything is sequential fp32. */
static void attention_core(const float* q, int64_t q_len, int64_t kv_len, int64_t Hq, int64_t Hkv, int64_t D,
                           const float* kbase, const float* vbase, const int32_t* table, int64_t bs,
                           int contiguous, float* out) {
    int64_t group = Hq / Hkv;
    float* qs = (float*)malloc(sizeof(float) * (size_t)(q_len * D + 1));
    float* ks = (float*)malloc(sizeof(float) * (size_t)(kv_len * D + 1));
    float* vs = (float*)malloc(sizeof(float) * (size_t)(kv_len * D + 1));
    float* sc = (float*)malloc(sizeof(float) * (size_t)(q_len * kv_len + 1));
    float sqrt_d = sqrtf((float)D);
    for (int64_t h = 0; h < Hq; h++) {
        for (int64_t i = 0; i < q_len; i++) memcpy(qs + i * D, q + (i * Hq + h) * D, sizeof(float) * (size_t)D);
        int64_t kvh = h / group;
        for (int64_t i = 0; i < kv_len; i++) {
            int64_t row = contiguous ? i : (int64_t)table[i / bs] * bs + i % bs;
            memcpy(ks + i * D, kbase + (row * Hkv + kvh) * D, sizeof(float) * (size_t)D);
            memcpy(vs + i * D, vbase + (row * Hkv + kvh) * D, sizeof(float) * (size_t)D);
        }
        for (int64_t i = 0; i < q_len; i++) {
            const float* qr = qs + i * D;
            int64_t lim = (kv_len - q_len) + i;
            for (int64_t j = 0; j <= lim; j++) {
                const float* kr = ks + j * D;
                float dot = 0.0f;
                for (int64_t d = 0; d < D; d++) dot += qr[d] * kr[d];
                sc[i * kv_len + j] = dot / sqrt_d;
            }
        }
        for (int64_t i = 0; i < q_len; i++) {
            int64_t lim = (kv_len - q_len) + i;
            float* r = sc + i * kv_len;
            float mx = -INFINITY;
            for (int64_t j = 0; j <= lim; j++) mx = r[j] > mx ? r[j] : mx;
            float sum = 0.0f;
            for (int64_t j = 0; j <= lim; j++) {
                r[j] = expf(r[j] - mx);
                sum += r[j];
            }
            for (int64_t j = 0; j <= lim; j++) r[j] /= sum;
            for (int64_t j = lim + 1; j < kv_len; j++) r[j] = 0.0f;
        }
        for (int64_t i = 0; i < q_len; i++) {
            const float* r = sc + i * kv_len;
            int64_t lim = (kv_len - q_len) + i;
            float* dst = out + (i * Hq + h) * D;
            for (int64_t d = 0; d < D; d++) dst[d] = 0.0f;
            for (int64_t j = 0; j <= lim; j++) {
                float p = r[j];
                const float* vr = vs + j * D;
                for (int64_t d = 0; d < D; d++) dst[d] += p * vr[d];
            }
        }
    }
    free(qs);
    free(ks);
    free(vs);
    free(sc);
}

/* GQA_attention over contiguous K/V [kv_len, Hkv, D] (attention.cpp:13-126). */
void kvo_gqa_attention(const float* q, const float* k, const float* v, int64_t q_len, int64_t kv_len, int64_t Hq,
                       int64_t Hkv, int64_t D, float* out) {
    attention_core(q, q_len, kv_len, Hq, Hkv, D, k, v, NULL, 1, 1, out);
}

/* GQA_attention_paged: K/V row of token i lives at pool row
 * table[i / bs] * bs + i % bs (attention.cpp:159-176). */
void kvo_gqa_attention_paged(const float* q, int64_t q_len, const float* pool_k, const float* pool_v,
                             const int32_t* table, int64_t kv_len, int64_t bs, int64_t Hq, int64_t Hkv, int64_t D,
                             float* out) {
    attention_core(q, q_len, kv_len, Hq, Hkv, D, pool_k, pool_v, table, bs, 0, out);
}

/* ------------------------------------------------------------------ */
/* Block pool (src/infer/kv_block_pool.cpp) + sharing semantics        */
/* ------------------------------------------------------------------ */

typedef struct {
    uint64_t id;
    int32_t* table;
    int64_t n_blocks;
    int64_t cap;
    int64_t tokens_in_last;
} kvo_seq;

typedef struct {
    uint64_t hash;
    uint64_t parent;
    int32_t block;
    int32_t* tokens; /* bs token ids */
} kvo_cached;

typedef struct kvo_pool {
    int64_t H, D, max_blocks, bs;
    float* k; /* [max_blocks * bs, H, D], zero-filled (kv_block_pool.cpp:12-13) */
    float* v;
    int32_t* free_list; /* LIFO; top = free_list[n_free - 1] */
    int64_t n_free;
    int32_t* rc;         /* per block refcount */
    int32_t* cached;     /* per block: index+1 into cache entries, 0 = not cached */
    int32_t* lru;        /* zero-refcount cached blocks, oldest first */
    int64_t n_lru;
    kvo_seq* seqs;
    int64_t n_seqs, cap_seqs;
    kvo_cached* cache;
    int64_t n_cache, cap_cache;
} kvo_pool;

/* Constructor: storage zero-filled; free list pushed 0..max_blocks-1 so the
 * first allocation returns max_blocks-1 (kv_block_pool.cpp:6-18). */
kvo_pool* kvo_pool_new(int64_t H, int64_t D, int64_t max_blocks, int64_t bs) {
    kvo_pool* p = (kvo_pool*)calloc(1, sizeof(kvo_pool));
    p->H = H;
    p->D = D;
    p->max_blocks = max_blocks;
    p->bs = bs;
    size_t n = (size_t)(max_blocks * bs * H * D);
    p->k = (float*)calloc(n + 1, sizeof(float));
    p->v = (float*)calloc(n + 1, sizeof(float));
    p->free_list = (int32_t*)malloc(sizeof(int32_t) * (size_t)(max_blocks + 1));
    p->rc = (int32_t*)calloc((size_t)max_blocks + 1, sizeof(int32_t));
    p->cached = (int32_t*)calloc((size_t)max_blocks + 1, sizeof(int32_t));
    p->lru = (int32_t*)malloc(sizeof(int32_t) * (size_t)(max_blocks + 1));
    for (int64_t i = 0; i < max_blocks; i++) p->free_list[i] = (int32_t)i;
    p->n_free = max_blocks;
    return p;
}

void kvo_pool_free(kvo_pool* p) {
    if (!p) return;
    for (int64_t i = 0; i < p->n_seqs; i++) free(p->seqs[i].table);
    for (int64_t i = 0; i < p->n_cache; i++) free(p->cache[i].tokens);
    free(p->seqs);
    free(p->cache);
    free(p->k);
    free(p->v);
    free(p->free_list);
    free(p->rc);
    free(p->cached);
    free(p->lru);
    free(p);
}

/* Replace the free list (bottom .. top) before any allocation.  Used to
 * start from a seeded shuffle; equivalent to the filler-append / remove
 * trick the reference tests use (tests/test_attention.cpp:76-78). */
int kvo_set_free_list(kvo_pool* p, const int32_t* order, int64_t n) {
    if (n != p->n_free) return KVO_EINVAL;
    memcpy(p->free_list, order, sizeof(int32_t) * (size_t)n);
    return KVO_OK;
}

float* kvo_pool_k(kvo_pool* p) { return p->k; }
float* kvo_pool_v(kvo_pool* p) { return p->v; }
int64_t kvo_num_free(const kvo_pool* p) { return p->n_free; }
int64_t kvo_num_lru(const kvo_pool* p) { return p->n_lru; }

int64_t kvo_free_list(const kvo_pool* p, int32_t* out, int64_t cap) {
    int64_t n = p->n_free < cap ? p->n_free : cap;
    memcpy(out, p->free_list, sizeof(int32_t) * (size_t)n);
    return p->n_free;
}

int64_t kvo_lru_list(const kvo_pool* p, int32_t* out, int64_t cap) {
    int64_t n = p->n_lru < cap ? p->n_lru : cap;
    memcpy(out, p->lru, sizeof(int32_t) * (size_t)n);
    return p->n_lru;
}

static kvo_seq* find_seq(const kvo_pool* p, uint64_t id) {
    for (int64_t i = 0; i < p->n_seqs; i++)
        if (p->seqs[i].id == id) return &p->seqs[i];
    return NULL;
}

/* sequences_[id] creates an empty entry when absent (kv_block_pool.cpp:28). */
static kvo_seq* get_or_create(kvo_pool* p, uint64_t id) {
    kvo_seq* s = find_seq(p, id);
    if (s) return s;
    if (p->n_seqs == p->cap_seqs) {
        p->cap_seqs = p->cap_seqs ? p->cap_seqs * 2 : 16;
        p->seqs = (kvo_seq*)realloc(p->seqs, sizeof(kvo_seq) * (size_t)p->cap_seqs);
    }
    s = &p->seqs[p->n_seqs++];
    memset(s, 0, sizeof(*s));
    s->id = id;
    return s;
}

static void seq_push(kvo_seq* s, int32_t b) {
    if (s->n_blocks == s->cap) {
        s->cap = s->cap ? s->cap * 2 : 8;
        s->table = (int32_t*)realloc(s->table, sizeof(int32_t) * (size_t)s->cap);
    }
    s->table[s->n_blocks++] = b;
}

static int64_t seq_len(const kvo_pool* p, const kvo_seq* s) {
    if (!s || s->n_blocks == 0) return 0;
    return (s->n_blocks - 1) * p->bs + s->tokens_in_last;
}

int64_t kvo_length(const kvo_pool* p, uint64_t id) { return seq_len(p, find_seq(p, id)); }
int kvo_has_seq(const kvo_pool* p, uint64_t id) { return find_seq(p, id) != NULL; }

static void cache_unregister(kvo_pool* p, int32_t b) {
    int32_t idx = p->cached[b] - 1;
    if (idx < 0) return;
    free(p->cache[idx].tokens);
    int64_t last = p->n_cache - 1;
    if (idx != last) {
        p->cache[idx] = p->cache[last];
        p->cached[p->cache[idx].block] = idx + 1;
    }
    p->n_cache--;
    p->cached[b] = 0;
}

static void lru_remove(kvo_pool* p, int32_t b) {
    for (int64_t i = 0; i < p->n_lru; i++) {
        if (p->lru[i] == b) {
            memmove(p->lru + i, p->lru + i + 1, sizeof(int32_t) * (size_t)(p->n_lru - i - 1));
            p->n_lru--;
            return;
        }
    }
}

/* Allocation: top of the LIFO free list (kv_block_pool.cpp:40-41); when it
 * is empty, evict the least recently released zero-refcount cached block. */
static int32_t alloc_block(kvo_pool* p) {
    int32_t b;
    if (p->n_free > 0) {
        b = p->free_list[--p->n_free];
    } else if (p->n_lru > 0) {
        b = p->lru[0];
        memmove(p->lru, p->lru + 1, sizeof(int32_t) * (size_t)(p->n_lru - 1));
        p->n_lru--;
        cache_unregister(p, b);
    } else {
        return -1;
    }
    p->rc[b] = 1;
    return b;
}

/* Drop one reference; at zero a cached block goes to the LRU tail, any
 * other block back on top of the free list. */
static void release_block(kvo_pool* p, int32_t b) {
    if (--p->rc[b] > 0) return;
    if (p->cached[b]) p->lru[p->n_lru++] = b;
    else p->free_list[p->n_free++] = b;
}

static void copy_block(kvo_pool* p, int32_t dst, int32_t src) {
    size_t n = (size_t)(p->bs * p->H * p->D);
    memcpy(p->k + (size_t)dst * n, p->k + (size_t)src * n, n * sizeof(float));
    memcpy(p->v + (size_t)dst * n, p->v + (size_t)src * n, n * sizeof(float));
}

/* Allocation half of append (kv_block_pool.cpp:20-65): returns the slot of
 * each new token.  On exhaustion the tokens placed so far stay placed and
 * KVO_ENOBLOCKS is returned with *n_done set, like the reference's
 * throw-after-partial-progress.  Before writing into a partially filled
 * last block that is shared (refcount > 1) or registered in the prefix
 * cache, the block is copied to a fresh one (copy-on-write). */
int kvo_reserve(kvo_pool* p, uint64_t id, int64_t T, int32_t* slots, int64_t* n_done, int32_t* cow_src,
                int32_t* cow_dst) {
    kvo_seq* s = get_or_create(p, id);
    if (n_done) *n_done = 0;
    if (cow_src) *cow_src = -1;
    if (cow_dst) *cow_dst = -1;
    if (T > 0 && s->n_blocks > 0 && s->tokens_in_last < p->bs) {
        int32_t last = s->table[s->n_blocks - 1];
        if (p->rc[last] > 1 || p->cached[last]) {
            int32_t nb = alloc_block(p);
            if (nb < 0) return KVO_ENOBLOCKS;
            copy_block(p, nb, last);
            release_block(p, last);
            s->table[s->n_blocks - 1] = nb;
            if (cow_src) *cow_src = last;
            if (cow_dst) *cow_dst = nb;
        }
    }
    int64_t i = 0;
    while (i < T) {
        int32_t b;
        if (s->tokens_in_last == p->bs || s->n_blocks == 0) {
            b = alloc_block(p);
            if (b < 0) {
                if (n_done) *n_done = i;
                return KVO_ENOBLOCKS;
            }
            seq_push(s, b);
            s->tokens_in_last = 0;
        } else {
            b = s->table[s->n_blocks - 1];
        }
        int64_t room = p->bs - s->tokens_in_last;
        int64_t take = room < T - i ? room : T - i;
        for (int64_t t = 0; t < take; t++) slots[i + t] = (int32_t)(b * p->bs + s->tokens_in_last + t);
        s->tokens_in_last += take;
        i += take;
        if (n_done) *n_done = i;
    }
    return KVO_OK;
}

/* KVBlockPool::append: reserve slots, then copy each token's [H, D] rows
 * (kv_block_pool.cpp:53-59). */
int kvo_append(kvo_pool* p, uint64_t id, const float* k, const float* v, int64_t T) {
    int32_t* slots = (int32_t*)malloc(sizeof(int32_t) * (size_t)(T + 1));
    int64_t done = 0;
    int rc = kvo_reserve(p, id, T, slots, &done, NULL, NULL);
    size_t row = (size_t)(p->H * p->D);
    for (int64_t t = 0; t < done; t++) {
        memcpy(p->k + (size_t)slots[t] * row, k + (size_t)t * row, row * sizeof(float));
        memcpy(p->v + (size_t)slots[t] * row, v + (size_t)t * row, row * sizeof(float));
    }
    free(slots);
    return rc;
}

/* get_k / get_v (kv_block_pool.cpp:67-132): contiguous [len, H, D]. */
int kvo_get(const kvo_pool* p, uint64_t id, int which, float* out) {
    const kvo_seq* s = find_seq(p, id);
    if (!s) return KVO_ENOSEQ;
    int64_t len = seq_len(p, s);
    const float* src = which ? p->v : p->k;
    size_t row = (size_t)(p->H * p->D);
    for (int64_t i = 0; i < len; i++) {
        int64_t r = (int64_t)s->table[i / p->bs] * p->bs + i % p->bs;
        memcpy(out + (size_t)i * row, src + (size_t)r * row, row * sizeof(float));
    }
    return KVO_OK;
}

/* remove (kv_block_pool.cpp:148-161): blocks released in table order. */
int kvo_remove(kvo_pool* p, uint64_t id) {
    kvo_seq* s = find_seq(p, id);
    if (!s) return KVO_ENOSEQ;
    for (int64_t i = 0; i < s->n_blocks; i++) release_block(p, s->table[i]);
    free(s->table);
    int64_t idx = s - p->seqs;
    memmove(p->seqs + idx, p->seqs + idx + 1, sizeof(kvo_seq) * (size_t)(p->n_seqs - idx - 1));
    p->n_seqs--;
    return KVO_OK;
}

/* truncate (kv_block_pool.cpp:163-190): tail blocks released last-first. */
int kvo_truncate(kvo_pool* p, uint64_t id, int64_t keep) {
    kvo_seq* s = find_seq(p, id);
    if (!s) return KVO_ENOSEQ;
    if (keep >= seq_len(p, s)) return KVO_OK;
    int64_t keep_blocks = 0, in_last = 0;
    if (keep > 0) {
        keep_blocks = (keep - 1) / p->bs + 1;
        in_last = keep - (keep_blocks - 1) * p->bs;
    }
    while (s->n_blocks > keep_blocks) release_block(p, s->table[--s->n_blocks]);
    s->tokens_in_last = in_last;
    return KVO_OK;
}

int kvo_block_table(const kvo_pool* p, uint64_t id, int32_t* out, int64_t cap, int64_t* n) {
    const kvo_seq* s = find_seq(p, id);
    if (!s) return KVO_ENOSEQ;
    int64_t m = s->n_blocks < cap ? s->n_blocks : cap;
    memcpy(out, s->table, sizeof(int32_t) * (size_t)m);
    *n = s->n_blocks;
    return KVO_OK;
}

int32_t kvo_refcount(const kvo_pool* p, int32_t b) {
    if (b < 0 || b >= p->max_blocks) return -1;
    return p->rc[b];
}

int kvo_is_cached(const kvo_pool* p, int32_t b) { return p->cached[b] != 0; }

/* fork: dst shares src's first ceil(n / bs) blocks (refcount + 1 each); no
 * data moves until one side appends into the shared partial tail. */
int kvo_fork(kvo_pool* p, uint64_t src, uint64_t dst, int64_t n) {
    kvo_seq* s = find_seq(p, src);
    if (!s) return KVO_ENOSEQ;
    if (find_seq(p, dst) || n < 0 || n > seq_len(p, s)) return KVO_EINVAL;
    int64_t nb = n > 0 ? (n - 1) / p->bs + 1 : 0;
    int32_t* tb = (int32_t*)malloc(sizeof(int32_t) * (size_t)(nb + 1));
    memcpy(tb, s->table, sizeof(int32_t) * (size_t)nb);
    kvo_seq* d = get_or_create(p, dst); /* may move s */
    for (int64_t i = 0; i < nb; i++) {
        seq_push(d, tb[i]);
        p->rc[tb[i]]++;
    }
    d->tokens_in_last = nb > 0 ? n - (nb - 1) * p->bs : 0;
    free(tb);
    return KVO_OK;
}

/* ---- hashed prefix cache ---- */

/* Chained 64-bit hash of one block of token ids: FNV-1a over the parent
 * hash and the ids, then a splitmix64 finaliser. */
uint64_t kvo_block_hash(uint64_t parent, const int32_t* tokens, int64_t bs) {
    uint64_t h = 0xcbf29ce484222325ull;
    for (int i = 0; i < 8; i++) {
        h ^= (parent >> (8 * i)) & 0xFF;
        h *= 0x100000001b3ull;
    }
    for (int64_t t = 0; t < bs; t++) {
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

static int64_t cache_find(const kvo_pool* p, uint64_t h, uint64_t parent, const int32_t* tokens) {
    for (int64_t i = 0; i < p->n_cache; i++) {
        const kvo_cached* c = &p->cache[i];
        if (c->hash == h && c->parent == parent && memcmp(c->tokens, tokens, sizeof(int32_t) * (size_t)p->bs) == 0)
            return i;
    }
    return -1;
}

/* Register seq's full blocks covering tokens[0:n) under chained hashes.
 * A block already registered, or a chain link whose hash is already held
 * by another block, is skipped.  Returns the number of newly cached blocks. */
int64_t kvo_prefix_insert(kvo_pool* p, uint64_t id, const int32_t* tokens, int64_t n) {
    kvo_seq* s = find_seq(p, id);
    if (!s || n > seq_len(p, s)) return -1;
    int64_t nb = n / p->bs, added = 0;
    uint64_t parent = 0;
    for (int64_t i = 0; i < nb; i++) {
        const int32_t* tk = tokens + i * p->bs;
        uint64_t h = kvo_block_hash(parent, tk, p->bs);
        int32_t b = s->table[i];
        if (cache_find(p, h, parent, tk) < 0 && !p->cached[b]) {
            if (p->n_cache == p->cap_cache) {
                p->cap_cache = p->cap_cache ? p->cap_cache * 2 : 64;
                p->cache = (kvo_cached*)realloc(p->cache, sizeof(kvo_cached) * (size_t)p->cap_cache);
            }
            kvo_cached* c = &p->cache[p->n_cache++];
            c->hash = h;
            c->parent = parent;
            c->block = b;
            c->tokens = (int32_t*)malloc(sizeof(int32_t) * (size_t)p->bs);
            memcpy(c->tokens, tk, sizeof(int32_t) * (size_t)p->bs);
            p->cached[b] = (int32_t)p->n_cache;
            added++;
        }
        parent = h;
    }
    return added;
}

/* Start sequence dst from the longest cached chain matching tokens[0:n);
 * each hit block gains a reference (leaving the LRU if it was idle).
 * Returns the number of tokens covered (a multiple of bs). */
int kvo_prefix_match(kvo_pool* p, uint64_t dst, const int32_t* tokens, int64_t n, int64_t* n_hit) {
    if (find_seq(p, dst)) return KVO_EINVAL;
    kvo_seq* d = get_or_create(p, dst);
    int64_t nb = n / p->bs, hit = 0;
    uint64_t parent = 0;
    for (int64_t i = 0; i < nb; i++) {
        const int32_t* tk = tokens + i * p->bs;
        uint64_t h = kvo_block_hash(parent, tk, p->bs);
        int64_t ci = cache_find(p, h, parent, tk);
        if (ci < 0) break;
        int32_t b = p->cache[ci].block;
        if (p->rc[b] == 0) lru_remove(p, b);
        p->rc[b]++;
        seq_push(d, b);
        hit++;
        parent = h;
    }
    d->tokens_in_last = hit > 0 ? p->bs : 0;
    *n_hit = hit * p->bs;
    return KVO_OK;
}

/* ======================= int8 projections ======================= */

/* quantize_tensor (src/quantized_tensor.cpp:9-47): per row, scale =
 * max|w| / 127 (1 when the row is all zero), q = round(w / scale) with
 * ties away from zero (std::round), cast to int8. */
void kvo_quantize_rows(const float* w, int64_t rows, int64_t cols, int8_t* q, float* scales) {
    for (int64_t r = 0; r < rows; r++) {
        float mx = 0.0f;
        for (int64_t c = 0; c < cols; c++) {
            float a = fabsf(w[r * cols + c]);
            mx = (mx < a) ? a : mx; /* std::max(row_max, |val|), NaN included */
        }
        float scale = (mx > 0.0f) ? mx / 127.0f : 1.0f;
        scales[r] = scale;
        for (int64_t c = 0; c < cols; c++) q[r * cols + c] = (int8_t)roundf(w[r * cols + c] / scale);
    }
}

/* matmul_quantized_range_blocked (src/quantized_tensor.cpp:60-100) over all
 * columns: out[i][j] = sum over k in order of x[i][k] * (q[k][j] * s[k]),
 * each product and sum rounded to fp32 on its own (the AVX lanes and the
 * scalar tail compute the same sequence). */
void kvo_matmul_int8(const float* x, int64_t M, int64_t K, const int8_t* q, const float* s, int64_t N, float* out) {
    for (int64_t i = 0; i < M; i++)
        for (int64_t j = 0; j < N; j++) {
            float sum = 0.0f;
            for (int64_t k = 0; k < K; k++) {
                float b = (float)q[k * N + j] * s[k];
                float prod = x[i * K + k] * b;
                sum = sum + prod;
            }
            out[i * N + j] = sum;
        }
}
