// api.cpp -- C-ABI entry points that launch device work: the batched step
// (begin / rope_append / attention / host-buffer layer step / end) and the
// single-call kernels (append, rope_append, apply_rope, gather, cow_copy,
// attention, attention_contig).
//
// A batch does the host bookkeeping of one decode or prefill step once for
// all layers: it reserves slots (KVBlockPool::append's allocation,
// kv_block_pool.cpp:20-65), derives positions (start_pos = length before
// the append, src/nn/attention.cpp:304), plans the split-K work list, and
// uploads slots, positions, rows and work items in one copy.  Every layer's
// kernels then reuse that upload.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>

#include "internal.h"

namespace s1kv {
int flush(s1kv_pool* p, cudaStream_t stream);
int seq_row(const s1kv_pool* p, uint64_t id, int32_t* row, int64_t* len);
int reserve_internal(s1kv_pool* p, uint64_t id, int64_t n, int32_t* slots, int64_t* n_done);

namespace {

constexpr int kSMs = 148;

size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

int check_pool(const s1kv_pool* p) {
    if (!p) return set_error(S1KV_EINVAL, "s1kv: null pool");
    if (p->host_only) return set_error(S1KV_EINVAL, "s1kv: host-only pool has no device storage");
    return S1KV_OK;
}

int check_layer(const s1kv_pool* p, int32_t layer) {
    if (layer < 0 || layer >= p->desc.num_layers)
        return set_error(S1KV_EINVAL, "s1kv: layer %d out of range [0, %d)", layer, p->desc.num_layers);
    return S1KV_OK;
}

// Split-K plan: tiles of 16 tokens; the split length (in tiles) targets
// about 8 waves of CTAs over the 148 SMs, at least one tile per warp, at
// most 32 tiles per warp where the rows allow it (the kernels prefetch 32
// block ids per warp and look further ones up as they go), and no more than
// kMaxSplitsPerRow splits of the longest row (the merge's counters and
// groups are sized for that).
int32_t plan_split_tiles(int64_t total_tiles, int64_t max_row_tiles, int32_t Hkv, int nw) {
    int64_t target = (int64_t)kSMs * 8;
    int64_t s = (total_tiles * Hkv + target - 1) / target;
    s = std::max<int64_t>(s, nw);
    s = std::min<int64_t>(s, 32 * nw);
    s = std::max<int64_t>(s, (max_row_tiles + kMaxSplitsPerRow - 1) / kMaxSplitsPerRow);
    return (int32_t)s;
}

float scale_log2(int D) { return 1.4426950408889634f / std::sqrt((float)D); }

// Split-K work list of a batch's query rows (host): split length, per-row
// split count and partial offset, items longest first.
void plan_items(const s1kv_pool* p, s1kv_batch* b) {
    const int32_t bs = p->desc.block_size;
    const int nw = tma_warps_per_cta(p->desc.dtype, p->desc.head_dim);
    int64_t total_tiles = 0, max_row_tiles = 0;
    for (const RowMeta& m : b->rows) {
        total_tiles += (m.kv_len + bs - 1) / bs;
        max_row_tiles = std::max<int64_t>(max_row_tiles, (m.kv_len + bs - 1) / bs);
    }
    b->split_tokens = plan_split_tiles(total_tiles, max_row_tiles, p->desc.num_kv_heads, nw) * 16;
    std::vector<WorkItem>& items = b->items;
    items.clear();
    int64_t n_part = 0;
    for (int64_t r = 0; r < (int64_t)b->rows.size(); r++) {
        RowMeta& m = b->rows[r];
        m.n_split = (m.kv_len + b->split_tokens - 1) / b->split_tokens;
        m.part_off = (int32_t)n_part;
        if (m.n_split > 1) n_part += m.n_split;
        for (int32_t s = 0; s < m.n_split; s++) items.push_back({(int32_t)r, s, m.table_row, m.kv_len});
    }
    // Longest work first: full splits, then the tails by length.
    auto item_tokens = [&](const WorkItem& w) {
        return std::min<int64_t>(b->split_tokens, b->rows[w.row].kv_len - (int64_t)w.split * b->split_tokens);
    };
    std::stable_sort(items.begin(), items.end(),
                     [&](const WorkItem& a, const WorkItem& c) { return item_tokens(a) > item_tokens(c); });
    b->n_items = (int64_t)items.size();
    b->n_part = n_part;
    b->items_planned = true;
}

}  // namespace
}  // namespace s1kv

using namespace s1kv;

extern "C" {

int s1kv_batch_begin(s1kv_pool* p, const uint64_t* seqs, const int32_t* n_append, const int32_t* q_lens,
                     int32_t n_seqs, void* stream_, s1kv_batch** out) {
    int st = check_pool(p);
    if (st) return st;
    if (!out || (n_seqs > 0 && !seqs) || n_seqs < 0) return set_error(S1KV_EINVAL, "s1kv_batch_begin: bad arguments");
    *out = nullptr;
    cudaStream_t stream = (cudaStream_t)stream_;
    S1KV_ON_DEVICE(p->device);

    auto* b = new s1kv_batch();
    b->pool = p;
    std::vector<int32_t> slots, pos;
    std::vector<int64_t> lens(n_seqs);
    std::vector<int32_t> trow(n_seqs);
    int64_t n_tok = 0;
    for (int32_t i = 0; i < n_seqs; i++) {
        n_tok += n_append ? std::max<int32_t>(n_append[i], 0) : 0;
        b->max_append = std::max<int32_t>(b->max_append, n_append ? n_append[i] : 0);
    }
    slots.resize(n_tok);
    pos.resize(n_tok);
    int64_t off = 0;
    // A failed reservation rolls back every sequence this call touched
    // (truncate to the old length, or remove if the call created it), so a
    // step is all-or-nothing.  Truncation pushes the blocks back in reverse
    // allocation order, which restores the free list's order.
    std::vector<std::pair<int64_t, bool>> before(n_seqs);
    auto rollback = [&](int32_t upto) {
        for (int32_t j = upto; j >= 0; j--) {
            if (before[j].second) s1kv_seq_truncate(p, seqs[j], before[j].first);
            else if (s1kv_seq_exists(p, seqs[j])) s1kv_seq_remove(p, seqs[j]);
        }
    };
    for (int32_t i = 0; i < n_seqs; i++) {
        const int32_t na = n_append ? n_append[i] : 0;
        if (na < 0) {
            rollback(i - 1);
            delete b;
            return set_error(S1KV_EINVAL, "s1kv_batch_begin: negative n_append");
        }
        const int64_t old = s1kv_seq_length(p, seqs[i]);
        before[i] = {old, s1kv_seq_exists(p, seqs[i]) != 0};
        if (n_append) {
            int64_t done = 0;
            st = reserve_internal(p, seqs[i], na, slots.data() + off, &done);
            if (st) {
                std::string msg = s1kv_last_error();
                rollback(i);
                delete b;
                return set_error(st, "%s", msg.c_str());
            }
        }
        for (int32_t t = 0; t < na; t++) pos[off + t] = (int32_t)(old + t);
        off += na;
        st = seq_row(p, seqs[i], &trow[i], &lens[i]);
        if (st) {
            delete b;
            return st;
        }
    }
    b->n_tokens = n_tok;
    b->max_pos = p->max_len_seen;

    // Attention rows: row r of sequence i attends to (L - q_len) + r + 1
    // tokens (the causal limit of attention.cpp:181, plus one).
    int64_t n_rows = 0;
    for (int32_t i = 0; i < n_seqs; i++) {
        const int32_t ql = q_lens ? q_lens[i] : (n_append ? n_append[i] : 0);
        if (ql < 0 || ql > lens[i]) {
            if (n_append) rollback(n_seqs - 1);
            delete b;
            return set_error(S1KV_EINVAL, "s1kv_batch_begin: q_len %d exceeds sequence length %lld", ql,
                             (long long)lens[i]);
        }
        if (ql != 1 && ql != 0) b->decode_rows = false;
        if (ql != (n_append ? n_append[i] : 0)) b->rows_are_tokens = false;
        n_rows += ql;
    }
    b->rows.resize(n_rows);
    {
        int64_t r = 0;
        for (int32_t i = 0; i < n_seqs; i++) {
            const int32_t ql = q_lens ? q_lens[i] : (n_append ? n_append[i] : 0);
            for (int32_t j = 0; j < ql; j++, r++) {
                RowMeta& m = b->rows[r];
                m.table_row = trow[i];
                m.kv_len = (int32_t)(lens[i] - ql + j + 1);
                m.n_split = 1;
                m.part_off = 0;
            }
        }
    }
    // Decode batches get their split-K work list now.  Query chunks take the
    // tensor-core prefill, which does not use it; it is planned on demand if
    // such a batch falls back to the split-K kernels.
    if (b->decode_rows) plan_items(p, b);
    const std::vector<WorkItem>& items = b->items;
    b->n_rows = n_rows;
    // Per-sequence view of the same rows, for the tensor-core prefill.
    std::vector<PrefillSeq> pseqs(n_seqs);
    {
        int32_t q_start = 0;
        for (int32_t i = 0; i < n_seqs; i++) {
            const int32_t ql = q_lens ? q_lens[i] : (n_append ? n_append[i] : 0);
            pseqs[i] = PrefillSeq{trow[i], (int32_t)lens[i], ql, q_start};
            q_start += ql;
            b->max_qlen = std::max(b->max_qlen, ql);
        }
    }
    b->n_seqs = n_seqs;

    // Device block tables and pending copy-on-write copies first.
    st = flush(p, stream);
    if (st) {
        delete b;
        return st;
    }
    // One upload of the step's metadata.  The per-row records go up only
    // with a decode batch's work list: query chunks take the tensor-core
    // prefill (per-sequence records), and a chunk batch that falls back to
    // the split-K kernels uploads its rows with its late-planned work list.
    const int64_t up_rows = b->items_planned ? n_rows : 0;
    size_t o_slots = 0, o_pos = align16(o_slots + n_tok * 4), o_rows = align16(o_pos + n_tok * 4),
           o_items = align16(o_rows + up_rows * sizeof(RowMeta)), o_pseq = align16(o_items + items.size() * sizeof(WorkItem)),
           o_qpos = align16(o_pseq + pseqs.size() * sizeof(PrefillSeq)),
           total = align16(o_qpos + (b->rows_are_tokens ? 0 : n_rows * 4));
    st = p->stager.acquire(total + 16, &b->seg);
    if (st) {
        delete b;
        return st;
    }
    char* h = b->seg->h;
    std::memcpy(h + o_slots, slots.data(), n_tok * 4);
    std::memcpy(h + o_pos, pos.data(), n_tok * 4);
    std::memcpy(h + o_rows, b->rows.data(), up_rows * sizeof(RowMeta));
    std::memcpy(h + o_items, items.data(), items.size() * sizeof(WorkItem));
    std::memcpy(h + o_pseq, pseqs.data(), pseqs.size() * sizeof(PrefillSeq));
    if (!b->rows_are_tokens) {
        int32_t* qp = reinterpret_cast<int32_t*>(h + o_qpos);
        for (int64_t r = 0; r < n_rows; r++) qp[r] = b->rows[r].kv_len - 1;
    }
    if (total) S1KV_CUDA(cudaMemcpyAsync(b->seg->d, h, total, cudaMemcpyHostToDevice, stream));
    b->d_slots = (const int32_t*)(b->seg->d + o_slots);
    b->d_pos = (const int32_t*)(b->seg->d + o_pos);
    b->d_rows = up_rows ? (const RowMeta*)(b->seg->d + o_rows) : nullptr;
    b->d_items = (const WorkItem*)(b->seg->d + o_items);
    b->items_uploaded = b->items_planned;
    b->d_pseqs = (const PrefillSeq*)(b->seg->d + o_pseq);
    b->d_qpos = b->rows_are_tokens ? nullptr : (const int32_t*)(b->seg->d + o_qpos);
    *out = b;
    return S1KV_OK;
}

int s1kv_batch_sizes(const s1kv_batch* b, int64_t* n_tokens, int64_t* n_rows) {
    if (!b) return set_error(S1KV_EINVAL, "null batch");
    if (n_tokens) *n_tokens = b->n_tokens;
    if (n_rows) *n_rows = b->n_rows;
    return S1KV_OK;
}

int s1kv_batch_plan(const s1kv_batch* b, int32_t* split_tokens, int64_t* n_items) {
    if (!b) return set_error(S1KV_EINVAL, "null batch");
    if (!b->items_planned) plan_items(b->pool, const_cast<s1kv_batch*>(b));
    if (split_tokens) *split_tokens = b->split_tokens;
    if (n_items) *n_items = b->n_items;
    return S1KV_OK;
}

static int batch_append_impl(s1kv_batch* b, int32_t layer, const float* q_in, float* q_out, int32_t Hq,
                             const float* k, const float* v, bool rope, cudaStream_t stream) {
    s1kv_pool* p = b->pool;
    int st = check_layer(p, layer);
    if (st) return st;
    if (b->n_tokens == 0 && !(rope && q_in && b->n_rows)) return S1KV_OK;
    S1KV_ON_DEVICE(p->device);
    if (b->n_tokens && (!k || !v)) return set_error(S1KV_EINVAL, "s1kv_batch_append: null k/v");
    if (q_in && (!q_out || Hq <= 0))
        return set_error(S1KV_EINVAL, "s1kv_batch_rope_append: q needs q_out and n_q_heads");
    // Query rows that are exactly the appended tokens rotate in the append
    // kernel; otherwise (a step mixing prompt appends without queries and
    // decode rows) q is rotated by row position in a second launch.
    const bool fused_q = rope && q_in && b->rows_are_tokens;
    AppendParams ap{};
    ap.k = k;
    ap.v = v;
    ap.q_in = fused_q ? q_in : nullptr;
    ap.q_out = q_out;
    ap.slots = b->d_slots;
    ap.pos = b->d_pos;
    ap.kpool = p->k + (size_t)layer * p->layer_bytes;
    ap.vpool = p->v + (size_t)layer * p->layer_bytes;
    ap.num_slots = p->num_slots;
    ap.n = b->n_tokens;
    ap.Hkv = p->desc.num_kv_heads;
    ap.Hq = Hq;
    ap.D = p->desc.head_dim;
    ap.err = p->d_err;
    if (rope) {
        ap.rope = rope_table(p->device, p->desc.head_dim, p->desc.rope_theta, std::max<int64_t>(b->max_pos, 1),
                             &ap.rope_cap, stream, &st);
        if (st) return st;
    }
    if (b->n_tokens) {
        st = launch_append(ap, p->desc.dtype, rope, stream, true);
        if (st) return st;
    }
    if (rope && q_in && !fused_q && b->n_rows)
        return launch_rope(q_in, q_out, ap.rope, ap.rope_cap, 0, b->n_rows, Hq, p->desc.head_dim, p->d_err, stream,
                           b->d_qpos);
    return S1KV_OK;
}

int s1kv_batch_rope_append(s1kv_batch* b, int32_t layer, const float* q_in, float* q_out, int32_t Hq, const float* k,
                           const float* v, void* stream) {
    if (!b) return set_error(S1KV_EINVAL, "null batch");
    return batch_append_impl(b, layer, q_in, q_out, Hq, k, v, true, (cudaStream_t)stream);
}

int s1kv_batch_norm_rope_append(s1kv_batch* b, int32_t layer, const float* q_in, float* q_out, int32_t Hq,
                                const float* q_norm_weight, const float* k, const float* v, const float* k_norm_weight,
                                float eps, void* stream_) {
    if (!b) return set_error(S1KV_EINVAL, "null batch");
    s1kv_pool* p = b->pool;
    int st = check_layer(p, layer);
    if (st) return st;
    const bool with_q = q_in && b->n_rows;
    if (b->n_tokens == 0 && !with_q) return S1KV_OK;
    S1KV_ON_DEVICE(p->device);
    cudaStream_t stream = (cudaStream_t)stream_;
    if (b->n_tokens && (!k || !v || !k_norm_weight))
        return set_error(S1KV_EINVAL, "s1kv_batch_norm_rope_append: null k/v/k_norm_weight");
    if (with_q && (!q_out || Hq <= 0 || !q_norm_weight))
        return set_error(S1KV_EINVAL, "s1kv_batch_norm_rope_append: q needs q_out, n_q_heads and q_norm_weight");
    if ((((uintptr_t)q_in | (uintptr_t)q_out | (uintptr_t)k | (uintptr_t)v) & 15) != 0)
        return set_error(S1KV_EINVAL, "s1kv_batch_norm_rope_append: q/k/v must be 16-byte aligned");
    AppendParams ap{};
    ap.k = k;
    ap.v = v;
    ap.q_in = with_q ? q_in : nullptr;
    ap.q_out = q_out;
    ap.slots = b->d_slots;
    ap.pos = b->d_pos;
    ap.kpool = p->k + (size_t)layer * p->layer_bytes;
    ap.vpool = p->v + (size_t)layer * p->layer_bytes;
    ap.num_slots = p->num_slots;
    ap.n = b->n_tokens;
    ap.Hkv = p->desc.num_kv_heads;
    ap.Hq = Hq;
    ap.D = p->desc.head_dim;
    ap.err = p->d_err;
    ap.rope = rope_table(p->device, p->desc.head_dim, p->desc.rope_theta, std::max<int64_t>(b->max_pos, 1), &ap.rope_cap,
                         stream, &st);
    if (st) return st;
    // query row i is token i unless the step mixes prompt appends without
    // queries and decode rows; then each row has its own position
    const int32_t* qpos = b->rows_are_tokens ? b->d_pos : b->d_qpos;
    return launch_norm_rope_append(ap, p->desc.dtype, q_norm_weight, k_norm_weight, eps, qpos, b->n_rows, stream);
}

int s1kv_batch_append(s1kv_batch* b, int32_t layer, const float* k, const float* v, void* stream) {
    if (!b) return set_error(S1KV_EINVAL, "null batch");
    return batch_append_impl(b, layer, nullptr, nullptr, 0, k, v, false, (cudaStream_t)stream);
}

}  // extern "C"

// The split-K decode path of s1kv_batch_attention; `ex` (optional) places the
// finished rows into the peer exchange.
static int split_k_attention(s1kv_batch* b, int32_t layer, const float* q, float* out, int32_t Hq,
                             const AttnParams* ex, cudaStream_t stream) {
    s1kv_pool* p = b->pool;
    int st = S1KV_OK;
    const int32_t Hkv = p->desc.num_kv_heads, D = p->desc.head_dim;
    const int G = Hq / Hkv;
    if (!b->items_uploaded) {
        // A query-chunk batch on the split-K kernels (shapes or alignments the
        // tensor-core prefill does not take): plan and upload its work list.
        if (!b->items_planned) plan_items(p, b);
        const size_t rb = b->rows.size() * sizeof(RowMeta), ib = b->items.size() * sizeof(WorkItem);
        st = p->late_meta.ensure(align16(rb) + ib + 16);
        if (st) return st;
        char* d = (char*)p->late_meta.p;
        S1KV_CUDA(cudaMemcpyAsync(d, b->rows.data(), rb, cudaMemcpyHostToDevice, stream));
        S1KV_CUDA(cudaMemcpyAsync(d + align16(rb), b->items.data(), ib, cudaMemcpyHostToDevice, stream));
        S1KV_CUDA(cudaStreamSynchronize(stream));  // the host vectors are pageable
        b->d_rows = (const RowMeta*)d;
        b->d_items = (const WorkItem*)(d + align16(rb));
        b->items_uploaded = true;
    }
    size_t need = (size_t)b->n_part * Hkv * G * (D + 2) * sizeof(float);
    if (need) {
        st = p->scratch.ensure(need);
        if (st) return st;
    }
    AttnParams ap{};
    ap.q = q;
    ap.out = out;
    ap.part_o = (float*)p->scratch.p;
    ap.part_ml = ap.part_o ? ap.part_o + (size_t)b->n_part * Hkv * G * D : nullptr;
    ap.table = p->d_table;
    ap.rows = b->d_rows;
    ap.items = b->d_items;
    ap.kbase = p->k + (size_t)layer * p->layer_bytes;
    ap.vbase = p->v + (size_t)layer * p->layer_bytes;
    ap.num_slots = p->num_slots;
    ap.max_bps = p->max_bps;
    ap.max_blocks = (int32_t)p->desc.max_blocks;
    ap.n_rows = (int32_t)b->n_rows;
    ap.n_items = (int32_t)b->n_items;
    ap.split_tokens = b->split_tokens;
    ap.block_size = p->desc.block_size;
    ap.Hq = Hq;
    ap.Hkv = Hkv;
    ap.D = D;
    ap.layer = layer;
    ap.scale_log2 = scale_log2(D);
    ap.err = p->d_err;
    // Decode rows: the kernels request the K/V tiles that lie entirely below
    // the last max_append tokens of each row before their wait for the
    // previous kernel of the stream.  Safe because the kernels of this
    // library that may still run then write the pool only at this batch's
    // appended tokens (the batch's RoPE + append of any layer; the decode
    // kernels read it): every other write of the pool -- single-call
    // appends, copy-on-write copies, block-table updates, prefix loads -- is
    // a plain launch or a copy, complete before any later kernel starts, and
    // the step's metadata is uploaded before the batch's first kernel.
    if (b->decode_rows) {
        ap.prewait = 1;
        ap.prewait_margin = b->max_append;
    }
    const size_t cbytes = (size_t)b->n_rows * Hkv * kCounterStride * sizeof(int32_t);
    if (p->counters.cap < cbytes) {
        st = p->counters.ensure(cbytes);
        if (st) return st;
        S1KV_CUDA(cudaMemsetAsync(p->counters.p, 0, p->counters.cap, stream));
    }
    ap.counters = (int32_t*)p->counters.p;
    if (ex) {
        ap.out_stride = ex->out_stride;
        ap.out_head0 = ex->out_head0;
        ap.n_peers = ex->n_peers;
        ap.xout = ex->xout;
        for (int k = 0; k < 7; k++) ap.xpeer[k] = ex->xpeer[k];
        ap.epoch = ex->epoch;
    }
    return launch_attention(p, ap, p->desc.dtype, stream);
}

extern "C" {

int s1kv_batch_attention(s1kv_batch* b, int32_t layer, const float* q, float* out, int32_t Hq, void* stream_) {
    if (!b) return set_error(S1KV_EINVAL, "null batch");
    s1kv_pool* p = b->pool;
    int st = check_layer(p, layer);
    if (st) return st;
    S1KV_ON_DEVICE(p->device);
    const int32_t Hkv = p->desc.num_kv_heads, D = p->desc.head_dim;
    if (Hq <= 0 || Hq % Hkv) return set_error(S1KV_EINVAL, "s1kv_batch_attention: n_q_heads must be a multiple of num_kv_heads");
    if (b->n_rows == 0) return S1KV_OK;
    if (!q || !out) return set_error(S1KV_EINVAL, "s1kv_batch_attention: null q/out");
    const int G = Hq / Hkv;
    cudaStream_t stream = (cudaStream_t)stream_;
    // Chunks of several query rows per sequence over bf16 K/V are a dense
    // contraction: tensor-core prefill.  Decode rows stay on the split-K
    // kernel.
    // (q and out are read and written by TMA there: 16-byte aligned.)
    if (!b->decode_rows && p->tmap_sw_ok && prefill_tc_supported(p->desc.dtype, D, G, p->desc.block_size) &&
        (((uintptr_t)q | (uintptr_t)out) & 15) == 0) {
        PrefillParams pp{};
        pp.q = q;
        pp.out = out;
        pp.table = p->d_table;
        pp.seqs = b->d_pseqs;
        pp.n_seqs = b->n_seqs;
        pp.max_chunks = (b->max_qlen + prefill_queries_per_cta(G) - 1) / prefill_queries_per_cta(G);
        pp.max_bps = p->max_bps;
        pp.max_blocks = (int32_t)p->desc.max_blocks;
        pp.Hq = Hq;
        pp.Hkv = Hkv;
        pp.layer = layer;
        pp.scale_log2 = scale_log2(D);
        pp.n_rows = b->n_rows;
        pp.err = p->d_err;
        if (pp.n_seqs == 0 || pp.max_chunks == 0) return S1KV_OK;
        return launch_prefill_tc(pp, p->tmap_k_sw, p->tmap_v_sw, stream);
    }
    return split_k_attention(b, layer, q, out, Hq, nullptr, stream);
}

int s1kv_batch_attention_exchange(s1kv_batch* b, int32_t layer, const float* q, int32_t Hq, s1kv_exchange* ex,
                                  int32_t head0, int32_t heads_total, uint32_t epoch, void* stream_) {
    if (!b || !ex) return set_error(S1KV_EINVAL, "null batch or exchange");
    s1kv_pool* p = b->pool;
    int st = check_layer(p, layer);
    if (st) return st;
    if (ex->device != p->device) return set_error(S1KV_EINVAL, "exchange and pool are on different devices");
    S1KV_ON_DEVICE(p->device);
    const int32_t Hkv = p->desc.num_kv_heads, D = p->desc.head_dim;
    if (Hq <= 0 || Hq % Hkv) return set_error(S1KV_EINVAL, "n_q_heads must be a multiple of num_kv_heads");
    const int G = Hq / Hkv;
    if (!b->decode_rows || !q) return set_error(S1KV_EINVAL, "exchange: decode batches only (one query row per sequence)");
    if (!p->tmap_ok || !(decode_mma_supported(p->desc.dtype, D, G, p->desc.block_size) ||
                         tma_attention_supported(p->desc.dtype, D, G, p->desc.block_size)))
        return set_error(S1KV_EINVAL, "exchange: shape not served by the split-K decode kernels");
    if (head0 < 0 || head0 + Hq > heads_total || (int64_t)b->n_rows * heads_total * D > ex->slot_floats)
        return set_error(S1KV_EINVAL, "exchange: rows x heads x head_dim exceed the exchange slot");
    if (epoch == 0) return set_error(S1KV_EINVAL, "exchange: epochs start at 1 (0 is the zeroed slot's)");
    AttnParams ex_p{};
    st = exchange_params(ex, epoch, head0, heads_total, &ex_p);
    if (st) return st;
    exchange_record(ex, epoch, (int64_t)b->n_rows * heads_total * D);
    if (b->n_rows == 0) return S1KV_OK;
    return split_k_attention(b, layer, q, nullptr, Hq, &ex_p, (cudaStream_t)stream_);
}

int s1kv_batch_layer_host(s1kv_batch* b, int32_t layer, const float* h_q, const float* h_k, const float* h_v,
                          float* h_out, int32_t Hq, void* stream_) {
    if (!b) return set_error(S1KV_EINVAL, "null batch");
    s1kv_pool* p = b->pool;
    S1KV_ON_DEVICE(p->device);
    cudaStream_t stream = (cudaStream_t)stream_;
    const int64_t D = p->desc.head_dim, Hkv = p->desc.num_kv_heads;
    const size_t qb = (size_t)b->n_rows * Hq * D * 4, kb = (size_t)b->n_tokens * Hkv * D * 4;
    const size_t oq = 0, ok = align16(qb), ov = ok + align16(kb), oqr = ov + align16(kb), oo = oqr + align16(qb),
                 slot_bytes = align16(oo + align16(qb));
    int st = p->io.ensure(2 * slot_bytes);
    if (st) return st;
    // Two slots alternate between calls: the inputs of this call go up on
    // the copy stream while the previous call's kernels run, and its output
    // comes back on the second copy stream while the next call's run.
    const int s = b->io_calls++ & 1;
    char* d = (char*)p->io.p + s * slot_bytes;
    cudaEvent_t in_ready = p->io_ev[s], slot_done = p->io_ev[2 + s], out_done = p->io_ev[4 + s];
    if (slot_bytes != p->io_slot_bytes) {
        // the slots moved: this slot may overlap either slot of earlier calls,
        // so wait for both before touching it
        for (int o = 0; o < 2; o++)
            if (p->io_slot_used[o]) {
                S1KV_CUDA(cudaStreamWaitEvent(p->copy_stream, p->io_ev[2 + o], 0));
                S1KV_CUDA(cudaStreamWaitEvent(p->copy_stream, p->io_ev[4 + o], 0));
                S1KV_CUDA(cudaStreamWaitEvent(stream, p->io_ev[4 + o], 0));
            }
        p->io_slot_bytes = slot_bytes;
    }
    if (p->io_slot_used[s]) S1KV_CUDA(cudaStreamWaitEvent(p->copy_stream, slot_done, 0));  // inputs consumed
    if (qb) S1KV_CUDA(cudaMemcpyAsync(d + oq, h_q, qb, cudaMemcpyHostToDevice, p->copy_stream));
    if (kb) {
        S1KV_CUDA(cudaMemcpyAsync(d + ok, h_k, kb, cudaMemcpyHostToDevice, p->copy_stream));
        S1KV_CUDA(cudaMemcpyAsync(d + ov, h_v, kb, cudaMemcpyHostToDevice, p->copy_stream));
    }
    S1KV_CUDA(cudaEventRecord(in_ready, p->copy_stream));
    S1KV_CUDA(cudaStreamWaitEvent(stream, in_ready, 0));
    if (p->io_slot_used[s]) S1KV_CUDA(cudaStreamWaitEvent(stream, out_done, 0));  // the slot's output read back
    const bool q_rows_are_tokens = b->n_rows == b->n_tokens && b->n_tokens > 0;
    st = s1kv_batch_rope_append(b, layer, q_rows_are_tokens ? (const float*)(d + oq) : nullptr, (float*)(d + oqr), Hq,
                                (const float*)(d + ok), (const float*)(d + ov), stream);
    if (st) return st;
    const float* qa = q_rows_are_tokens ? (const float*)(d + oqr) : (const float*)(d + oq);
    st = s1kv_batch_attention(b, layer, qa, (float*)(d + oo), Hq, stream);
    if (st) return st;
    S1KV_CUDA(cudaEventRecord(slot_done, stream));
    S1KV_CUDA(cudaStreamWaitEvent(p->d2h_stream, slot_done, 0));
    if (qb) S1KV_CUDA(cudaMemcpyAsync(h_out, d + oo, qb, cudaMemcpyDeviceToHost, p->d2h_stream));
    S1KV_CUDA(cudaEventRecord(out_done, p->d2h_stream));
    p->io_slot_used[s] = true;
    return S1KV_OK;
}

int s1kv_batch_end(s1kv_batch* b, void* stream) {
    if (!b) return S1KV_OK;
    S1KV_ON_DEVICE(b->pool->device);
    int st = S1KV_OK;
    // host outputs of s1kv_batch_layer_host are complete once the stream
    // passes this point
    for (int s = 0; s < 2 && s < b->io_calls; s++)
        if (cudaStreamWaitEvent((cudaStream_t)stream, b->pool->io_ev[4 + s], 0) != cudaSuccess)
            st = set_error(S1KV_ECUDA, "s1kv_batch_end: waiting for host copies");
    if (b->seg) st = b->pool->stager.release(b->seg, (cudaStream_t)stream);
    delete b;
    return st;
}

// ------------------------------------------------------ single-call API --

int s1kv_append(s1kv_pool* p, int32_t layer, const float* k, const float* v, const int32_t* slots, int64_t n,
                void* stream) {
    int st = check_pool(p);
    if (!st) st = check_layer(p, layer);
    if (st) return st;
    S1KV_ON_DEVICE(p->device);
    st = flush(p, (cudaStream_t)stream);
    if (st) return st;
    AppendParams ap{};
    ap.k = k;
    ap.v = v;
    ap.slots = slots;
    ap.kpool = p->k + (size_t)layer * p->layer_bytes;
    ap.vpool = p->v + (size_t)layer * p->layer_bytes;
    ap.num_slots = p->num_slots;
    ap.n = n;
    ap.Hkv = p->desc.num_kv_heads;
    ap.D = p->desc.head_dim;
    ap.err = p->d_err;
    return launch_append(ap, p->desc.dtype, false, (cudaStream_t)stream, false);
}

int s1kv_rope_append(s1kv_pool* p, int32_t layer, const float* q_in, float* q_out, int32_t Hq, const float* k,
                     const float* v, const int32_t* slots, const int32_t* pos, int64_t n, int64_t max_pos,
                     void* stream) {
    int st = check_pool(p);
    if (!st) st = check_layer(p, layer);
    if (st) return st;
    if (q_in && (!q_out || Hq <= 0)) return set_error(S1KV_EINVAL, "s1kv_rope_append: q needs q_out and n_q_heads");
    S1KV_ON_DEVICE(p->device);
    st = flush(p, (cudaStream_t)stream);
    if (st) return st;
    AppendParams ap{};
    ap.k = k;
    ap.v = v;
    ap.q_in = q_in;
    ap.q_out = q_out;
    ap.slots = slots;
    ap.pos = pos;
    ap.kpool = p->k + (size_t)layer * p->layer_bytes;
    ap.vpool = p->v + (size_t)layer * p->layer_bytes;
    ap.num_slots = p->num_slots;
    ap.n = n;
    ap.Hkv = p->desc.num_kv_heads;
    ap.Hq = Hq;
    ap.D = p->desc.head_dim;
    ap.err = p->d_err;
    // Without an explicit bound the positions are token indices of
    // sequences in this pool, so the longest sequence bounds them; the
    // kernel flags anything beyond the table.
    if (max_pos < 0) return set_error(S1KV_EINVAL, "s1kv_rope_append: negative max_pos");
    const int64_t bound = max_pos > 0 ? max_pos : std::max<int64_t>(p->max_len_seen, 1);
    ap.rope = rope_table(p->device, p->desc.head_dim, p->desc.rope_theta, bound, &ap.rope_cap, (cudaStream_t)stream,
                         &st);
    if (st) return st;
    return launch_append(ap, p->desc.dtype, true, (cudaStream_t)stream, false);
}

int s1kv_apply_rope(const float* x, float* out, int64_t start_pos, int64_t n, int32_t H, int32_t D, float theta,
                    void* stream) {
    if (n < 0 || H < 0 || D <= 0 || D % 2 || start_pos < 0 || (n > 0 && (!x || !out)))
        return set_error(S1KV_EINVAL, "s1kv_apply_rope: bad arguments");
    if (n == 0 || H == 0) return S1KV_OK;
    int dev = 0;
    S1KV_CUDA(cudaGetDevice(&dev));
    int st = S1KV_OK;
    int64_t cap = 0;
    const float2* tab = rope_table(dev, D, theta == 0.0f ? 1.0e6f : theta, start_pos + n, &cap, (cudaStream_t)stream, &st);
    if (st) return st;
    return launch_rope(x, out, tab, cap, start_pos, n, H, D, device_error_word(dev), (cudaStream_t)stream);
}

int s1kv_gather(s1kv_pool* p, int32_t layer, uint64_t seq, int32_t which, float* out, void* stream) {
    int st = check_pool(p);
    if (!st) st = check_layer(p, layer);
    if (st) return st;
    int32_t row;
    int64_t len;
    st = seq_row(p, seq, &row, &len);
    if (st) return st;
    S1KV_ON_DEVICE(p->device);
    st = flush(p, (cudaStream_t)stream);
    if (st) return st;
    return launch_gather(p, layer, row, len, which, out, (cudaStream_t)stream);
}

int s1kv_cow_copy(s1kv_pool* p, const int32_t* src, const int32_t* dst, int64_t n, void* stream) {
    int st = check_pool(p);
    if (st) return st;
    S1KV_ON_DEVICE(p->device);
    return launch_cow(p, src, dst, n, (cudaStream_t)stream);
}

int s1kv_attention(s1kv_pool* p, int32_t layer, const uint64_t* seqs, const int32_t* q_lens, int32_t n_seqs,
                   const float* q, float* out, int32_t Hq, void* stream) {
    int st = check_pool(p);
    if (!st) st = check_layer(p, layer);
    if (st) return st;
    if (!q_lens && n_seqs > 0) return set_error(S1KV_EINVAL, "s1kv_attention: q_lens required");
    for (int32_t i = 0; i < n_seqs; i++)
        if (!s1kv_seq_exists(p, seqs[i])) return set_error(S1KV_ENOSEQ, "Sequence ID not found");
    s1kv_batch* b = nullptr;
    st = s1kv_batch_begin(p, seqs, nullptr, q_lens, n_seqs, stream, &b);
    if (st) return st;
    st = s1kv_batch_attention(b, layer, q, out, Hq, stream);
    int st2 = s1kv_batch_end(b, stream);
    return st ? st : st2;
}

int s1kv_attention_contig(const float* q, const float* k, const float* v, int64_t q_len, int64_t kv_len, int32_t Hq,
                          int32_t Hkv, int32_t D, float* out, void* stream_) {
    if (q_len < 0 || kv_len < 0 || q_len > kv_len || Hkv <= 0 || Hq <= 0 || Hq % Hkv || D <= 0 || D > 256)
        return set_error(S1KV_EINVAL, "s1kv_attention_contig: bad shape");
    if (q_len == 0) return S1KV_OK;
    cudaStream_t stream = (cudaStream_t)stream_;
    int dev = 0;
    S1KV_CUDA(cudaGetDevice(&dev));
    std::vector<RowMeta> rows(q_len);
    for (int64_t i = 0; i < q_len; i++) rows[i] = {0, (int32_t)(kv_len - q_len + i + 1), 1, 0};
    RowMeta* d_rows = nullptr;
    S1KV_CUDA(cudaMallocAsync((void**)&d_rows, rows.size() * sizeof(RowMeta), stream));
    S1KV_CUDA(cudaMemcpyAsync(d_rows, rows.data(), rows.size() * sizeof(RowMeta), cudaMemcpyHostToDevice, stream));
    AttnParams ap{};
    ap.q = q;
    ap.out = out;
    ap.rows = d_rows;
    ap.kbase = k;
    ap.vbase = v;
    ap.num_slots = kv_len;
    ap.n_rows = (int32_t)q_len;
    ap.block_size = 1;
    ap.Hq = Hq;
    ap.Hkv = Hkv;
    ap.D = D;
    ap.scale_log2 = scale_log2(D);
    ap.err = device_error_word(dev);
    int st = launch_attention_generic(ap, S1KV_DTYPE_F32, stream);
    cudaError_t e = cudaFreeAsync(d_rows, stream);
    // The host copy must outlive the async upload.
    cudaError_t e2 = cudaStreamSynchronize(stream);
    if (st) return st;
    if (e != cudaSuccess) return cuda_error(e, "cudaFreeAsync");
    if (e2 != cudaSuccess) return cuda_error(e2, "cudaStreamSynchronize");
    return S1KV_OK;
}

}  // extern "C"

// ------------------------------------------------ storage read, disk prefix --

extern "C" {

int s1kv_pool_read(s1kv_pool* p, int32_t layer, int32_t which, int64_t slot0, int64_t n_slots, void* host_out) {
    int st = check_pool(p);
    if (!st) st = check_layer(p, layer);
    if (st) return st;
    if (slot0 < 0 || n_slots < 0 || slot0 + n_slots > p->num_slots || (n_slots && !host_out))
        return set_error(S1KV_EINVAL, "s1kv_pool_read: slot range out of bounds");
    S1KV_ON_DEVICE(p->device);
    S1KV_CUDA(cudaDeviceSynchronize());
    const size_t row = (size_t)p->desc.num_kv_heads * p->desc.head_dim * p->elem;
    const char* base = (which ? p->v : p->k) + (size_t)layer * p->layer_bytes + (size_t)slot0 * row;
    S1KV_CUDA(cudaMemcpy(host_out, base, (size_t)n_slots * row, cudaMemcpyDeviceToHost));
    return S1KV_OK;
}

int s1kv_prefix_save(s1kv_pool* p, uint64_t seq, const char* path) {
    int st = check_pool(p);
    if (st) return st;
    int32_t row;
    int64_t len;
    st = seq_row(p, seq, &row, &len);
    if (st) return st;
    FILE* f = std::fopen(path, "wb");
    if (!f) return set_error(S1KV_EINVAL, "s1kv_prefix_save: cannot open %s", path);
    const size_t n = (size_t)len * p->desc.num_kv_heads * p->desc.head_dim;
    std::vector<float> h(n);
    float* d = nullptr;
    cudaError_t e = cudaMalloc(&d, std::max<size_t>(n, 1) * sizeof(float));
    for (int32_t l = 0; l < p->desc.num_layers && e == cudaSuccess && st == S1KV_OK; l++) {
        for (int which = 0; which < 2 && st == S1KV_OK; which++) {
            st = s1kv_gather(p, l, seq, which, d, nullptr);
            if (st) break;
            e = cudaMemcpy(h.data(), d, n * sizeof(float), cudaMemcpyDeviceToHost);
            if (e != cudaSuccess) break;
            if (std::fwrite(h.data(), sizeof(float), n, f) != n) st = set_error(S1KV_EINVAL, "s1kv_prefix_save: short write");
        }
    }
    std::fclose(f);
    if (d) cudaFree(d);
    if (e != cudaSuccess) return cuda_error(e, "s1kv_prefix_save");
    return st;
}

int s1kv_prefix_load(s1kv_pool* p, uint64_t seq, int64_t n_tokens, const char* path) {
    int st = check_pool(p);
    if (st) return st;
    if (n_tokens < 0) return set_error(S1KV_EINVAL, "s1kv_prefix_load: negative length");
    FILE* f = std::fopen(path, "rb");
    if (!f) return set_error(S1KV_EINVAL, "s1kv_prefix_load: cannot open %s", path);
    const size_t n = (size_t)n_tokens * p->desc.num_kv_heads * p->desc.head_dim;
    std::vector<float> h(n * 2 * p->desc.num_layers);
    const size_t got = h.empty() ? 0 : std::fread(h.data(), sizeof(float), h.size(), f);
    std::fclose(f);
    if (got != h.size()) return set_error(S1KV_EINVAL, "s1kv_prefix_load: %s is shorter than %lld tokens", path, (long long)n_tokens);
    s1kv_batch* b = nullptr;
    const int32_t na = (int32_t)n_tokens, ql = 0;
    st = s1kv_batch_begin(p, &seq, &na, &ql, 1, nullptr, &b);
    if (st) return st;
    float* d = nullptr;
    cudaError_t e = cudaMalloc(&d, std::max<size_t>(2 * n, 1) * sizeof(float));
    for (int32_t l = 0; l < p->desc.num_layers && e == cudaSuccess && st == S1KV_OK; l++) {
        e = cudaMemcpy(d, h.data() + 2 * n * l, 2 * n * sizeof(float), cudaMemcpyHostToDevice);
        if (e == cudaSuccess) st = s1kv_batch_append(b, l, d, d + n, nullptr);
        if (e == cudaSuccess && st == S1KV_OK) e = cudaDeviceSynchronize();
    }
    int st2 = s1kv_batch_end(b, nullptr);
    if (d) cudaFree(d);
    if (e != cudaSuccess) return cuda_error(e, "s1kv_prefix_load");
    return st ? st : st2;
}

}  // extern "C"
