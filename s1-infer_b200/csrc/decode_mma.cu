// decode_mma.cu -- paged split-K GQA decode over bf16 K/V on the tensor
// cores (warp-level mma.sync m16n8k16, bf16 x bf16 -> fp32).
//
// GQA_attention_paged (src/nn/attention.cpp:128-239 of s1-infer) for decode
// rows (one query token per sequence) of a bf16 pool with head_dim 128.
// Same work decomposition and partial-result format as the CUDA-core decode
// kernel (attention.cu): a CTA takes one split-K item (row, token range) of
// one KV head; its 4 warps take the range's 16-token tiles (one block each)
// round-robin, each through its own TMA ring; the warps merge through shared
// memory and write the final row (single split) or a partial (max, sum, O)
// that combine_kernel merges.
//
// Why tensor cores for an HBM-bound kernel: with 8 query heads per KV head
// every K/V element feeds 8 multiply-adds plus a bf16 widening, which makes
// the CUDA-core kernel issue-bound well below the HBM roofline.  Here one
// 16-token tile costs 16 ldmatrix, 4 movmatrix and 32 mma per warp.
//   * Token-major products, so the 8 heads (or fewer) of a group fill the
//     N = 8 side of m16n8k16 and no M rows are padding:
//     S^T[token, head] = K Q^T with M = 16 tokens, K = 16 dims; a K (or V)
//     tile arrives by one TMA copy in the 128-byte-swizzled layout (the two
//     64-element halves of the rows one after the other), so ldmatrix reads
//     it without bank conflicts.
//   * The score fragment of a thread (tokens g, g+8; heads 2t, 2t+1) turns
//     into P's B fragment of O^T += V^T P^T (head g; tokens 2t, 2t+1,
//     2t+8, 2t+9) by one movmatrix transpose per 8x8 half, so P never
//     leaves registers; V^T fragments come from ldmatrix.trans.
//   * Precision: q (fp32, pre-scaled by log2(e)/sqrt(D)) and p are each
//     split into bf16 hi + lo parts and both parts are multiplied (K and V
//     are exact in bf16), so scores and outputs carry fp32-level error
//     (about 2^-17 relative), not bf16 error.
//   * Online softmax in the exp2 domain per head (a column held by 8
//     lanes); the reference max moves only when a tile's max outgrows it
//     by 2^8, and only then is the max reduced and that head's O rescaled.
// Waits are bounded (device error word on timeout, copies drained).
#include <cuda.h>
#include <cuda_bf16.h>

#include <cmath>

#include "combine.cuh"
#include "internal.h"

namespace s1kv {
namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr uint32_t kSpin = 1u << 22;
constexpr int kD = 128;
constexpr int kTile = 16;                      // tokens per stage (one block)
constexpr int kNW = 4;                         // warps per CTA
constexpr int kNS = 2;                         // stages per warp
constexpr int kMinCtas = 3;
constexpr int kBoxBytes = kTile * 128;         // 16 tokens x 64 bf16, 128B-swizzled
constexpr int kTileBytes = 2 * kBoxBytes;      // K (or V) of one tile: 4 KB
constexpr int kStageBytes = 2 * kTileBytes;    // K + V
constexpr int kRing = kNW * kNS * kStageBytes;
constexpr int kSmem = kRing + kNW * kNS * 8 + 16 + 1024;  // + barriers + last-CTA flag + slack for 1024 alignment
constexpr float kRescaleAt = 8.0f;             // log2 units

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void bar_init(uint64_t* b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void bar_expect(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t phase) {
    for (uint32_t i = 0; i < kSpin; i++) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(su32(b)), "r"(phase)
            : "memory");
        if (ok) return true;
    }
    return false;
}
__device__ __forceinline__ void tma5(void* dst, const CUtensorMap* m, uint64_t* b, int c0, int c1, int c2, int c3,
                                     int c4) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, %6}], "
        "[%7];" ::"r"(su32(dst)),
        "l"(m), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(su32(b))
        : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// c += A B for one m16n8k16 tile (bf16 x bf16 -> fp32).
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Transpose of an 8x8 b16 matrix held as the warp's m8n8 fragment (lane L:
// row L / 4, columns 2(L % 4), 2(L % 4) + 1).
__device__ __forceinline__ uint32_t movt(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// (a, b) -> bf16 pair (a in the low half) and the bf16 pair of the residuals.
__device__ __forceinline__ void split_bf16(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

// Shared-memory address of 16-byte chunk `chunk` (0..15 over 128 dims) of
// row `row` of a tile held as two 128B-swizzled 64-element halves.
__device__ __forceinline__ uint32_t tile_chunk(uint32_t base, int row, int chunk) {
    return base + (chunk >> 3) * kBoxBytes + row * 128 + (((chunk & 7) ^ (row & 7)) << 4);
}

}  // namespace

template <int G>
__global__ void __launch_bounds__(kNW * 32, kMinCtas)
    decode_mma_kernel(const __grid_constant__ AttnParams p, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV) {
    static_assert(G >= 1 && G <= 8, "query heads per KV head must fit the 8 live rows of an m16 tile");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, tq = lane & 3;  // mma fragment coordinates: head row, column pair
    // grid (items, heads): the CTAs of one head's items run side by side (the
    // heads-fastest order of the fp32 kernel measured 3% slower here)
    const int h = blockIdx.y;
    const WorkItem item = p.items[blockIdx.x];
    const int tok0 = item.split * p.split_tokens;
    const int tok1 = min(tok0 + p.split_tokens, item.kv_len);
    const int n_tiles = (tok1 - tok0 + kTile - 1) / kTile;
    const int my_tiles = n_tiles > warp ? (n_tiles - warp + kNW - 1) / kNW : 0;
    const int32_t* tab = p.table + (int64_t)item.table_row * p.max_bps;
    uint8_t* ring = smem + warp * kNS * kStageBytes;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kRing) + warp * kNS;

    // Storage row of this warp's k-th tile; lane k prefetches it for k < 32.
    auto tile_row = [&](int k, int& row) -> bool {
        const int base = tok0 + (warp + k * kNW) * kTile;
        const int32_t blk = tab[base >> 4];
        if ((uint32_t)blk >= (uint32_t)p.max_blocks) {
            row = p.max_blocks * 16;  // out of range: TMA zero-fills the box
            return false;
        }
        row = blk * 16;
        return true;
    };
    int my_row = 0;
    if (lane < my_tiles && !tile_row(lane, my_row)) atomicOr(p.err, kErrBounds);
    if (lane == 0) {
        for (int s = 0; s < kNS; s++) bar_init(&bar[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    auto issue = [&](int k, int row) {
        const int s = k % kNS;
        uint8_t* dst = ring + s * kStageBytes;
        bar_expect(&bar[s], kStageBytes);
        tma5(dst, &tmK, &bar[s], 0, row, 0, h, p.layer);  // both halves of the block's 16 rows
        tma5(dst + kTileBytes, &tmV, &bar[s], 0, row, 0, h, p.layer);
    };
    // The first copies: tiles entirely below the tokens this batch appends
    // are requested before the wait (items, block table and those K/V rows
    // were written before the previous kernel started), the rest after it.
    const int n_first = min(kNS, my_tiles);
    int pre = 0;
    if (p.prewait) {
        const int safe_end = item.kv_len - p.prewait_margin;
        while (pre < n_first && tok0 + (warp + pre * kNW) * kTile + kTile <= safe_end) pre++;
    }
    for (int k = 0; k < pre; k++) {
        const int row = __shfl_sync(kFull, my_row, k);
        if (lane == 0) issue(k, row);
    }
    pdl_wait();
    for (int k = pre; k < n_first; k++) {
        const int row = __shfl_sync(kFull, my_row, k);
        if (lane == 0) issue(k, row);
    }
    const RowMeta rm = p.rows[item.row];  // split count and partial offset, needed at the end

    // B fragments of q^T (pre-scaled, split hi + lo): k-step ks covers dims
    // 16ks .. 16ks+15; this lane holds dims 2tq, 2tq+1 (b0) and 2tq+8, 2tq+9
    // (b1) of head gq (zero for the padding heads gq >= G).
    uint32_t qh[kD / 16][2], ql[kD / 16][2];
    {
        const float* qrow = p.q + ((int64_t)item.row * p.Hq + h * G + (gq < G ? gq : 0)) * kD;
#pragma unroll
        for (int ks = 0; ks < kD / 16; ks++)
#pragma unroll
            for (int half = 0; half < 2; half++) {
                float2 v = make_float2(0.f, 0.f);
                if (gq < G) v = __ldg(reinterpret_cast<const float2*>(qrow + ks * 16 + half * 8 + 2 * tq));
                split_bf16(v.x * p.scale_log2, v.y * p.scale_log2, qh[ks][half], ql[ks][half]);
            }
    }

    // O^T accumulators: m-block mb covers dims 16mb .. 16mb+15; [mb][0] and
    // [mb][1] are dim 16mb + gq of heads 2tq and 2tq+1, [2] and [3] dim
    // 16mb + gq + 8 of the same heads.
    float o[kD / 16][4];
#pragma unroll
    for (int mb = 0; mb < kD / 16; mb++) o[mb][0] = o[mb][1] = o[mb][2] = o[mb][3] = 0.0f;
    // heads 2tq, 2tq+1: reference max (log2 units, the same in the 8 lanes of
    // a head) and this lane's share of the sum (tokens gq, gq+8 of each tile)
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;

    // ldmatrix row addresses: lane L supplies row (L & 7) of matrix L >> 3.
    const int mi = lane >> 3, r8 = lane & 7;
    bool failed = false;
    int consumed = 0;
    for (int k = 0; k < my_tiles; k++) {
        const int s = k % kNS;
        if (!bar_wait(&bar[s], (uint32_t)((k / kNS) & 1))) {
            failed = true;
            break;
        }
        consumed = k + 1;
        const uint32_t Kt = su32(ring + s * kStageBytes), Vt = Kt + kTileBytes;
        const int base = tok0 + (warp + k * kNW) * kTile;
        const int valid = min(kTile, tok1 - base);

        // ---- S^T = K Q^T: M = the 16 tokens, N = the 8 head columns ----
        // four accumulators (hi / lo part of q, even / odd k-step) keep the
        // dependent chains four mma long
        float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
        float sc[4] = {0.f, 0.f, 0.f, 0.f}, sd[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ks = 0; ks < kD / 16; ks += 2) {
            uint32_t a[4], a2[4];  // matrix mi: tokens 8(mi & 1) + r8, dims 16ks + 8(mi >> 1) ..
            ldsm_x4(tile_chunk(Kt, (mi & 1) * 8 + r8, ks * 2 + (mi >> 1)), a);
            ldsm_x4(tile_chunk(Kt, (mi & 1) * 8 + r8, (ks + 1) * 2 + (mi >> 1)), a2);
            mma16816(sa, a, qh[ks][0], qh[ks][1]);
            mma16816(sb, a, ql[ks][0], ql[ks][1]);
            mma16816(sc, a2, qh[ks + 1][0], qh[ks + 1][1]);
            mma16816(sd, a2, ql[ks + 1][0], ql[ks + 1][1]);
        }
        // this lane: [0] token gq head 2tq, [1] token gq head 2tq+1,
        // [2] token gq+8 head 2tq, [3] token gq+8 head 2tq+1
        float x[4];
#pragma unroll
        for (int i = 0; i < 4; i++) x[i] = (sa[i] + sc[i]) + (sb[i] + sd[i]);
        if (valid < kTile) {
            if (gq >= valid) x[0] = x[1] = -INFINITY;
            if (gq + 8 >= valid) x[2] = x[3] = -INFINITY;
        }
        // the reference max of a head moves only when one of its scores
        // outgrows it by 2^8; the head's max over the tile is reduced (over
        // the 8 lanes of a column) only on such a tile
        float mx0 = fmaxf(x[0], x[2]), mx1 = fmaxf(x[1], x[3]);
        if (__any_sync(kFull, mx0 > m0 + kRescaleAt || mx1 > m1 + kRescaleAt)) {
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                mx0 = fmaxf(mx0, __shfl_xor_sync(kFull, mx0, off));
                mx1 = fmaxf(mx1, __shfl_xor_sync(kFull, mx1, off));
            }
            const bool r0 = mx0 > m0 + kRescaleAt, r1 = mx1 > m1 + kRescaleAt;
            const float c0 = r0 ? ex2(m0 - mx0) : 1.0f, c1 = r1 ? ex2(m1 - mx1) : 1.0f;  // 0 from m = -inf
            if (r0) {
                m0 = mx0;
                l0 *= c0;
            }
            if (r1) {
                m1 = mx1;
                l1 *= c1;
            }
#pragma unroll
            for (int mb = 0; mb < kD / 16; mb++) {
                o[mb][0] *= c0;
                o[mb][1] *= c1;
                o[mb][2] *= c0;
                o[mb][3] *= c1;
            }
        }
        const float p0 = ex2(x[0] - m0), p1 = ex2(x[1] - m1), p2 = ex2(x[2] - m0), p3 = ex2(x[3] - m1);
        l0 += p0 + p2;
        l1 += p1 + p3;
        // P^T fragments (token rows, head columns) in bf16 hi + lo, then
        // transposed in registers into the B fragments of O^T += V^T P^T:
        // head gq, tokens 2tq, 2tq+1 (b0) and 2tq+8, 2tq+9 (b1)
        uint32_t h0, l0p, h1, l1p;
        split_bf16(p0, p1, h0, l0p);
        split_bf16(p2, p3, h1, l1p);
        const uint32_t bh0 = movt(h0), bh1 = movt(h1), bl0 = movt(l0p), bl1 = movt(l1p);

        // ---- O^T += V^T P^T: M = 16 dims per m-block, K = the 16 tokens ----
#pragma unroll
        for (int mb = 0; mb < kD / 16; mb++) {
            uint32_t a[4];  // matrix mi: tokens 8(mi >> 1) + r8, dims 16mb + 8(mi & 1) .., transposed
            ldsm_x4_t(tile_chunk(Vt, (mi >> 1) * 8 + r8, mb * 2 + (mi & 1)), a);
            mma16816(o[mb], a, bh0, bh1);
            mma16816(o[mb], a, bl0, bl1);
        }
        __syncwarp();
        if (k + kNS < my_tiles) {
            int row = __shfl_sync(kFull, my_row, (k + kNS) & 31);
            if (k + kNS >= 32) {
                // past the 32 prefetched block ids: look the block up directly
                if (!tile_row(k + kNS, row) && lane == 0) atomicOr(p.err, kErrBounds);
            }
            if (lane == 0) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                issue(k + kNS, row);
            }
        }
    }

    // The next kernel of the stream may launch once every CTA got here: its
    // CTAs then take the slots this launch frees as it ends (and overlap the
    // merge of the splits) instead of slots beside CTAs still streaming K/V,
    // which skews the next launch's CTAs over the SMs.  This kernel waits
    // for the previous one (griddepcontrol.wait) before reading what it
    // writes.
    pdl_trigger();
    if (failed) {
        // drain this warp's copies still in flight before the CTA exits
        if (lane == 0) atomicOr(p.err, kErrTimeout);
        const int issued = min(my_tiles, consumed + kNS);
        for (int k = consumed + 1; k < issued; k++) bar_wait(&bar[k % kNS], (uint32_t)((k / kNS) & 1));
        m0 = m1 = -INFINITY;
        l0 = l1 = 0.0f;
#pragma unroll
        for (int mb = 0; mb < kD / 16; mb++) o[mb][0] = o[mb][1] = o[mb][2] = o[mb][3] = 0.0f;
    }
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
        l0 += __shfl_xor_sync(kFull, l0, off);
        l1 += __shfl_xor_sync(kFull, l1, off);
    }

    // ---- merge the warps through shared memory (aliases the rings) ----
    __syncthreads();
    float* mo = reinterpret_cast<float*>(smem);  // [kNW][G][kD]
    float* mml = mo + kNW * G * kD;              // [kNW][G][2]
    if (2 * tq < G) {
        float* dst = &mo[(warp * G + 2 * tq) * kD + gq];
#pragma unroll
        for (int mb = 0; mb < kD / 16; mb++) {
            dst[16 * mb] = o[mb][0];
            dst[16 * mb + 8] = o[mb][2];
        }
        if (gq == 0) {
            mml[(warp * G + 2 * tq) * 2] = m0;
            mml[(warp * G + 2 * tq) * 2 + 1] = l0;
        }
    }
    if (2 * tq + 1 < G) {
        float* dst = &mo[(warp * G + 2 * tq + 1) * kD + gq];
#pragma unroll
        for (int mb = 0; mb < kD / 16; mb++) {
            dst[16 * mb] = o[mb][1];
            dst[16 * mb + 8] = o[mb][3];
        }
        if (gq == 0) {
            mml[(warp * G + 2 * tq + 1) * 2] = m1;
            mml[(warp * G + 2 * tq + 1) * 2 + 1] = l1;
        }
    }
    __syncthreads();
    const int64_t part = (int64_t)(rm.part_off + item.split) * p.Hkv + h;
    for (int idx = threadIdx.x; idx < G * kD; idx += kNW * 32) {
        const int g = idx / kD, d = idx % kD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kNW; w++) M = fmaxf(M, mml[(w * G + g) * 2]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < kNW; w++) {
            const float mw = mml[(w * G + g) * 2];
            const float f = (mw == -INFINITY) ? 0.0f : ex2(mw - M);
            L = fmaf(mml[(w * G + g) * 2 + 1], f, L);
            O = fmaf(mo[(w * G + g) * kD + d], f, O);
        }
        if (rm.n_split == 1) {
            store_out(p, item.row, h * G + g, d, kD, O / L);
        } else {
            p.part_o[(part * G + g) * kD + d] = O;
            if (d == 0) {
                p.part_ml[(part * G + g) * 2] = M;
                p.part_ml[(part * G + g) * 2 + 1] = L;
            }
        }
    }
    if (p.counters && rm.n_split > 1)
        finish_split_row(p, item.row, h, item.split, rm.n_split, G, kD, reinterpret_cast<int*>(smem + kRing + kNW * kNS * 8),
                         reinterpret_cast<float*>(smem), kRing / 4);  // the rings are free by now
}

bool decode_mma_supported(int dtype, int D, int G, int block_size) {
    return dtype == S1KV_DTYPE_BF16 && D == kD && block_size == 16 && G >= 1 && G <= 8 &&
           (G == 1 || G == 2 || G == 4 || G == 7 || G == 8);
}

template <int G>
static int launch_mma_g(const AttnParams& p, const CUtensorMap& tk, const CUtensorMap& tv, cudaStream_t stream) {
    static std::atomic<uint64_t> attr_set{0};  // per device
    int st = once_per_device(attr_set, [] {
        S1KV_CUDA(cudaFuncSetAttribute(decode_mma_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
        return S1KV_OK;
    });
    if (st) return st;
    dim3 grid((unsigned)p.n_items, (unsigned)p.Hkv);
    S1KV_CUDA(launch_pdl(decode_mma_kernel<G>, grid, dim3(kNW * 32), kSmem, stream, p, tk, tv));
    g_launches++;
    S1KV_CUDA(cudaGetLastError());
    return S1KV_OK;
}

int launch_decode_mma(const AttnParams& p, const CUtensorMap& tk_sw, const CUtensorMap& tv_sw, cudaStream_t stream) {
    switch (p.Hq / p.Hkv) {
        case 1: return launch_mma_g<1>(p, tk_sw, tv_sw, stream);
        case 2: return launch_mma_g<2>(p, tk_sw, tv_sw, stream);
        case 4: return launch_mma_g<4>(p, tk_sw, tv_sw, stream);
        case 7: return launch_mma_g<7>(p, tk_sw, tv_sw, stream);
        case 8: return launch_mma_g<8>(p, tk_sw, tv_sw, stream);
        default: return set_error(S1KV_EINVAL, "decode: unsupported group size %d", p.Hq / p.Hkv);
    }
}

}  // namespace s1kv
