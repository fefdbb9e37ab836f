// attention.cu -- paged GQA attention for sm_100a.
//
// Computes GQA_attention_paged of s1-infer (src/nn/attention.cpp:128-239):
// for q head h, kv head h / (Hq/Hkv) (:155); scores q.k / sqrt(D) over the
// causal range j <= (kv_len - q_len) + i (:181, :190); softmax (:194-218);
// PV (:220-235).  Here every query row carries its own causal length, so a
// decode row (q_len 1) attends to all kv_len tokens and row i of a prefill
// chunk to (kv_len - q_len) + i + 1 tokens.
//
// Fast path (block_size 16, head_dim 64/128, group size 1/2/4/7/8): a
// split-K ("flash-decoding") kernel that is bound by HBM bandwidth.
//   * grid = (work item, kv head); a work item is one query row and one
//     split of split_tokens tokens (a multiple of 16).
//   * one CTA keeps all G query heads of its KV group, so every K/V byte
//     is read from HBM exactly once per row.
//   * each warp is an independent worker over tiles warp, warp+NW, ... of
//     the split.  A tile is one 16-token block; its K rows and V rows for
//     the kv head are two TMA boxes (16 rows x head_dim) landing in the
//     warp's ring of NS shared-memory stages, completion tracked by one
//     mbarrier per stage (bounded waits; a timeout sets the device error
//     word).  No TMA multicast anywhere.
//   * QK: LPT lanes share one token; lane part p reads 16-byte chunks
//     p, p+LPT, ... of the row, so each quarter-warp phase hits 8 distinct
//     bank groups.  q stays in registers (G x D/LPT floats).  Partial dots
//     are combined with log2(LPT) xor-shuffles.
//   * online softmax per tile in the exp2 domain; PV with lanes over head
//     dims (D/32 each) and p broadcast by shuffle.
//   * warps merge through shared memory; multi-split rows write partial
//     (max, sum, o) and a combine kernel finishes them.
// Generic path: one warp per query head, one token at a time; used for the
// reference's tiny test shapes (head_dim 1-2, block_size 2-4) and for
// contiguous K/V (GQA_attention).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <cfloat>
#include <cmath>

#include "internal.h"

namespace s1kv {

constexpr uint32_t kSpinLimit = 1u << 22;
constexpr unsigned kFull = 0xffffffffu;

// ------------------------------------------------------------ PTX helpers --
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase; false after kSpinLimit polls.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t phase) {
    for (uint32_t i = 0; i < kSpinLimit; i++)
        if (mbar_try_wait(bar, phase)) return true;
    return false;
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// 16 bytes of storage -> EPC floats.
template <typename T>
__device__ __forceinline__ void load_chunk(const T* src, float* x);

template <>
__device__ __forceinline__ void load_chunk<float>(const float* src, float* x) {
    float4 a = *reinterpret_cast<const float4*>(src);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
}

template <>
__device__ __forceinline__ void load_chunk<uint16_t>(const uint16_t* src, float* x) {
    uint4 a = *reinterpret_cast<const uint4*>(src);
    x[0] = bf16lo(a.x); x[1] = bf16hi(a.x); x[2] = bf16lo(a.y); x[3] = bf16hi(a.y);
    x[4] = bf16lo(a.z); x[5] = bf16hi(a.z); x[6] = bf16lo(a.w); x[7] = bf16hi(a.w);
}

// N consecutive storage elements (N = D/32: 2 or 4) -> floats.
template <typename T, int N>
__device__ __forceinline__ void load_vec(const T* src, float* x) {
    if constexpr (sizeof(T) == 4) {
        if constexpr (N == 4) {
            float4 a = *reinterpret_cast<const float4*>(src);
            x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        } else {
            float2 a = *reinterpret_cast<const float2*>(src);
            x[0] = a.x; x[1] = a.y;
        }
    } else {
        if constexpr (N == 4) {
            uint2 a = *reinterpret_cast<const uint2*>(src);
            x[0] = bf16lo(a.x); x[1] = bf16hi(a.x); x[2] = bf16lo(a.y); x[3] = bf16hi(a.y);
        } else {
            uint32_t a = *reinterpret_cast<const uint32_t*>(src);
            x[0] = bf16lo(a); x[1] = bf16hi(a);
        }
    }
}

template <typename T>
__device__ __forceinline__ float load_elem(const T* src) {
    if constexpr (sizeof(T) == 4) return *reinterpret_cast<const float*>(src);
    else return __uint_as_float((uint32_t)(*reinterpret_cast<const uint16_t*>(src)) << 16);
}

// ------------------------------------------------------- configuration ---
template <typename T, int D, int G>
struct DecodeCfg {
    static constexpr int kBS = 16;                                  // tokens per tile (= block_size)
    static constexpr int kEPC = 16 / (int)sizeof(T);                // elements per 16-byte chunk
    static constexpr int kNCH = D / kEPC;                           // chunks per row
    static constexpr int kLPT = (G * D / 8 > 64 && kNCH >= 16) ? 16 : 8;  // lanes per token (QK)
    static constexpr int kIT = kNCH / kLPT;                         // chunks per lane per row
    static constexpr int kDQ = D / kLPT;                            // q dims per lane
    static constexpr int kTPS = 32 / kLPT;                          // tokens per QK step
    static constexpr int kSTEPS = kBS / kTPS;                       // QK steps per tile
    static constexpr int kDPL = D / 32;                             // PV dims per lane
    static constexpr int kTileBytes = kBS * D * (int)sizeof(T);     // one K (or V) tile
    static constexpr int kStageBytes = 2 * kTileBytes;
    static constexpr int kNW = (sizeof(T) == 4 && D == 128) ? 4 : 8;  // warps per CTA
    static constexpr int kNS = (kStageBytes <= 4096) ? 4 : 3;         // stages per warp
    static constexpr int kSmem = kNW * kNS * kStageBytes + kNW * kNS * 8;
    static_assert(kNCH % kLPT == 0, "chunks must split evenly over lanes");
    static_assert(kLPT >= 8, "a quarter-warp phase must read 8 distinct chunks");
    static_assert(kNW * kNS * kStageBytes >= kNW * G * (D + 2) * 4, "merge area must fit in the stage ring");
};

// ------------------------------------------------------------- decode ----
template <typename T, int D, int G>
__global__ void __launch_bounds__(DecodeCfg<T, D, G>::kNW * 32, 1)
    decode_tma_kernel(const __grid_constant__ AttnParams p, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV) {
    using C = DecodeCfg<T, D, G>;
    constexpr int NW = C::kNW, NS = C::kNS, LPT = C::kLPT, IT = C::kIT, EPC = C::kEPC, TPS = C::kTPS,
                  STEPS = C::kSTEPS, DPL = C::kDPL, DQ = C::kDQ;
    extern __shared__ __align__(1024) uint8_t smem[];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.y;
    const WorkItem item = p.items[blockIdx.x];
    const RowMeta rm = p.rows[item.row];
    const int tok0 = item.split * p.split_tokens;
    const int tok1 = min(tok0 + p.split_tokens, rm.kv_len);
    const int n_tiles = (tok1 - tok0 + 15) >> 4;
    const int my_tiles = n_tiles > warp ? (n_tiles - warp + NW - 1) / NW : 0;
    const int32_t* tab = p.table + (int64_t)rm.table_row * p.max_bps + (tok0 >> 4);

    uint8_t* ring = smem + warp * NS * C::kStageBytes;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + NW * NS * C::kStageBytes) + warp * NS;

    // Block ids of this warp's first 32 tiles, one per lane.
    int32_t my_blk = 0;
    if (lane < my_tiles) my_blk = tab[warp + lane * NW];
    if (lane < my_tiles && (uint32_t)my_blk >= (uint32_t)p.max_blocks) {
        atomicOr(p.err, kErrBounds);
        my_blk = p.max_blocks;  // TMA zero-fills boxes that start out of range
    }
    if (lane == 0) {
        for (int s = 0; s < NS; s++) mbar_init(&bar[s], 1);
        fence_barrier_init();
    }
    __syncwarp();

    auto issue = [&](int k, int32_t blk) {
        const int s = k % NS;
        uint8_t* dst = ring + s * C::kStageBytes;
        mbar_expect_tx(&bar[s], C::kStageBytes);
        tma_load_4d(dst, &tmK, &bar[s], 0, h, blk * 16, p.layer);
        tma_load_4d(dst + C::kTileBytes, &tmV, &bar[s], 0, h, blk * 16, p.layer);
    };
    {
        const int pre = min(NS, my_tiles);
        for (int k = 0; k < pre; k++) {
            int32_t blk = __shfl_sync(kFull, my_blk, k);
            if (lane == 0) issue(k, blk);
        }
    }

    // q for the G heads of this group: lane part `pp` holds chunks pp,
    // pp+LPT, ... of every head.
    const int pp = lane % LPT;
    const int tl = lane / LPT;
    float qr[G][DQ];
#pragma unroll
    for (int g = 0; g < G; g++) {
        const float* qrow = p.q + ((int64_t)item.row * p.Hq + h * G + g) * D;
#pragma unroll
        for (int it = 0; it < IT; it++) {
            const float4* src = reinterpret_cast<const float4*>(qrow + (it * LPT + pp) * EPC);
#pragma unroll
            for (int e4 = 0; e4 < EPC / 4; e4++) {
                float4 v = __ldg(src + e4);
                qr[g][it * EPC + e4 * 4 + 0] = v.x;
                qr[g][it * EPC + e4 * 4 + 1] = v.y;
                qr[g][it * EPC + e4 * 4 + 2] = v.z;
                qr[g][it * EPC + e4 * 4 + 3] = v.w;
            }
        }
    }

    float m[G], l[G], o[G][DPL];
#pragma unroll
    for (int g = 0; g < G; g++) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int d = 0; d < DPL; d++) o[g][d] = 0.0f;
    }

    bool failed = false;
    int consumed = 0;
    for (int k = 0; k < my_tiles; k++) {
        const int s = k % NS;
        if (!mbar_wait_bounded(&bar[s], (uint32_t)((k / NS) & 1))) {
            failed = true;
            break;
        }
        consumed = k + 1;
        const T* Ks = reinterpret_cast<const T*>(ring + s * C::kStageBytes);
        const T* Vs = Ks + 16 * D;
        const int base = tok0 + (warp + k * NW) * 16;
        const int valid = min(16, tok1 - base);

        // ---- scores for the tile ----
        float sc[STEPS][G];
#pragma unroll
        for (int j = 0; j < STEPS; j++) {
            const int t = j * TPS + tl;
            const T* krow = Ks + t * D;
            float acc[G];
#pragma unroll
            for (int g = 0; g < G; g++) acc[g] = 0.0f;
#pragma unroll
            for (int it = 0; it < IT; it++) {
                float kf[EPC];
                load_chunk<T>(krow + (it * LPT + pp) * EPC, kf);
#pragma unroll
                for (int g = 0; g < G; g++)
#pragma unroll
                    for (int e = 0; e < EPC; e++) acc[g] = fmaf(qr[g][it * EPC + e], kf[e], acc[g]);
            }
#pragma unroll
            for (int off = LPT / 2; off >= 1; off >>= 1)
#pragma unroll
                for (int g = 0; g < G; g++) acc[g] += __shfl_xor_sync(kFull, acc[g], off);
#pragma unroll
            for (int g = 0; g < G; g++) sc[j][g] = (t < valid) ? acc[g] * p.scale_log2 : -INFINITY;
        }

        // ---- online softmax update ----
        float corr[G];
#pragma unroll
        for (int g = 0; g < G; g++) {
            float mx = sc[0][g];
#pragma unroll
            for (int j = 1; j < STEPS; j++) mx = fmaxf(mx, sc[j][g]);
#pragma unroll
            for (int off = LPT; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, off));
            const float mn = fmaxf(m[g], mx);
            corr[g] = exp2f(m[g] - mn);
            m[g] = mn;
            float ls = 0.0f;
#pragma unroll
            for (int j = 0; j < STEPS; j++) {
                sc[j][g] = exp2f(sc[j][g] - mn);
                ls += sc[j][g];
            }
            l[g] = fmaf(l[g], corr[g], ls);
#pragma unroll
            for (int d = 0; d < DPL; d++) o[g][d] *= corr[g];
        }

        // ---- PV ----
#pragma unroll
        for (int u = 0; u < 16; u++) {
            if (u < valid) {
                float vf[DPL];
                load_vec<T, DPL>(Vs + u * D + lane * DPL, vf);
#pragma unroll
                for (int g = 0; g < G; g++) {
                    const float pv = __shfl_sync(kFull, sc[u / TPS][g], (u % TPS) * LPT);
#pragma unroll
                    for (int d = 0; d < DPL; d++) o[g][d] = fmaf(pv, vf[d], o[g][d]);
                }
            }
        }
        __syncwarp();
        if (k + NS < my_tiles) {
            int32_t blk = __shfl_sync(kFull, my_blk, (k + NS) & 31);
            if (k + NS >= 32) {
                // Tiles past the 32 prefetched ids (splits longer than
                // 32 * NW tiles): read the id directly.
                blk = tab[warp + (k + NS) * NW];
                if ((uint32_t)blk >= (uint32_t)p.max_blocks) {
                    if (lane == 0) atomicOr(p.err, kErrBounds);
                    blk = p.max_blocks;
                }
            }
            if (lane == 0) {
                fence_proxy_async();
                issue(k + NS, blk);
            }
        }
    }

    if (failed) {
        // Drain this warp's copies still in flight before the CTA exits.
        if (lane == 0) atomicOr(p.err, kErrTimeout);
        const int issued = min(my_tiles, consumed + NS);
        for (int k = consumed + 1; k < issued; k++) mbar_wait_bounded(&bar[k % NS], (uint32_t)((k / NS) & 1));
#pragma unroll
        for (int g = 0; g < G; g++) {
            m[g] = -INFINITY;
            l[g] = 0.0f;
#pragma unroll
            for (int d = 0; d < DPL; d++) o[g][d] = 0.0f;
        }
    }

    // Per-warp totals: l summed over token lanes (part lanes hold copies).
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int off = LPT; off < 32; off <<= 1) l[g] += __shfl_xor_sync(kFull, l[g], off);

    // ---- merge the NW warps through shared memory (aliases the rings) ----
    __syncthreads();
    float* mo = reinterpret_cast<float*>(smem);            // [NW][G][D]
    float* mml = mo + NW * G * D;                           // [NW][G][2]
#pragma unroll
    for (int g = 0; g < G; g++) {
#pragma unroll
        for (int d = 0; d < DPL; d++) mo[(warp * G + g) * D + lane * DPL + d] = o[g][d];
        if (lane == 0) {
            mml[(warp * G + g) * 2] = m[g];
            mml[(warp * G + g) * 2 + 1] = l[g];
        }
    }
    __syncthreads();
    const int64_t part = (int64_t)(rm.part_off + item.split) * p.Hkv + h;
    for (int idx = threadIdx.x; idx < G * D; idx += NW * 32) {
        const int g = idx / D, d = idx % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; w++) M = fmaxf(M, mml[(w * G + g) * 2]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; w++) {
            const float mw = mml[(w * G + g) * 2];
            const float f = (mw == -INFINITY) ? 0.0f : exp2f(mw - M);
            L = fmaf(mml[(w * G + g) * 2 + 1], f, L);
            O = fmaf(mo[(w * G + g) * D + d], f, O);
        }
        if (rm.n_split == 1) {
            p.out[((int64_t)item.row * p.Hq + h * G + g) * D + d] = O / L;
        } else {
            p.part_o[(part * G + g) * D + d] = O;
            if (d == 0) {
                p.part_ml[(part * G + g) * 2] = M;
                p.part_ml[(part * G + g) * 2 + 1] = L;
            }
        }
    }
}

// Combines the split partials of multi-split rows: rescale to the global
// max, sum, normalise.
__global__ void combine_kernel(const AttnParams p, int G) {
    const RowMeta rm = p.rows[blockIdx.x];
    if (rm.n_split <= 1) return;
    const int h = blockIdx.y, D = p.D;
    for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
        const int g = idx / D, d = idx % D;
        float M = -INFINITY;
        for (int s = 0; s < rm.n_split; s++) {
            const int64_t part = (int64_t)(rm.part_off + s) * p.Hkv + h;
            M = fmaxf(M, p.part_ml[(part * G + g) * 2]);
        }
        float L = 0.0f, O = 0.0f;
        for (int s = 0; s < rm.n_split; s++) {
            const int64_t part = (int64_t)(rm.part_off + s) * p.Hkv + h;
            const float ms = p.part_ml[(part * G + g) * 2];
            const float f = (ms == -INFINITY) ? 0.0f : exp2f(ms - M);
            L = fmaf(p.part_ml[(part * G + g) * 2 + 1], f, L);
            O = fmaf(p.part_o[(part * G + g) * D + d], f, O);
        }
        p.out[((int64_t)blockIdx.x * p.Hq + h * G + g) * D + d] = O / L;
    }
}

// ------------------------------------------------------------ generic ----
// One CTA per (query row, kv head); warp w serves query heads w, w+nw, ...
// of the group, one token at a time with an online softmax.  head_dim up
// to 256.  table == NULL reads contiguous K/V [kv_len][Hkv][D].
template <typename T>
__global__ void attn_generic_kernel(const AttnParams p) {
    const int row = blockIdx.x, h = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int G = p.Hq / p.Hkv, D = p.D, bs = p.block_size;
    const RowMeta rm = p.rows[row];
    const int32_t* tab = p.table ? p.table + (int64_t)rm.table_row * p.max_bps : nullptr;
    const T* K = reinterpret_cast<const T*>(p.kbase);
    const T* V = reinterpret_cast<const T*>(p.vbase);
    for (int g = warp; g < G; g += nw) {
        const float* q = p.q + ((int64_t)row * p.Hq + h * G + g) * D;
        float qv[8], o[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int d = lane + 32 * i;
            qv[i] = d < D ? q[d] : 0.0f;
            o[i] = 0.0f;
        }
        float m = -INFINITY, l = 0.0f;
        for (int j = 0; j < rm.kv_len; j++) {
            int64_t slot = j;
            if (tab) {
                const int32_t b = tab[j / bs];
                if ((uint32_t)b >= (uint32_t)p.max_blocks) {
                    if (lane == 0) atomicOr(p.err, kErrBounds);
                    continue;
                }
                slot = (int64_t)b * bs + j % bs;
            }
            const T* kr = K + (slot * p.Hkv + h) * D;
            const T* vr = V + (slot * p.Hkv + h) * D;
            float dot = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int d = lane + 32 * i;
                if (d < D) dot = fmaf(qv[i], load_elem<T>(kr + d), dot);
            }
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) dot += __shfl_xor_sync(kFull, dot, off);
            const float s = dot * p.scale_log2;
            const float mn = fmaxf(m, s);
            const float c = exp2f(m - mn);
            const float pj = exp2f(s - mn);
            l = fmaf(l, c, pj);
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int d = lane + 32 * i;
                if (d < D) o[i] = fmaf(pj, load_elem<T>(vr + d), o[i] * c);
            }
            m = mn;
        }
        float* out = p.out + ((int64_t)row * p.Hq + h * G + g) * D;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int d = lane + 32 * i;
            if (d < D) out[d] = o[i] / l;
        }
    }
}

// -------------------------------------------------------------- launch ----
bool tma_attention_supported(int dtype, int D, int G, int block_size) {
    (void)dtype;
    return block_size == 16 && (D == 64 || D == 128) && (G == 1 || G == 2 || G == 4 || G == 7 || G == 8);
}

int tma_warps_per_cta(int dtype, int D) { return (dtype == S1KV_DTYPE_F32 && D == 128) ? 4 : 8; }

template <typename T, int D, int G>
static int launch_decode_t(s1kv_pool* pool, const AttnParams& p, cudaStream_t stream) {
    using C = DecodeCfg<T, D, G>;
    static bool attr_set = false;
    if (!attr_set) {
        S1KV_CUDA(cudaFuncSetAttribute(decode_tma_kernel<T, D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       C::kSmem));
        attr_set = true;
    }
    dim3 grid((unsigned)p.n_items, (unsigned)p.Hkv);
    decode_tma_kernel<T, D, G><<<grid, C::kNW * 32, C::kSmem, stream>>>(p, pool->tmap_k, pool->tmap_v);
    g_launches++;
    S1KV_CUDA(cudaGetLastError());
    bool any_multi = true;  // combine exits early for single-split rows
    if (any_multi) {
        combine_kernel<<<dim3((unsigned)p.n_rows, (unsigned)p.Hkv), 128, 0, stream>>>(p, G);
        g_launches++;
        S1KV_CUDA(cudaGetLastError());
    }
    return S1KV_OK;
}

template <typename T, int D>
static int launch_decode_g(s1kv_pool* pool, const AttnParams& p, int G, cudaStream_t stream) {
    switch (G) {
        case 1: return launch_decode_t<T, D, 1>(pool, p, stream);
        case 2: return launch_decode_t<T, D, 2>(pool, p, stream);
        case 4: return launch_decode_t<T, D, 4>(pool, p, stream);
        case 7: return launch_decode_t<T, D, 7>(pool, p, stream);
        case 8: return launch_decode_t<T, D, 8>(pool, p, stream);
        default: return set_error(S1KV_EINVAL, "decode: unsupported group size %d", G);
    }
}

int launch_attention_generic(const AttnParams& p, int dtype, cudaStream_t stream) {
    if (p.n_rows <= 0) return S1KV_OK;
    if (p.D > 256) return set_error(S1KV_EINVAL, "attention: head_dim > 256 unsupported");
    const int G = p.Hq / p.Hkv;
    const int threads = 32 * std::min(G, 8);
    dim3 grid((unsigned)p.n_rows, (unsigned)p.Hkv);
    if (dtype == S1KV_DTYPE_F32) attn_generic_kernel<float><<<grid, threads, 0, stream>>>(p);
    else attn_generic_kernel<uint16_t><<<grid, threads, 0, stream>>>(p);
    g_launches++;
    S1KV_CUDA(cudaGetLastError());
    return S1KV_OK;
}

int launch_attention(s1kv_pool* pool, const AttnParams& p, int dtype, cudaStream_t stream) {
    if (p.n_rows <= 0) return S1KV_OK;
    const int G = p.Hq / p.Hkv;
    if (p.table && pool->tmap_ok && p.items && tma_attention_supported(dtype, p.D, G, p.block_size)) {
        if (dtype == S1KV_DTYPE_F32)
            return p.D == 128 ? launch_decode_g<float, 128>(pool, p, G, stream)
                              : launch_decode_g<float, 64>(pool, p, G, stream);
        return p.D == 128 ? launch_decode_g<uint16_t, 128>(pool, p, G, stream)
                          : launch_decode_g<uint16_t, 64>(pool, p, G, stream);
    }
    return launch_attention_generic(p, dtype, stream);
}

// --------------------------------------------------------- tensor maps ---
// One 4-D map per storage tensor: (head_dim, kv head, slot, layer), box
// (head_dim, 1, 16, 1): one KV head's 16 rows of one block.  No swizzle:
// the kernels' chunk assignment is already conflict-free.
int make_tensor_maps(s1kv_pool* p) {
    p->tmap_ok = false;
    const int D = p->desc.head_dim;
    if (p->desc.block_size != 16 || !(D == 64 || D == 128)) return S1KV_OK;  // generic kernel only
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        S1KV_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !fn)
            return set_error(S1KV_ECUDA, "s1kv: cuTensorMapEncodeTiled unavailable");
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    const CUtensorMapDataType dt =
        p->desc.dtype == S1KV_DTYPE_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const cuuint64_t e = p->elem;
    cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)p->desc.num_kv_heads, (cuuint64_t)p->num_slots,
                          (cuuint64_t)p->desc.num_layers};
    cuuint64_t strides[3] = {D * e, (cuuint64_t)p->desc.num_kv_heads * D * e,
                             (cuuint64_t)p->num_slots * p->desc.num_kv_heads * D * e};
    cuuint32_t box[4] = {(cuuint32_t)D, 1, 16, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    for (int which = 0; which < 2; which++) {
        CUresult r = encode(which ? &p->tmap_v : &p->tmap_k, dt, 4, which ? (void*)p->v : (void*)p->k, dims, strides,
                            box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return set_error(S1KV_ECUDA, "s1kv: cuTensorMapEncodeTiled failed (%d)", (int)r);
    }
    p->tmap_ok = true;
    return S1KV_OK;
}

}  // namespace s1kv
