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
//     the split.  A tile is 8 or 16 tokens of one block; its K rows and V
//     rows for the kv head are two TMA boxes (tile rows x head_dim) landing
//     in the warp's ring of NS shared-memory stages, completion tracked by
//     one mbarrier per stage (bounded waits; a timeout sets the device
//     error word).  Rings are small so 3-4 CTAs (12-16 warps) share an SM.
//     No TMA multicast anywhere.
//   * QK: LPT lanes share one token; lane part p reads 16-byte chunks
//     p, p+LPT, ... of the row, so each quarter-warp phase hits 8 distinct
//     bank groups.  q stays in registers as float pairs and the dot runs on
//     packed fp32 FMA (__ffma2_rn).  A transpose-reduce leaves each lane
//     with ONE full (token, head) score, so exponentials are not repeated
//     across lanes.
//   * online softmax per tile in the exp2 domain (ex2.approx); PV with
//     lanes over head dims (D/32 each, packed FMA) and p broadcast from a
//     small per-warp shared-memory table.
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

#include "combine.cuh"
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

template <typename T>
__device__ __forceinline__ float load_elem(const T* src) {
    if constexpr (sizeof(T) == 4) return *reinterpret_cast<const float*>(src);
    else return __uint_as_float((uint32_t)(*reinterpret_cast<const uint16_t*>(src)) << 16);
}

// ------------------------------------------------------- configuration ---
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

constexpr int ilog2(int x) { return x <= 1 ? 0 : 1 + ilog2(x / 2); }
constexpr int pow2ceil(int x) { return x <= 1 ? 1 : 2 * pow2ceil((x + 1) / 2); }

// Tokens per pipeline stage (one TMA box of K and one of V) and stages per
// warp, by storage type and head dim: the ring of 4 warps fits 3-4 CTAs per
// SM (12-16 resident warps) while keeping >= 64 KB of loads in flight.
template <int ELEM, int D>
struct StageCfg;
template <> struct StageCfg<4, 128> { static constexpr int kTile = 8, kNS = 2, kMinCtas = 3; };
template <> struct StageCfg<2, 128> { static constexpr int kTile = 16, kNS = 2, kMinCtas = 3; };
template <> struct StageCfg<4, 64> { static constexpr int kTile = 16, kNS = 2, kMinCtas = 3; };
template <> struct StageCfg<2, 64> { static constexpr int kTile = 16, kNS = 3, kMinCtas = 4; };

int decode_tile_rows(int dtype, int D) {
    if (dtype == S1KV_DTYPE_F32) return D == 128 ? StageCfg<4, 128>::kTile : StageCfg<4, 64>::kTile;
    return D == 128 ? StageCfg<2, 128>::kTile : StageCfg<2, 64>::kTile;
}

template <typename T, int D, int G>
struct DecodeCfg {
    using S = StageCfg<(int)sizeof(T), D>;
    static constexpr int kNV = pow2ceil(G);                           // heads padded to a power of two
    static constexpr int kH = ilog2(kNV);                             // halving levels of the reduce
    static constexpr int kEPC = 16 / (int)sizeof(T);                  // elements per 16-byte chunk
    static constexpr int kNCH = D / kEPC;                             // chunks per row
    static constexpr int kLPT = (kNV * D / 8 > 64 && kNCH >= 16) ? 16 : 8;  // lanes per token (QK)
    static constexpr int kIT = kNCH / kLPT;                           // chunks per lane per row
    static constexpr int kDQ = D / kLPT;                              // q dims per lane per head
    static constexpr int kTPS = 32 / kLPT;                            // tokens per QK step
    static constexpr int kTile = S::kTile;                            // tokens per stage
    static constexpr int kSteps = kTile / kTPS;                       // QK steps per stage
    static constexpr int kDPL = D / 32;                               // PV dims per lane
    static constexpr int kTileBytes = kTile * D * (int)sizeof(T);     // one K (or V) box
    static constexpr int kStageBytes = 2 * kTileBytes;
    static constexpr int kNW = 4;                                     // warps per CTA
    static constexpr int kNS = S::kNS;                                // stages per warp
    static constexpr int kPFloats = (kTile * kNV + kNV + 3) / 4 * 4;  // p[tile][head] + corr[head]
    static constexpr int kRing = kNW * kNS * kStageBytes;
    static constexpr int kSmem = kRing + kNW * kPFloats * 4 + kNW * kNS * 8 + 16;  // + last-CTA flag
    static_assert(kNCH % kLPT == 0, "chunks must split evenly over lanes");
    static_assert(kLPT >= 8, "a quarter-warp phase must read 8 distinct chunks");
    static_assert((1 << kH) <= kLPT, "one halving level per lane bit");
    static_assert(kTile % kTPS == 0 && 16 % kTile == 0, "tiles are whole QK steps inside one block");
    static_assert(kRing >= kNW * kNV * (D + 2) * 4, "merge area must fit in the stage ring");
    static_assert((kPFloats * 4) % 16 == 0, "p area keeps 16-byte alignment");
};

// Sums NV per-lane partial dots over the LPT lanes of a token so that each
// lane ends with ONE full dot: halving levels trade half of the values with
// the partner lane (one shuffle per traded value), then plain butterflies
// finish.  The lane keeps head index sum_i hi_i * (NV >> (i+1)), where hi_i
// is the lane bit (LPT >> (i+1)).
template <int NV, int LPT>
__device__ __forceinline__ float reduce_transpose(float (&a)[NV], int lane) {
    constexpr int H = ilog2(NV);
#pragma unroll
    for (int i = 0; i < H; i++) {
        const int off = LPT >> (i + 1);
        const int half = NV >> (i + 1);
        const bool hi = (lane & off) != 0;
#pragma unroll
        for (int x = 0; x < half; x++) {
            const float send = hi ? a[x] : a[x + half];
            const float keep = hi ? a[x + half] : a[x];
            a[x] = keep + __shfl_xor_sync(kFull, send, off);
        }
    }
#pragma unroll
    for (int off = LPT >> (H + 1); off >= 1; off >>= 1) a[0] += __shfl_xor_sync(kFull, a[0], off);
    return a[0];
}

template <int NV, int LPT>
__device__ __forceinline__ int reduced_head(int lane) {
    constexpr int H = ilog2(NV);
    int g = 0;
#pragma unroll
    for (int i = 0; i < H; i++) g |= ((lane & (LPT >> (i + 1))) ? 1 : 0) << (H - 1 - i);
    return g;
}

// 16 bytes of storage -> EPC/2 float pairs.
template <typename T>
__device__ __forceinline__ void load_pairs(const T* src, float2* x);

template <>
__device__ __forceinline__ void load_pairs<float>(const float* src, float2* x) {
    float4 a = *reinterpret_cast<const float4*>(src);
    x[0] = make_float2(a.x, a.y);
    x[1] = make_float2(a.z, a.w);
}

template <>
__device__ __forceinline__ void load_pairs<uint16_t>(const uint16_t* src, float2* x) {
    uint4 a = *reinterpret_cast<const uint4*>(src);
    x[0] = make_float2(bf16lo(a.x), bf16hi(a.x));
    x[1] = make_float2(bf16lo(a.y), bf16hi(a.y));
    x[2] = make_float2(bf16lo(a.z), bf16hi(a.z));
    x[3] = make_float2(bf16lo(a.w), bf16hi(a.w));
}

// N = D/32 consecutive storage elements (2 or 4) -> N/2 float pairs.
template <typename T, int N>
__device__ __forceinline__ void load_vpairs(const T* src, float2* x) {
    if constexpr (sizeof(T) == 4) {
        if constexpr (N == 4) {
            float4 a = *reinterpret_cast<const float4*>(src);
            x[0] = make_float2(a.x, a.y);
            x[1] = make_float2(a.z, a.w);
        } else {
            x[0] = *reinterpret_cast<const float2*>(src);
        }
    } else {
        if constexpr (N == 4) {
            uint2 a = *reinterpret_cast<const uint2*>(src);
            x[0] = make_float2(bf16lo(a.x), bf16hi(a.x));
            x[1] = make_float2(bf16lo(a.y), bf16hi(a.y));
        } else {
            uint32_t a = *reinterpret_cast<const uint32_t*>(src);
            x[0] = make_float2(bf16lo(a), bf16hi(a));
        }
    }
}

// ------------------------------------------------------------- decode ----
template <typename T, int D, int G>
__global__ void __launch_bounds__(DecodeCfg<T, D, G>::kNW * 32, DecodeCfg<T, D, G>::S::kMinCtas)
    decode_tma_kernel(const __grid_constant__ AttnParams p, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV) {
    using C = DecodeCfg<T, D, G>;
    constexpr int NW = C::kNW, NS = C::kNS, NV = C::kNV, LPT = C::kLPT, IT = C::kIT, EPC = C::kEPC,
                  TPS = C::kTPS, STEPS = C::kSteps, DPL = C::kDPL, DQ = C::kDQ, TILE = C::kTile;
    extern __shared__ __align__(1024) uint8_t smem[];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // CTA index = item * Hkv + head: the heads of one item run side by side
    // and read the same token rows of the pool together
    const int h = (int)(blockIdx.x % (unsigned)p.Hkv);
    const WorkItem item = p.items[blockIdx.x / (unsigned)p.Hkv];
    const int tok0 = item.split * p.split_tokens;
    const int tok1 = min(tok0 + p.split_tokens, item.kv_len);
    const int n_tiles = (tok1 - tok0 + TILE - 1) / TILE;
    const int my_tiles = n_tiles > warp ? (n_tiles - warp + NW - 1) / NW : 0;
    const int32_t* tab = p.table + (int64_t)item.table_row * p.max_bps;

    uint8_t* ring = smem + warp * NS * C::kStageBytes;
    float* Ps = reinterpret_cast<float*>(smem + C::kRing) + warp * C::kPFloats;  // [TILE][NV]
    float* Cs = Ps + TILE * NV;                                                 // [NV]
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::kRing + NW * C::kPFloats * 4) + warp * NS;

    // TMA row coordinate of this warp's k-th tile for k = lane (first 32).
    auto tile_row = [&](int k, int& row) -> bool {
        const int base = tok0 + (warp + k * NW) * TILE;
        const int32_t blk = tab[base >> 4];
        if ((uint32_t)blk >= (uint32_t)p.max_blocks) {
            row = p.max_blocks * 16;  // out of range: TMA zero-fills the box
            return false;
        }
        row = blk * 16 + (base & 15);
        return true;
    };
    int my_row = 0;
    if (lane < my_tiles && !tile_row(lane, my_row)) atomicOr(p.err, kErrBounds);
    if (lane == 0) {
        for (int s = 0; s < NS; s++) mbar_init(&bar[s], 1);
        fence_barrier_init();
    }
    __syncwarp();

    auto issue = [&](int k, int row) {
        const int s = k % NS;
        uint8_t* dst = ring + s * C::kStageBytes;
        mbar_expect_tx(&bar[s], C::kStageBytes);
        tma_load_4d(dst, &tmK, &bar[s], 0, h, row, p.layer);
        tma_load_4d(dst + C::kTileBytes, &tmV, &bar[s], 0, h, row, p.layer);
    };
    {
        // The first copies: tiles entirely below the tokens this batch
        // appends are requested before the wait (items, block table and those
        // K/V rows were written before the previous kernel started), the
        // rest after it.
        const int n_first = min(NS, my_tiles);
        int pre = 0;
        if (p.prewait) {
            const int safe_end = item.kv_len - p.prewait_margin;
            while (pre < n_first && tok0 + (warp + pre * NW) * TILE + TILE <= safe_end) pre++;
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
    }
    const RowMeta rm = p.rows[item.row];  // split count and partial offset, needed at the end

    // q of the group's heads (padded heads are zero): lane part pp holds
    // chunks pp, pp+LPT, ... of each head as float pairs.
    const int pp = lane % LPT;
    const int tl = lane / LPT;
    const int my_g = reduced_head<NV, LPT>(lane);
    float2 q2[NV][DQ / 2];
#pragma unroll
    for (int g = 0; g < NV; g++) {
        const float* qrow = p.q + ((int64_t)item.row * p.Hq + h * G + (g < G ? g : 0)) * D;
#pragma unroll
        for (int it = 0; it < IT; it++) {
            const float4* src = reinterpret_cast<const float4*>(qrow + (it * LPT + pp) * EPC);
#pragma unroll
            for (int e4 = 0; e4 < EPC / 4; e4++) {
                float4 v = g < G ? __ldg(src + e4) : make_float4(0.f, 0.f, 0.f, 0.f);
                q2[g][(it * EPC + e4 * 4) / 2] = make_float2(v.x, v.y);
                q2[g][(it * EPC + e4 * 4) / 2 + 1] = make_float2(v.z, v.w);
            }
        }
    }

    float m = -INFINITY, l = 0.0f;  // running max / sum of head my_g (this lane's tokens)
    float2 o2[NV][DPL / 2];
#pragma unroll
    for (int g = 0; g < NV; g++)
#pragma unroll
        for (int d = 0; d < DPL / 2; d++) o2[g][d] = make_float2(0.f, 0.f);

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
        const T* Vs = Ks + TILE * D;
        const int base = tok0 + (warp + k * NW) * TILE;
        const int valid = min(TILE, tok1 - base);

        // ---- scores: one (token, head) per lane per step ----
        float sc[STEPS];
#pragma unroll
        for (int j = 0; j < STEPS; j++) {
            const int t = j * TPS + tl;
            const T* krow = Ks + t * D;
            float2 acc2[NV];
#pragma unroll
            for (int g = 0; g < NV; g++) acc2[g] = make_float2(0.f, 0.f);
#pragma unroll
            for (int it = 0; it < IT; it++) {
                float2 kf[EPC / 2];
                load_pairs<T>(krow + (it * LPT + pp) * EPC, kf);
#pragma unroll
                for (int g = 0; g < NV; g++)
#pragma unroll
                    for (int e = 0; e < EPC / 2; e++) acc2[g] = __ffma2_rn(q2[g][it * EPC / 2 + e], kf[e], acc2[g]);
            }
            float acc[NV];
#pragma unroll
            for (int g = 0; g < NV; g++) acc[g] = acc2[g].x + acc2[g].y;
            const float dot = reduce_transpose<NV, LPT>(acc, lane);
            sc[j] = (t < valid) ? dot * p.scale_log2 : -INFINITY;
        }

        // ---- online softmax for head my_g ----
        float mx = sc[0];
#pragma unroll
        for (int j = 1; j < STEPS; j++) mx = fmaxf(mx, sc[j]);
#pragma unroll
        for (int off = LPT; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, off));
        const float mn = fmaxf(m, mx);
        const float corr = ex2(m - mn);
        m = mn;
        float ls = 0.0f;
#pragma unroll
        for (int j = 0; j < STEPS; j++) {
            const float pj = ex2(sc[j] - mn);
            ls += pj;
            Ps[(j * TPS + tl) * NV + my_g] = pj;
        }
        l = fmaf(l, corr, ls);
        if (tl == 0) Cs[my_g] = corr;
        __syncwarp();

        // ---- PV: lanes over head dims, p broadcast from shared memory ----
        float cg[NV];
#pragma unroll
        for (int g = 0; g < NV; g++) cg[g] = Cs[g];
#pragma unroll
        for (int g = 0; g < NV; g++)
#pragma unroll
            for (int d = 0; d < DPL / 2; d++) o2[g][d] = __fmul2_rn(o2[g][d], make_float2(cg[g], cg[g]));
#pragma unroll
        for (int u = 0; u < TILE; u++) {
            if (u < valid) {
                float2 vf[DPL / 2];
                load_vpairs<T, DPL>(Vs + u * D + lane * DPL, vf);
                float pu[NV];
#pragma unroll
                for (int g = 0; g < NV; g++) pu[g] = Ps[u * NV + g];
#pragma unroll
                for (int g = 0; g < NV; g++)
#pragma unroll
                    for (int d = 0; d < DPL / 2; d++) o2[g][d] = __ffma2_rn(make_float2(pu[g], pu[g]), vf[d], o2[g][d]);
            }
        }
        __syncwarp();
        if (k + NS < my_tiles) {
            int row = __shfl_sync(kFull, my_row, (k + NS) & 31);
            if (k + NS >= 32) {
                // Past the 32 prefetched rows (splits longer than 32 tiles per
                // warp): look the block up directly.
                if (!tile_row(k + NS, row) && lane == 0) atomicOr(p.err, kErrBounds);
            }
            if (lane == 0) {
                fence_proxy_async();
                issue(k + NS, row);
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
        // Drain this warp's copies still in flight before the CTA exits.
        if (lane == 0) atomicOr(p.err, kErrTimeout);
        const int issued = min(my_tiles, consumed + NS);
        for (int k = consumed + 1; k < issued; k++) mbar_wait_bounded(&bar[k % NS], (uint32_t)((k / NS) & 1));
        m = -INFINITY;
        l = 0.0f;
#pragma unroll
        for (int g = 0; g < NV; g++)
#pragma unroll
            for (int d = 0; d < DPL / 2; d++) o2[g][d] = make_float2(0.f, 0.f);
    }

    // Sum l of head my_g over the token lanes (lanes inside one token group
    // hold copies).
#pragma unroll
    for (int off = LPT; off < 32; off <<= 1) l += __shfl_xor_sync(kFull, l, off);

    // ---- merge the NW warps through shared memory (aliases the rings) ----
    __syncthreads();
    float* mo = reinterpret_cast<float*>(smem);   // [NW][NV][D]
    float* mml = mo + NW * NV * D;                 // [NW][NV][2]
#pragma unroll
    for (int g = 0; g < NV; g++)
#pragma unroll
        for (int d = 0; d < DPL / 2; d++)
            *reinterpret_cast<float2*>(&mo[(warp * NV + g) * D + lane * DPL + 2 * d]) = o2[g][d];
    if (tl == 0) {
        mml[(warp * NV + my_g) * 2] = m;
        mml[(warp * NV + my_g) * 2 + 1] = l;
    }
    __syncthreads();
    const int64_t part = (int64_t)(rm.part_off + item.split) * p.Hkv + h;
    for (int idx = threadIdx.x; idx < G * D; idx += NW * 32) {
        const int g = idx / D, d = idx % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; w++) M = fmaxf(M, mml[(w * NV + g) * 2]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; w++) {
            const float mw = mml[(w * NV + g) * 2];
            const float f = (mw == -INFINITY) ? 0.0f : ex2(mw - M);
            L = fmaf(mml[(w * NV + g) * 2 + 1], f, L);
            O = fmaf(mo[(w * NV + g) * D + d], f, O);
        }
        if (rm.n_split == 1) {
            store_out(p, item.row, h * G + g, d, D, O / L);
        } else {
            p.part_o[(part * G + g) * D + d] = O;
            if (d == 0) {
                p.part_ml[(part * G + g) * 2] = M;
                p.part_ml[(part * G + g) * 2 + 1] = L;
            }
        }
    }
    if (p.counters && rm.n_split > 1)
        finish_split_row(p, item.row, h, item.split, rm.n_split, G, D,
                         reinterpret_cast<int*>(smem + C::kRing + NW * C::kPFloats * 4 + NW * NS * 8),
                         reinterpret_cast<float*>(smem), C::kRing / 4);  // the rings are free by now
}

// Combines the split partials of multi-split rows (separate pass, for
// launches without arrival counters): rescale to the global max, sum,
// normalise.
__global__ void combine_kernel(const AttnParams p, int G) {
    if (p.rows[blockIdx.x].n_split <= 1) return;
    combine_partials(p, blockIdx.x, blockIdx.y, G, p.D, threadIdx.x, blockDim.x);
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

int tma_warps_per_cta(int dtype, int D) {
    (void)dtype;
    (void)D;
    return 4;
}

template <typename T, int D, int G>
static int launch_decode_t(s1kv_pool* pool, const AttnParams& p, cudaStream_t stream) {
    using C = DecodeCfg<T, D, G>;
    static std::atomic<uint64_t> attr_set{0};  // per device
    int st = once_per_device(attr_set, [] {
        S1KV_CUDA(cudaFuncSetAttribute(decode_tma_kernel<T, D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       C::kSmem));
        return S1KV_OK;
    });
    if (st) return st;
    if ((int64_t)p.n_items * p.Hkv > INT32_MAX) return set_error(S1KV_EINVAL, "decode: too many work items");
    const dim3 grid((unsigned)((int64_t)p.n_items * p.Hkv));
    S1KV_CUDA(launch_pdl(decode_tma_kernel<T, D, G>, grid, dim3(C::kNW * 32), C::kSmem, stream, p, pool->tmap_k,
                         pool->tmap_v));
    g_launches++;
    S1KV_CUDA(cudaGetLastError());
    if (!p.counters) {  // otherwise the last CTA of each split row merged it; combine exits early for single-split rows
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
    if (p.table && pool->tmap_sw_ok && p.items && decode_mma_supported(dtype, p.D, G, p.block_size)) {
        // bf16 K/V, head_dim 128: tensor-core decode, then the shared combine
        int st = launch_decode_mma(p, pool->tmap_k_blk, pool->tmap_v_blk, stream);
        if (st || p.counters) return st;
        combine_kernel<<<dim3((unsigned)p.n_rows, (unsigned)p.Hkv), 128, 0, stream>>>(p, G);
        g_launches++;
        S1KV_CUDA(cudaGetLastError());
        return S1KV_OK;
    }
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
// (head_dim, 1, tile, 1): one KV head's rows of one decode tile (8 or 16
// tokens of one block).  No swizzle:
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
    cuuint32_t box[4] = {(cuuint32_t)D, 1, (cuuint32_t)decode_tile_rows(p->desc.dtype, D), 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    for (int which = 0; which < 2; which++) {
        CUresult r = encode(which ? &p->tmap_v : &p->tmap_k, dt, 4, which ? (void*)p->v : (void*)p->k, dims, strides,
                            box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return set_error(S1KV_ECUDA, "s1kv: cuTensorMapEncodeTiled failed (%d)", (int)r);
    }
    p->tmap_ok = true;
    // Tensor-core prefill reads 64-element halves of each row with 128B
    // swizzle, the layout UMMA consumes (bf16 pools, head_dim 128).
    p->tmap_sw_ok = false;
    if (p->desc.dtype == S1KV_DTYPE_BF16 && D == 128) {
        cuuint32_t box_sw[4] = {64, 1, 16, 1};
        for (int which = 0; which < 2; which++) {
            CUresult r = encode(which ? &p->tmap_v_sw : &p->tmap_k_sw, dt, 4, which ? (void*)p->v : (void*)p->k, dims,
                                strides, box_sw, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            if (r != CUDA_SUCCESS) return set_error(S1KV_ECUDA, "s1kv: cuTensorMapEncodeTiled (swizzled) failed (%d)", (int)r);
        }
        // The bf16 decode kernel takes a whole block of one KV head in one
        // copy: dimensions (64 elements, slot, half of the row, head, layer),
        // box (64, 16, 2, 1, 1).  Shared memory receives the two 128-byte
        // halves of the 16 rows one after the other, the layout of two
        // (64, 1, 16, 1) boxes above, with one TMA operation instead of two
        // (measured 1-2% faster on one-KV-head rows of 131,072 tokens).
        cuuint64_t dims5[5] = {64, (cuuint64_t)p->num_slots, 2, (cuuint64_t)p->desc.num_kv_heads,
                               (cuuint64_t)p->desc.num_layers};
        cuuint64_t strides5[4] = {(cuuint64_t)p->desc.num_kv_heads * D * e, 64 * e, (cuuint64_t)D * e,
                                  (cuuint64_t)p->num_slots * p->desc.num_kv_heads * D * e};
        cuuint32_t box5[5] = {64, 16, 2, 1, 1};
        cuuint32_t estr5[5] = {1, 1, 1, 1, 1};
        for (int which = 0; which < 2; which++) {
            CUresult r = encode(which ? &p->tmap_v_blk : &p->tmap_k_blk, dt, 5, which ? (void*)p->v : (void*)p->k,
                                dims5, strides5, box5, estr5, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            if (r != CUDA_SUCCESS) return set_error(S1KV_ECUDA, "s1kv: cuTensorMapEncodeTiled (block) failed (%d)", (int)r);
        }
        p->tmap_sw_ok = true;
    }
    return S1KV_OK;
}

}  // namespace s1kv

// ------------------------------------------ caller-supplied storage path ---
// Helpers for the no-allocation entry point (noalloc.cu): tensor maps over
// one layer of caller-owned K/V storage, and a launcher that takes them
// instead of a pool's.

namespace s1kv {

int encode_kv_maps(const void* k, const void* v, int dtype, int Hkv, int D, int64_t num_slots, CUtensorMap* tk,
                   CUtensorMap* tv) {
    // the driver entry point is looked up once per process
    static std::atomic<PFN_cuTensorMapEncodeTiled_v12000> cached{nullptr};
    PFN_cuTensorMapEncodeTiled_v12000 encode = cached.load(std::memory_order_acquire);
    if (!encode) {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        S1KV_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !fn)
            return set_error(S1KV_ECUDA, "s1kv: cuTensorMapEncodeTiled unavailable");
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
        cached.store(encode, std::memory_order_release);
    }
    const cuuint64_t e = dtype == S1KV_DTYPE_F32 ? 4 : 2;
    const CUtensorMapDataType dt =
        dtype == S1KV_DTYPE_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)Hkv, (cuuint64_t)num_slots, 1};
    cuuint64_t strides[3] = {D * e, (cuuint64_t)Hkv * D * e, (cuuint64_t)num_slots * Hkv * D * e};
    cuuint32_t box[4] = {(cuuint32_t)D, 1, (cuuint32_t)decode_tile_rows(dtype, D), 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    for (int which = 0; which < 2; which++) {
        CUresult r = encode(which ? tv : tk, dt, 4, const_cast<void*>(which ? v : k), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return set_error(S1KV_EINVAL, "s1kv: tensor map over the K/V storage rejected (%d)", (int)r);
    }
    return S1KV_OK;
}

template <typename T, int D, int G>
static int launch_with_maps_t(const AttnParams& p, const CUtensorMap& tk, const CUtensorMap& tv, cudaStream_t stream) {
    using C = DecodeCfg<T, D, G>;
    static std::atomic<uint64_t> attr_set{0};  // per device
    int st = once_per_device(attr_set, [] {
        S1KV_CUDA(cudaFuncSetAttribute(decode_tma_kernel<T, D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       C::kSmem));
        return S1KV_OK;
    });
    if (st) return st;
    if ((int64_t)p.n_items * p.Hkv > INT32_MAX) return set_error(S1KV_EINVAL, "decode: too many work items");
    decode_tma_kernel<T, D, G><<<dim3((unsigned)((int64_t)p.n_items * p.Hkv)), C::kNW * 32, C::kSmem, stream>>>(p, tk, tv);
    g_launches++;
    S1KV_CUDA(cudaGetLastError());
    combine_kernel<<<dim3((unsigned)p.n_rows, (unsigned)p.Hkv), 128, 0, stream>>>(p, G);
    g_launches++;
    S1KV_CUDA(cudaGetLastError());
    return S1KV_OK;
}

template <typename T, int D>
static int launch_with_maps_g(const AttnParams& p, const CUtensorMap& tk, const CUtensorMap& tv, int G,
                              cudaStream_t stream) {
    switch (G) {
        case 1: return launch_with_maps_t<T, D, 1>(p, tk, tv, stream);
        case 2: return launch_with_maps_t<T, D, 2>(p, tk, tv, stream);
        case 4: return launch_with_maps_t<T, D, 4>(p, tk, tv, stream);
        case 7: return launch_with_maps_t<T, D, 7>(p, tk, tv, stream);
        case 8: return launch_with_maps_t<T, D, 8>(p, tk, tv, stream);
        default: return set_error(S1KV_EINVAL, "decode: unsupported group size %d", G);
    }
}

int launch_decode_with_maps(const AttnParams& p, const CUtensorMap& tk, const CUtensorMap& tv, int dtype,
                            cudaStream_t stream) {
    const int G = p.Hq / p.Hkv;
    if (dtype == S1KV_DTYPE_F32)
        return p.D == 128 ? launch_with_maps_g<float, 128>(p, tk, tv, G, stream)
                          : launch_with_maps_g<float, 64>(p, tk, tv, G, stream);
    return p.D == 128 ? launch_with_maps_g<uint16_t, 128>(p, tk, tv, G, stream)
                      : launch_with_maps_g<uint16_t, 64>(p, tk, tv, G, stream);
}

}  // namespace s1kv
