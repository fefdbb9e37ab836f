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
// 16-token tile costs 16 ldmatrix and 64 mma instructions per warp.
//   * S[head, token] = Q K^T: M = query heads of the group (padded to 16,
//     rows >= G are zero), N = 8 tokens, K = 16 dims.  K tiles arrive by
//     TMA in the 128-byte-swizzled layout (two 64-element halves per row),
//     so ldmatrix reads them without bank conflicts.
//   * The score fragment of a thread (head g, tokens 2t, 2t+1, 2t+8, 2t+9)
//     is exactly its A fragment of O += P V, so P never leaves registers;
//     V fragments come from ldmatrix.trans.
//   * Precision: q (fp32, pre-scaled by log2(e)/sqrt(D)) and p are each
//     split into bf16 hi + lo parts and both parts are multiplied (K and V
//     are exact in bf16), so scores and outputs carry fp32-level error
//     (about 2^-17 relative), not bf16 error.
//   * Online softmax in the exp2 domain per head, replicated over the 4
//     lanes of a head; the reference max moves only when a tile's max
//     outgrows it by 2^8, and only then is that head's O rescaled.
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
constexpr int kNS = 3;                         // stages per warp
constexpr int kMinCtas = 2;
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
__device__ __forceinline__ void tma4(void* dst, const CUtensorMap* m, uint64_t* b, int c0, int c1, int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];" ::"r"(su32(dst)),
        "l"(m), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(su32(b))
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

// c += A B for one m16n8k16 tile; A rows 8..15 (padding heads) are zero.
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
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
    pdl_enter();
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, tq = lane & 3;  // mma fragment coordinates: head row, column pair
    const int h = blockIdx.y;
    const WorkItem item = p.items[blockIdx.x];
    const RowMeta rm = p.rows[item.row];
    const int tok0 = item.split * p.split_tokens;
    const int tok1 = min(tok0 + p.split_tokens, rm.kv_len);
    const int n_tiles = (tok1 - tok0 + kTile - 1) / kTile;
    const int my_tiles = n_tiles > warp ? (n_tiles - warp + kNW - 1) / kNW : 0;
    const int32_t* tab = p.table + (int64_t)rm.table_row * p.max_bps;
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
        tma4(dst, &tmK, &bar[s], 0, h, row, p.layer);
        tma4(dst + kBoxBytes, &tmK, &bar[s], 64, h, row, p.layer);
        tma4(dst + kTileBytes, &tmV, &bar[s], 0, h, row, p.layer);
        tma4(dst + kTileBytes + kBoxBytes, &tmV, &bar[s], 64, h, row, p.layer);
    };
    for (int k = 0; k < min(kNS, my_tiles); k++) {
        const int row = __shfl_sync(kFull, my_row, k);
        if (lane == 0) issue(k, row);
    }

    // A fragments of q (pre-scaled, split hi + lo): k-step ks covers dims
    // 16ks .. 16ks+15; this lane holds dims 2tq, 2tq+1 (a0) and 2tq+8, 2tq+9
    // (a2) of head gq.
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

    float o[kD / 8][4];  // O[head gq][8nb + 2tq + {0,1}] in [nb][0..1]; [2..3] are padding rows
#pragma unroll
    for (int nb = 0; nb < kD / 8; nb++) o[nb][0] = o[nb][1] = o[nb][2] = o[nb][3] = 0.0f;
    float m = -INFINITY, l = 0.0f;  // head gq: reference max (log2 units), this lane's share of the sum

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

        // ---- S = Q K^T: n-block 0 = tokens 0-7, 1 = tokens 8-15 ----
        float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ks = 0; ks < kD / 16; ks++) {
            uint32_t b[4];  // matrix mi: tokens 8(mi >> 1) + r8, dims 16ks + 8(mi & 1) ..
            ldsm_x4(tile_chunk(Kt, (mi >> 1) * 8 + r8, ks * 2 + (mi & 1)), b);
            mma16816(s0, qh[ks][0], qh[ks][1], b[0], b[1]);
            mma16816(s0, ql[ks][0], ql[ks][1], b[0], b[1]);
            mma16816(s1, qh[ks][0], qh[ks][1], b[2], b[3]);
            mma16816(s1, ql[ks][0], ql[ks][1], b[2], b[3]);
        }
        // this lane: head gq, tokens 2tq, 2tq+1, 2tq+8, 2tq+9
        float x[4] = {s0[0], s0[1], s1[0], s1[1]};
        if (valid < kTile) {
            if (2 * tq >= valid) x[0] = -INFINITY;
            if (2 * tq + 1 >= valid) x[1] = -INFINITY;
            if (2 * tq + 8 >= valid) x[2] = -INFINITY;
            if (2 * tq + 9 >= valid) x[3] = -INFINITY;
        }
        float mx = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
        mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 2));
        const bool raise = mx > m + kRescaleAt;
        if (__any_sync(kFull, raise)) {
            const float corr = raise ? ex2(m - mx) : 1.0f;  // 0 on the first tile (m = -inf)
            if (raise) {
                m = mx;
                l *= corr;
            }
#pragma unroll
            for (int nb = 0; nb < kD / 8; nb++) {
                o[nb][0] *= corr;
                o[nb][1] *= corr;
            }
        }
        float pr[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            pr[i] = ex2(x[i] - m);
            l += pr[i];
        }
        uint32_t ph01, pl01, ph23, pl23;  // A fragment of P: tokens (2tq, 2tq+1) and (2tq+8, 2tq+9)
        split_bf16(pr[0], pr[1], ph01, pl01);
        split_bf16(pr[2], pr[3], ph23, pl23);

        // ---- O += P V: two n-blocks (16 dims) per ldmatrix.x4.trans ----
#pragma unroll
        for (int nb2 = 0; nb2 < kD / 16; nb2++) {
            uint32_t b[4];  // matrix mi: tokens 8(mi & 1) + r8, dims 16nb2 + 8(mi >> 1) ..
            ldsm_x4_t(tile_chunk(Vt, (mi & 1) * 8 + r8, nb2 * 2 + (mi >> 1)), b);
            mma16816(o[2 * nb2], ph01, ph23, b[0], b[1]);
            mma16816(o[2 * nb2], pl01, pl23, b[0], b[1]);
            mma16816(o[2 * nb2 + 1], ph01, ph23, b[2], b[3]);
            mma16816(o[2 * nb2 + 1], pl01, pl23, b[2], b[3]);
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

    if (failed) {
        // drain this warp's copies still in flight before the CTA exits
        if (lane == 0) atomicOr(p.err, kErrTimeout);
        const int issued = min(my_tiles, consumed + kNS);
        for (int k = consumed + 1; k < issued; k++) bar_wait(&bar[k % kNS], (uint32_t)((k / kNS) & 1));
        m = -INFINITY;
        l = 0.0f;
#pragma unroll
        for (int nb = 0; nb < kD / 8; nb++) o[nb][0] = o[nb][1] = 0.0f;
    }
    l += __shfl_xor_sync(kFull, l, 1);
    l += __shfl_xor_sync(kFull, l, 2);

    // ---- merge the warps through shared memory (aliases the rings) ----
    __syncthreads();
    float* mo = reinterpret_cast<float*>(smem);  // [kNW][G][kD]
    float* mml = mo + kNW * G * kD;              // [kNW][G][2]
    if (gq < G) {
#pragma unroll
        for (int nb = 0; nb < kD / 8; nb++)
            *reinterpret_cast<float2*>(&mo[(warp * G + gq) * kD + nb * 8 + 2 * tq]) = make_float2(o[nb][0], o[nb][1]);
        if (tq == 0) {
            mml[(warp * G + gq) * 2] = m;
            mml[(warp * G + gq) * 2 + 1] = l;
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
    if (rm.n_split == 1) signal_done(p);
    if (p.counters && rm.n_split > 1)
        finish_split_row(p, item.row, h, rm.n_split, G, kD, reinterpret_cast<int*>(smem + kRing + kNW * kNS * 8),
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
