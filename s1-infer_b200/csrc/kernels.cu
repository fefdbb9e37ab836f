// kernels.cu -- data-movement kernels of the paged KV cache: fused RoPE +
// slot-mapped append, plain append, standalone RoPE, copy-on-write block
// copy, gather (materialise a sequence), device block-table updates.
//
// All are HBM-bound byte movers: every thread moves 16-byte vectors, grids
// are sized in multiples of the 148 SMs, and nothing is staged through
// shared memory because nothing is reused.
#include <cuda_bf16.h>

#include <cmath>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "internal.h"

namespace s1kv {

constexpr int kSMs = 148;

// ------------------------------------------------------------ bf16 utils --
// Round-to-nearest-even narrowing; NaN becomes the quiet NaN 0x7FC0 with
// the input's sign.  Written out in integer arithmetic so the host oracle
// and the device agree on every input.
__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu) != 0) return (uint16_t)(((u >> 16) & 0x8000u) | 0x7FC0u);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

__device__ __forceinline__ float bf16_to_f32(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }

__device__ __forceinline__ void flag_error(int* err, int bit) {
    if (err) atomicOr(err, bit);
}

// -------------------------------------------------------- table updates --
__global__ void table_update_kernel(const TableUpdate* __restrict__ upd, int64_t n, int32_t* __restrict__ table,
                                    int32_t max_bps) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        TableUpdate u = upd[i];
        table[(int64_t)u.row * max_bps + u.col] = u.block;
    }
}

int launch_table_update(const TableUpdate* d_upd, int64_t n, int32_t* table, int32_t max_bps, cudaStream_t stream) {
    int grid = (int)std::min<int64_t>((n + 255) / 256, kSMs * 4);
    table_update_kernel<<<grid, 256, 0, stream>>>(d_upd, n, table, max_bps);
    g_launches++;
    S1KV_CUDA(cudaGetLastError());
    return S1KV_OK;
}

// ------------------------------------------------------ copy-on-write ----
// Copies whole physical blocks src[i] -> dst[i] of K and V in every layer.
// One block of one layer is bs * Hkv * D * elem bytes, contiguous.
__global__ void cow_kernel(const int32_t* __restrict__ src, const int32_t* __restrict__ dst, int64_t n_pairs,
                           int32_t n_layers, char* __restrict__ k, char* __restrict__ v, size_t layer_bytes,
                           size_t block_bytes, int32_t max_blocks, int* err) {
    const int64_t vec_per_block = (int64_t)(block_bytes / 16);
    const int64_t total = n_pairs * n_layers * 2 * vec_per_block;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t e = i % vec_per_block;
        int64_t r = i / vec_per_block;
        int which = (int)(r & 1);
        r >>= 1;
        int64_t layer = r % n_layers;
        int64_t pair = r / n_layers;
        int32_t s = src[pair], d = dst[pair];
        if ((uint32_t)s >= (uint32_t)max_blocks || (uint32_t)d >= (uint32_t)max_blocks) {
            flag_error(err, kErrBounds);
            continue;
        }
        char* base = (which ? v : k) + layer * layer_bytes;
        const int4* ps = reinterpret_cast<const int4*>(base + (size_t)s * block_bytes) + e;
        int4* pd = reinterpret_cast<int4*>(base + (size_t)d * block_bytes) + e;
        *pd = __ldcs(ps);
    }
}

int launch_cow(s1kv_pool* p, const int32_t* d_src, const int32_t* d_dst, int64_t n, cudaStream_t stream) {
    if (n <= 0) return S1KV_OK;
    size_t block_bytes = (size_t)p->desc.block_size * p->desc.num_kv_heads * p->desc.head_dim * p->elem;
    if (block_bytes % 16)
        return set_error(S1KV_EINVAL, "s1kv_cow_copy: block bytes (%zu) not a multiple of 16", block_bytes);
    int64_t total = n * p->desc.num_layers * 2 * (int64_t)(block_bytes / 16);
    int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, kSMs * 8));
    cow_kernel<<<grid, 256, 0, stream>>>(d_src, d_dst, n, p->desc.num_layers, p->k, p->v, p->layer_bytes, block_bytes,
                                         (int32_t)p->desc.max_blocks, p->d_err);
    g_launches++;
    S1KV_CUDA(cudaGetLastError());
    return S1KV_OK;
}

// -------------------------------------------------------------- append ----
// Work unit = 8 rotation pairs (j .. j+7 and j+D/2 .. j+D/2+7) of one
// (token, head): two 32-byte fp32 loads, two stores of 8 elements (32 B
// fp32, 16 B bf16).  Units cover K heads, then V heads, then Q heads.
//
// Rotation (src/nn/RoPE.cpp:32-33): out1 = x1*c - x2*s, out2 = x2*c + x1*s,
// each product and sum rounded separately (no fused multiply-add), as the
// reference's build computes them.

template <typename T>
__device__ __forceinline__ void store8(T* dst, const float* x);

template <>
__device__ __forceinline__ void store8<float>(float* dst, const float* x) {
    reinterpret_cast<float4*>(dst)[0] = make_float4(x[0], x[1], x[2], x[3]);
    reinterpret_cast<float4*>(dst)[1] = make_float4(x[4], x[5], x[6], x[7]);
}

template <>
__device__ __forceinline__ void store8<uint16_t>(uint16_t* dst, const float* x) {
    uint4 w;
    w.x = (uint32_t)f32_to_bf16(x[0]) | ((uint32_t)f32_to_bf16(x[1]) << 16);
    w.y = (uint32_t)f32_to_bf16(x[2]) | ((uint32_t)f32_to_bf16(x[3]) << 16);
    w.z = (uint32_t)f32_to_bf16(x[4]) | ((uint32_t)f32_to_bf16(x[5]) << 16);
    w.w = (uint32_t)f32_to_bf16(x[6]) | ((uint32_t)f32_to_bf16(x[7]) << 16);
    *reinterpret_cast<uint4*>(dst) = w;
}

__device__ __forceinline__ void load8(const float* src, float* x) {
    float4 a = __ldcs(reinterpret_cast<const float4*>(src));
    float4 b = __ldcs(reinterpret_cast<const float4*>(src) + 1);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

__device__ __forceinline__ void rotate8(float* x1, float* x2, const float2* cs) {
#pragma unroll
    for (int i = 0; i < 8; i++) {
        float c = cs[i].x, s = cs[i].y;
        float a = __fsub_rn(__fmul_rn(x1[i], c), __fmul_rn(x2[i], s));
        float b = __fadd_rn(__fmul_rn(x2[i], c), __fmul_rn(x1[i], s));
        x1[i] = a;
        x2[i] = b;
    }
}

template <typename T, bool ROPE>
__global__ void __launch_bounds__(256) append_vec_kernel(const AppendParams p) {
    pdl_enter();
    const int D = p.D, half = D / 2;
    const int upr = half / 8;  // units per (token, head)
    const int64_t kv_units = p.n * p.Hkv * upr;
    const int64_t q_units = (ROPE && p.q_in) ? p.n * p.Hq * upr : 0;
    const int64_t total = 2 * kv_units + q_units;
    for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < total; u += (int64_t)gridDim.x * blockDim.x) {
        int part;  // 0 = K, 1 = V, 2 = Q
        int64_t w;
        if (u < kv_units) { part = 0; w = u; }
        else if (u < 2 * kv_units) { part = 1; w = u - kv_units; }
        else { part = 2; w = u - 2 * kv_units; }
        const int H = part == 2 ? p.Hq : p.Hkv;
        const int j = (int)(w % upr) * 8;
        const int64_t th = w / upr;  // token * H + head
        const int64_t t = th / H;
        const float* src = (part == 0 ? p.k : part == 1 ? p.v : p.q_in) + th * D;
        float x1[8], x2[8];
        load8(src + j, x1);
        load8(src + half + j, x2);
        if (ROPE && part != 1) {
            int32_t pos = p.pos[t];
            if ((uint64_t)pos >= (uint64_t)p.rope_cap) {
                flag_error(p.err, kErrBounds);
                continue;
            }
            float2 cs[8];
            const float4* row = reinterpret_cast<const float4*>(p.rope + (int64_t)pos * half + j);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                float4 c = __ldg(row + i);
                cs[2 * i] = make_float2(c.x, c.y);
                cs[2 * i + 1] = make_float2(c.z, c.w);
            }
            rotate8(x1, x2, cs);
        }
        if (part == 2) {
            float* dst = p.q_out + th * D;
            store8<float>(dst + j, x1);
            store8<float>(dst + half + j, x2);
            continue;
        }
        int32_t slot = p.slots[t];
        if ((uint64_t)slot >= (uint64_t)p.num_slots) {
            flag_error(p.err, kErrBounds);
            continue;
        }
        T* dst = reinterpret_cast<T*>(part == 0 ? p.kpool : p.vpool) + ((int64_t)slot * p.Hkv + (th % H)) * D;
        store8<T>(dst + j, x1);
        store8<T>(dst + half + j, x2);
    }
}

// Element-wise fallback for head dims that are not a multiple of 16 or
// unaligned inputs (the reference's own tests use head_dim 1 and 2).
template <typename T, bool ROPE>
__global__ void append_scalar_kernel(const AppendParams p) {
    pdl_enter();
    const int D = p.D, half = D / 2;
    const int64_t kv_elems = p.n * p.Hkv * D;
    const int64_t q_elems = (ROPE && p.q_in) ? p.n * p.Hq * D : 0;
    const int64_t total = 2 * kv_elems + q_elems;
    for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < total; u += (int64_t)gridDim.x * blockDim.x) {
        int part;
        int64_t w;
        if (u < kv_elems) { part = 0; w = u; }
        else if (u < 2 * kv_elems) { part = 1; w = u - kv_elems; }
        else { part = 2; w = u - 2 * kv_elems; }
        const int H = part == 2 ? p.Hq : p.Hkv;
        const int d = (int)(w % D);
        const int64_t th = w / D;
        const int64_t t = th / H;
        const float* src = (part == 0 ? p.k : part == 1 ? p.v : p.q_in) + th * D;
        float y = src[d];
        if (ROPE && part != 1) {
            int32_t pos = p.pos[t];
            if ((uint64_t)pos >= (uint64_t)p.rope_cap) {
                flag_error(p.err, kErrBounds);
                continue;
            }
            int jj = d < half ? d : d - half;
            float2 cs = p.rope[(int64_t)pos * half + jj];
            float x1 = src[jj], x2 = src[jj + half];
            y = d < half ? __fsub_rn(__fmul_rn(x1, cs.x), __fmul_rn(x2, cs.y))
                         : __fadd_rn(__fmul_rn(x2, cs.x), __fmul_rn(x1, cs.y));
        }
        if (part == 2) {
            p.q_out[th * D + d] = y;
            continue;
        }
        int32_t slot = p.slots[t];
        if ((uint64_t)slot >= (uint64_t)p.num_slots) {
            flag_error(p.err, kErrBounds);
            continue;
        }
        int64_t idx = ((int64_t)slot * p.Hkv + (th % H)) * D + d;
        if constexpr (sizeof(T) == 4) reinterpret_cast<float*>(part == 0 ? p.kpool : p.vpool)[idx] = y;
        else reinterpret_cast<uint16_t*>(part == 0 ? p.kpool : p.vpool)[idx] = f32_to_bf16(y);
    }
}

static bool aligned16(const void* ptr) { return ((uintptr_t)ptr & 15) == 0; }

int launch_append(const AppendParams& p, int dtype, bool rope, cudaStream_t stream, bool pdl) {
    if (p.n <= 0) return S1KV_OK;
    if (rope && (p.D % 2)) return set_error(S1KV_EINVAL, "RoPE needs an even head_dim");
    bool vec = (p.D % 16 == 0) && aligned16(p.k) && aligned16(p.v) && (!p.q_in || (aligned16(p.q_in) && aligned16(p.q_out)));
    int64_t units = vec ? (2 * p.n * p.Hkv + (rope && p.q_in ? p.n * p.Hq : 0)) * (p.D / 16)
                        : (2 * p.n * p.Hkv + (rope && p.q_in ? p.n * p.Hq : 0)) * p.D;
    int grid = (int)std::max<int64_t>(1, std::min<int64_t>((units + 255) / 256, kSMs * 16));
#define S1KV_APPEND(T, R)                                                                                    \
    do {                                                                                                     \
        if (pdl)                                                                                             \
            S1KV_CUDA(vec ? launch_pdl(append_vec_kernel<T, R>, dim3(grid), dim3(256), 0, stream, p)            \
                          : launch_pdl(append_scalar_kernel<T, R>, dim3(grid), dim3(256), 0, stream, p));       \
        else if (vec)                                                                                        \
            append_vec_kernel<T, R><<<grid, 256, 0, stream>>>(p);                                            \
        else                                                                                                 \
            append_scalar_kernel<T, R><<<grid, 256, 0, stream>>>(p);                                         \
    } while (0)
    if (dtype == S1KV_DTYPE_F32) {
        if (rope) S1KV_APPEND(float, true);
        else S1KV_APPEND(float, false);
    } else {
        if (rope) S1KV_APPEND(uint16_t, true);
        else S1KV_APPEND(uint16_t, false);
    }
#undef S1KV_APPEND
    g_launches++;
    S1KV_CUDA(cudaGetLastError());
    return S1KV_OK;
}

// ------------------------------------------- q/k RMSNorm + RoPE + append --
// x / d correctly rounded from r = RN(1 / d), for many x over one d:
// Markstein's FMA correction (P. Markstein, IBM J. Res. Dev. 34(1), 1990;
// Muller et al., Handbook of Floating-Point Arithmetic, division by FMA):
// q0 = RN(x r), the residual e = x - q0 d is exact in one FMA, and
// RN(q0 + e r) is the correctly rounded quotient.  e == 0 keeps q0 (exact
// quotients, and the sign of a zero x).  Checked against __fdiv_rn by
// s1kv_debug_div_check on millions of inputs.
__device__ __forceinline__ float div_by(float x, float d, float r) {
    const float q0 = __fmul_rn(x, r);
    const float e = __fmaf_rn(-q0, d, x);
    return e == 0.0f ? q0 : __fmaf_rn(e, r, q0);
}


// The projection outputs of one step straight into the cache
// (src/nn/attention.cpp:316-322): q and k rows are RMS-normalised with their
// weights (src/nn/rmsnorm.cpp:4-33: squares summed in order, sqrt(sum / D +
// eps), x / rms * w, each operation rounded separately as in the reference's
// build), rotated (RoPE), k written to its slot, q to q_out; v rows are
// copied to their slots.  One thread per (token, head) row keeps the
// reference's summation order, so the results are bit-exact.
template <typename T, int D>
__global__ void __launch_bounds__(256) norm_rope_append_kernel(const AppendParams p, const float* __restrict__ qw,
                                                               const float* __restrict__ kw, float eps,
                                                               const int32_t* __restrict__ qpos, int64_t n_q_rows) {
    // Each warp moves RG = 16 consecutive rows of one part (q, k or v)
    // through a shared tile: asynchronous 16-byte copies (the whole tile in
    // flight at once); lane r < 16 sums the squares of row r in order (the
    // reference's sequential sum), then lanes r and r + 16 normalise, weight
    // and rotate one half of row r's pairs each, in place, and the warp
    // stores the tile with coalesced vector stores.  Tile rows are D + 4
    // floats apart: 16-byte aligned, and the lanes' float4 row accesses take
    // the minimum number of shared-memory wavefronts.  Eight warps of 16 rows
    // (3 CTAs, 24 warps per SM) hide the copies' latency better than four of
    // 32 rows (cfg3 step, 74.8K tokens: 0.70 ms against 0.89 ms).
    constexpr int half = D / 2, RS = D + 4, C4 = D / 4;
    extern __shared__ __align__(16) float tile_all[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int RG = 16;
    float* tile = tile_all + warp * RG * RS;
    const int64_t nq = p.q_in ? n_q_rows * p.Hq : 0, nk = p.n * p.Hkv;
    const int64_t gq = (nq + RG - 1) / RG, gk = (nk + RG - 1) / RG;
    const int64_t groups = gq + 2 * gk;
    const int64_t wid = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp, nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t gi = wid; gi < groups; gi += nwarps) {
        int part;  // 0 = q, 1 = k, 2 = v
        int64_t r0, nrows;
        if (gi < gq) { part = 0; r0 = gi * RG; nrows = nq; }
        else if (gi < gq + gk) { part = 1; r0 = (gi - gq) * RG; nrows = nk; }
        else { part = 2; r0 = (gi - gq - gk) * RG; nrows = nk; }
        const int nr = (int)(nrows - r0 < RG ? nrows - r0 : RG);
        const int H = part == 0 ? p.Hq : p.Hkv;
        const float* src = (part == 0 ? p.q_in : part == 1 ? p.k : p.v) + r0 * D;
        for (int idx = lane; idx < nr * C4; idx += 32)
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                             (uint32_t)__cvta_generic_to_shared(tile + (idx / C4) * RS + (idx % C4) * 4)),
                         "l"(src + (int64_t)idx * 4)
                         : "memory");
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncwarp();
        if (part != 2) {
            // pass 1: lane r < RG sums the squares of row r in order
            float rms = 1.0f, rrms = 1.0f;
            if (lane < nr) {
                const float* rw = tile + lane * RS;
                float sum = 0.0f;
#pragma unroll 8
                for (int j = 0; j < D; j += 4) {
                    const float4 a = *reinterpret_cast<const float4*>(rw + j);
                    sum = __fadd_rn(sum, __fmul_rn(a.x, a.x));
                    sum = __fadd_rn(sum, __fmul_rn(a.y, a.y));
                    sum = __fadd_rn(sum, __fmul_rn(a.z, a.z));
                    sum = __fadd_rn(sum, __fmul_rn(a.w, a.w));
                }
                rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)D), eps));
                rrms = __frcp_rn(rms);
            }
            // pass 2: LPR lanes per row, each a contiguous share of its pairs
            // (the same operations on every element as one lane would do)
            constexpr int LPR = 32 / RG, PPL = half / LPR;
            const int rr = lane % RG, share = lane / RG;
            rms = __shfl_sync(0xffffffffu, rms, rr);
            rrms = __shfl_sync(0xffffffffu, rrms, rr);
            if (rr < nr) {
                float* row = tile + rr * RS;
                const int64_t t = (r0 + rr) / H;
                const float* w = part == 0 ? qw : kw;
                const int32_t pos = part == 0 ? qpos[t] : p.pos[t];
                if ((uint64_t)pos >= (uint64_t)p.rope_cap) {
                    if (share == 0) flag_error(p.err, kErrBounds);
                } else {
                    const float2* cs = p.rope + (int64_t)pos * half;
#pragma unroll 2
                    for (int j = share * PPL; j < (share + 1) * PPL; j += 4) {
                        const float4 l4 = *reinterpret_cast<const float4*>(row + j);
                        const float4 h4 = *reinterpret_cast<const float4*>(row + j + half);
                        const float lo[4] = {l4.x, l4.y, l4.z, l4.w}, hi[4] = {h4.x, h4.y, h4.z, h4.w};
                        float ro[4], rh[4];
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const float2 c = __ldg(cs + j + e);
                            const float x1 = __fmul_rn(div_by(lo[e], rms, rrms), __ldg(w + j + e));
                            const float x2 = __fmul_rn(div_by(hi[e], rms, rrms), __ldg(w + j + e + half));
                            ro[e] = __fsub_rn(__fmul_rn(x1, c.x), __fmul_rn(x2, c.y));
                            rh[e] = __fadd_rn(__fmul_rn(x2, c.x), __fmul_rn(x1, c.y));
                        }
                        *reinterpret_cast<float4*>(row + j) = make_float4(ro[0], ro[1], ro[2], ro[3]);
                        *reinterpret_cast<float4*>(row + j + half) = make_float4(rh[0], rh[1], rh[2], rh[3]);
                    }
                }
            }
        }
        __syncwarp();
        if (part == 0) {
            float* dst = p.q_out + r0 * D;
            for (int idx = lane; idx < nr * C4; idx += 32)
                *reinterpret_cast<float4*>(dst + (int64_t)idx * 4) =
                    *reinterpret_cast<const float4*>(tile + (idx / C4) * RS + (idx % C4) * 4);
        } else {
            // four elements per lane: 8-byte (bf16) or 16-byte stores; lane i
            // looks up row i's slot once and the warp shares it by shuffle
            const int32_t my_slot = lane < nr ? p.slots[(r0 + lane) / H] : 0;
            for (int base = 0; base < nr * C4; base += 32) {  // warp-uniform trip count (shuffle inside)
                const int idx = base + lane;
                const int r = min(idx / C4, nr - 1), c = (idx % C4) * 4;
                const int32_t slot = __shfl_sync(0xffffffffu, my_slot, r);
                if (idx >= nr * C4) continue;
                const int64_t th = r0 + r;
                if ((uint64_t)slot >= (uint64_t)p.num_slots) {
                    flag_error(p.err, kErrBounds);
                    continue;
                }
                T* dst = reinterpret_cast<T*>(part == 1 ? p.kpool : p.vpool) + ((int64_t)slot * p.Hkv + (th % H)) * D + c;
                const float4 a = *reinterpret_cast<const float4*>(tile + r * RS + c);
                if constexpr (sizeof(T) == 4) {
                    *reinterpret_cast<float4*>(dst) = a;
                } else {
                    *reinterpret_cast<uint2*>(dst) = make_uint2((uint32_t)f32_to_bf16(a.x) | ((uint32_t)f32_to_bf16(a.y) << 16),
                                                                (uint32_t)f32_to_bf16(a.z) | ((uint32_t)f32_to_bf16(a.w) << 16));
                }
            }
        }
        __syncwarp();
    }
}

int launch_norm_rope_append(const AppendParams& p, int dtype, const float* qw, const float* kw, float eps,
                            const int32_t* qpos, int64_t n_q_rows, cudaStream_t stream) {
    const int64_t units = (p.q_in ? n_q_rows * p.Hq : 0) + 2 * p.n * p.Hkv;
    if (units <= 0) return S1KV_OK;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((units + 127) / 128, kSMs * 16));
    // 8 warps, each a 16-row tile of head_dim + 4 floats per row
#define S1KV_NRA(T, DD)                                                                                     \
    do {                                                                                                   \
        const int sm = 8 * 16 * (DD + 4) * 4;                                                              \
        S1KV_CUDA(cudaFuncSetAttribute(norm_rope_append_kernel<T, DD>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm)); \
        norm_rope_append_kernel<T, DD><<<grid, 256, sm, stream>>>(p, qw, kw, eps, qpos, n_q_rows);        \
    } while (0)
    if (p.D == 128) {
        if (dtype == S1KV_DTYPE_F32) S1KV_NRA(float, 128);
        else S1KV_NRA(uint16_t, 128);
    } else if (p.D == 64) {
        if (dtype == S1KV_DTYPE_F32) S1KV_NRA(float, 64);
        else S1KV_NRA(uint16_t, 64);
    } else {
        return set_error(S1KV_EINVAL, "norm_rope_append: head_dim %d (64 or 128 supported)", p.D);
    }
#undef S1KV_NRA
    g_launches++;
    S1KV_CUDA(cudaGetLastError());
    return S1KV_OK;
}

// ------------------------------------------------------- standalone RoPE --
__global__ void rope_kernel(const float* __restrict__ x, float* __restrict__ out, const float2* __restrict__ tab,
                            int64_t cap, int64_t start_pos, const int32_t* __restrict__ pos_of, int64_t n, int H, int D,
                            int* err) {
    const int half = D / 2;
    const int64_t total = n * H * half;
    for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < total; u += (int64_t)gridDim.x * blockDim.x) {
        int j = (int)(u % half);
        int64_t th = u / half;
        int64_t pos = pos_of ? (int64_t)pos_of[th / H] : start_pos + th / H;
        if (pos >= cap) {
            flag_error(err, kErrBounds);
            continue;
        }
        float2 cs = tab[pos * half + j];
        float x1 = x[th * D + j], x2 = x[th * D + j + half];
        out[th * D + j] = __fsub_rn(__fmul_rn(x1, cs.x), __fmul_rn(x2, cs.y));
        out[th * D + j + half] = __fadd_rn(__fmul_rn(x2, cs.x), __fmul_rn(x1, cs.y));
    }
}

int launch_rope(const float* x, float* out, const float2* table, int64_t cap, int64_t start_pos, int64_t n, int32_t H,
                int32_t D, int* err, cudaStream_t stream, const int32_t* pos) {
    int64_t total = n * H * (D / 2);
    if (total <= 0) return S1KV_OK;
    int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, kSMs * 16));
    rope_kernel<<<grid, 256, 0, stream>>>(x, out, table, cap, start_pos, pos, n, H, D, err);
    g_launches++;
    S1KV_CUDA(cudaGetLastError());
    return S1KV_OK;
}

// ---------------------------------------------------------------- gather --
// get_k / get_v (kv_block_pool.cpp:67-132): token i of the sequence is read
// from slot table[i / bs] * bs + i % bs and widened to fp32.
template <typename T>
__global__ void gather_kernel(const T* __restrict__ pool, const int32_t* __restrict__ trow, int64_t len, int bs,
                              int row_elems, int32_t max_blocks, float* __restrict__ out, int* err) {
    const int64_t total = len * row_elems;
    for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < total; u += (int64_t)gridDim.x * blockDim.x) {
        int64_t i = u / row_elems;
        int e = (int)(u % row_elems);
        int32_t b = trow[i / bs];
        if ((uint32_t)b >= (uint32_t)max_blocks) {
            flag_error(err, kErrBounds);
            out[u] = 0.0f;
            continue;
        }
        int64_t src = ((int64_t)b * bs + i % bs) * row_elems + e;
        if constexpr (sizeof(T) == 4) out[u] = reinterpret_cast<const float*>(pool)[src];
        else out[u] = bf16_to_f32(reinterpret_cast<const uint16_t*>(pool)[src]);
    }
}

int launch_gather(s1kv_pool* p, int32_t layer, int32_t row, int64_t len, int which, float* out, cudaStream_t stream) {
    if (len <= 0) return S1KV_OK;
    const char* base = (which ? p->v : p->k) + (size_t)layer * p->layer_bytes;
    const int32_t* trow = p->d_table + (int64_t)row * p->max_bps;
    int row_elems = p->desc.num_kv_heads * p->desc.head_dim;
    int64_t total = len * row_elems;
    int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, kSMs * 16));
    if (p->desc.dtype == S1KV_DTYPE_F32)
        gather_kernel<float><<<grid, 256, 0, stream>>>((const float*)base, trow, len, p->desc.block_size, row_elems,
                                                      (int32_t)p->desc.max_blocks, out, p->d_err);
    else
        gather_kernel<uint16_t><<<grid, 256, 0, stream>>>((const uint16_t*)base, trow, len, p->desc.block_size,
                                                         row_elems, (int32_t)p->desc.max_blocks, out, p->d_err);
    g_launches++;
    S1KV_CUDA(cudaGetLastError());
    return S1KV_OK;
}

}  // namespace s1kv

// ----------------------------------------------------------- self-check --
namespace s1kv {
// Counts the (x, d) pairs on which div_by differs from __fdiv_rn: x from
// xs, d from ds (all pairs), result added to *mismatch (device).
__global__ void div_check_kernel(const float* xs, int64_t nx, const float* ds, int64_t nd, unsigned long long* mismatch) {
    const int64_t total = nx * nd;
    unsigned long long bad = 0;
    for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < total; u += (int64_t)gridDim.x * blockDim.x) {
        const float x = xs[u % nx], d = ds[u / nx];
        if (__float_as_uint(div_by(x, d, __frcp_rn(d))) != __float_as_uint(__fdiv_rn(x, d))) bad++;
    }
    if (bad) atomicAdd(mismatch, bad);
}
}  // namespace s1kv

extern "C" int s1kv_debug_div_check(const float* xs, int64_t nx, const float* ds, int64_t nd,
                                   unsigned long long* mismatch, void* stream) {
    s1kv::div_check_kernel<<<148 * 8, 256, 0, (cudaStream_t)stream>>>(xs, nx, ds, nd, mismatch);
    return cudaGetLastError() == cudaSuccess ? S1KV_OK : S1KV_ECUDA;
}
