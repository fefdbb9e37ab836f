// int8_gemv.cu -- int8 weight projections: row quantization and the int8
// GEMV / skinny GEMM either side of the KV path (q/k/v projections before
// the append, o_proj after the attention, the MLP and the LM head).
//
// Reference: src/quantized_tensor.cpp.  quantize_tensor (:9-47) gives every
// ROW k of a [K, N] (pre-transposed, model.cpp:8-33) weight its own scale
// max|w[k,:]| / 127 (1 for an all-zero row) and stores round(w / scale) as
// int8; matmul_quantized (:102-122, kernel :60-100) computes
// out[i, j] = sum_k x[i, k] * (q[k, j] * scale[k]) in fp32, k in order.
//
// B200 layout and schedule:
//   * q [K][N] int8 row-major, scales [K] fp32, x [M][K], out [M][N] fp32:
//     the reference's own layout, so its QuantizedTensor uploads unchanged.
//   * A CTA (8 warps) owns 128-512 output columns and a range of K rows,
//     the warps stacked along K; each lane 4, 8 or 16 columns (one 4-, 8- or
//     16-byte load per row).  Wide row segments stream best (the rows of a
//     tile are N bytes apart), narrow ones give small matrices enough CTAs
//     (gemv_shape).  A warp issues the loads of 32 words per lane (8-32
//     rows) back to back, with no branch between them, before using any.
//   * x * scale is staged in shared memory once per CTA.  int8 -> float
//     without the conversion unit: the byte (biased to unsigned) is placed
//     in the mantissa of 2^23 with a byte permute and 2^23 + 128 is
//     subtracted (exact); then packed FMAs (f32x2) accumulate.
//   * K is split over the CTAs of one thread-block cluster (up to 16) and the
//     8 warps of each: warp partials are summed in shared memory, then CTA
//     rank r of the cluster sums every rank's partial for its share of the
//     columns through distributed shared memory, in rank order.  One launch,
//     no workspace, no atomics, the same result on every run.
//   * Launched as a programmatic dependent launch: weights and scales never
//     depend on the previous kernel, so a CTA requests its first weights and
//     its scales, lets the next grid launch, and only then waits for the
//     previous grid (griddepcontrol.wait) before reading x.  Back-to-back
//     projections overlap their launch and weight latency.
//   * The sum over k is not in the reference's sequential order: results
//     agree to within 2e-5 of the output scale (fp32), not bit for bit.
//     Quantization is bit-exact (IEEE division, round half away from zero).
#include <cooperative_groups.h>

#include <algorithm>

#include "internal.h"

namespace cg = cooperative_groups;

namespace s1kv {
namespace {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kMaxRowsCta = 512;  // K rows per CTA at most (x staging)
constexpr int kMaxCluster = 16;
// shared memory of the largest launch: x staging + warp partials + CTA partial
// (largest MB x NC is 1024: 2 x 512, 4 x 256 or 8 x 128)
constexpr int kGemvSmemMax = 4 * (8 * kMaxRowsCta + (kGemvWarps + 1) * 1024);

// CPL columns per lane (4, 8 or 16: one 4-, 8- or 16-byte load per weight
// row, 128-512 contiguous bytes per warp); MB x CPL accumulators at most 32
// float2.  A warp issues the loads of CHUNK rows before using any: 32 words
// of loaded weights per lane whatever CPL is.
template <int MB, int CPL>
struct GemvTile {
    static_assert(MB * CPL <= 64 && (CPL == 4 || CPL == 8 || CPL == 16), "tile");
    static constexpr int NC = 32 * CPL;       // columns per CTA
    static constexpr int CHUNK = 128 / CPL;   // rows loaded together
};

// The CPL int8 values at row[c..c+CPL) as 32-bit words: one CPL-byte load
// (aligned, all columns inside the row), no branch, so the loads of a chunk
// issue back to back.
template <int CPL>
__device__ __forceinline__ void load_vec(const int8_t* p, uint32_t (&w)[CPL / 4]) {
    if constexpr (CPL == 16) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
        w[0] = v.x, w[1] = v.y, w[2] = v.z, w[3] = v.w;
    } else if constexpr (CPL == 8) {
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
        w[0] = v.x, w[1] = v.y;
    } else {
        w[0] = __ldg(reinterpret_cast<const uint32_t*>(p));
    }
}
// The same by bytes, zero past column N (a ragged last tile or an unaligned
// matrix).
template <int CPL>
__device__ __forceinline__ void load_bytes(const int8_t* row, int c, int N, uint32_t (&w)[CPL / 4]) {
#pragma unroll
    for (int i = 0; i < CPL / 4; i++) {
        uint32_t v = 0;
#pragma unroll
        for (int b = 0; b < 4; b++) {
            const int cc = c + 4 * i + b;
            v |= (cc < N ? (uint32_t)(uint8_t)__ldg(row + cc) : 0u) << (8 * b);
        }
        w[i] = v;
    }
}

// Up to kMaxGroup products sharing x and K (q/k/v; gate/up) in one launch:
// the grid's x dimension runs over every matrix's column tiles, matrix i
// starting at tile `tile0`.
constexpr int kMaxGroup = 4;
struct GemvMat {
    const int8_t* q;
    const float* scales;
    float* out;
    int N, tile0, vec_loads;
};
struct GemvGroup {
    GemvMat m[kMaxGroup];
    int n;
};

template <int MB, int CPL>
__global__ void __launch_bounds__(kGemvThreads, 1) matmul_int8_kernel(const float* __restrict__ x, int M, int K,
                                                                    const __grid_constant__ GemvGroup grp,
                                                                    int rows_per_cta) {
    constexpr int NC = GemvTile<MB, CPL>::NC, kChunk = GemvTile<MB, CPL>::CHUNK;
    extern __shared__ float gemv_smem[];
    float* xs = gemv_smem;                   // [MB][rows_per_cta]: x * scale
    float* red = xs + MB * rows_per_cta;     // [warps][MB][NC]
    float* part = red + kGemvWarps * MB * NC;  // [MB][NC]: this CTA's partial
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int mi = 0;  // this CTA's matrix (uniform)
#pragma unroll
    for (int i = 1; i < kMaxGroup; i++)
        if (i < grp.n && (int)blockIdx.x >= grp.m[i].tile0) mi = i;
    const int8_t* __restrict__ q = grp.m[mi].q;
    const float* __restrict__ scales = grp.m[mi].scales;
    float* __restrict__ out = grp.m[mi].out;
    const int N = grp.m[mi].N, vec_loads = grp.m[mi].vec_loads;
    const int n0 = ((int)blockIdx.x - grp.m[mi].tile0) * NC;
    const int m0 = blockIdx.z * MB;
    const int k0 = blockIdx.y * rows_per_cta;
    const int k_end = min(K, k0 + rows_per_cta);
    const int rows_per_warp = rows_per_cta / kGemvWarps;
    // a split over K reduces through the cluster's shared memory: announce
    // that this CTA has started (waited for before the first remote store)
    if (gridDim.y > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");

    const int c = n0 + CPL * lane;  // this lane's columns [c, c + CPL)
    const int wr0 = warp * rows_per_warp;
    uint32_t w[kChunk][CPL / 4];
    // Rows past K read row K - 1 (its staged x is 0); a lane whose columns
    // all lie inside the row loads them in one piece.
    const bool lane_vec = vec_loads && c + CPL <= N;
    auto load_chunk = [&](int r) {
        if (lane_vec) {
#pragma unroll
            for (int i = 0; i < kChunk; i++)
                load_vec<CPL>(q + (size_t)min(k0 + wr0 + r + i, K - 1) * N + c, w[i]);
        } else {
#pragma unroll
            for (int i = 0; i < kChunk; i++) {
                if (c < N) load_bytes<CPL>(q + (size_t)min(k0 + wr0 + r + i, K - 1) * N, c, N, w[i]);
                else
#pragma unroll
                    for (int j = 0; j < CPL / 4; j++) w[i][j] = 0u;
            }
        }
    };
    // The weights and scales do not depend on the kernel before this one in
    // the stream: the first chunk is requested before waiting for it
    // (programmatic dependent launch; without one the wait returns at once).
    load_chunk(0);
    static_assert(kMaxRowsCta <= 2 * kGemvThreads, "two staged rows per thread");
    const int ka = k0 + tid, kb = k0 + tid + kGemvThreads;  // this thread's staged rows
    const float sa = tid < rows_per_cta && ka < K ? __ldg(scales + ka) : 0.0f;
    const float sb = tid + kGemvThreads < rows_per_cta && kb < K ? __ldg(scales + kb) : 0.0f;
    // The next grid may launch as soon as every CTA of this one has got this
    // far (all of them resident), and request its own weights while this one
    // runs; it still waits for this grid to finish before reading its x.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // x (written by the previous kernel) times the scale, 0 past K or M
#pragma unroll
    for (int m = 0; m < MB; m++) {
        const bool row_ok = m0 + m < M;
        if (tid < rows_per_cta) xs[m * rows_per_cta + tid] = row_ok && ka < K ? x[(size_t)(m0 + m) * K + ka] * sa : 0.0f;
        if (tid + kGemvThreads < rows_per_cta)
            xs[m * rows_per_cta + tid + kGemvThreads] = row_ok && kb < K ? x[(size_t)(m0 + m) * K + kb] * sb : 0.0f;
    }
    __syncthreads();

    float2 acc[MB][CPL / 2];
#pragma unroll
    for (int m = 0; m < MB; m++)
#pragma unroll
        for (int j = 0; j < CPL / 2; j++) acc[m][j] = make_float2(0.0f, 0.0f);
    const float2 bias = make_float2(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
    for (int r = 0; r < rows_per_warp; r += kChunk) {
        if (r > 0) load_chunk(r);
#pragma unroll
        for (int i = 0; i < kChunk; i++) {
            if (r + i >= rows_per_warp) break;
            const int kk = wr0 + r + i;
            float a[MB];
#pragma unroll
            for (int m = 0; m < MB; m++) a[m] = xs[m * rows_per_cta + kk];
#pragma unroll
            for (int j = 0; j < CPL / 4; j++) {
                // four int8 values, exact: bias each byte to unsigned u, then
                // 2^23 + u - (2^23 + 128)
                const uint32_t u = w[i][j] ^ 0x80808080u;
                const float2 lo = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440u)),
                                                         __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441u))),
                                             bias);
                const float2 hi = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442u)),
                                                         __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443u))),
                                             bias);
#pragma unroll
                for (int m = 0; m < MB; m++) {
                    acc[m][2 * j] = __ffma2_rn(make_float2(a[m], a[m]), lo, acc[m][2 * j]);
                    acc[m][2 * j + 1] = __ffma2_rn(make_float2(a[m], a[m]), hi, acc[m][2 * j + 1]);
                }
            }
        }
    }
#pragma unroll
    for (int m = 0; m < MB; m++)
#pragma unroll
        for (int j = 0; j < CPL / 2; j++)
            *reinterpret_cast<float2*>(&red[(warp * MB + m) * NC + CPL * lane + 2 * j]) = acc[m][j];
    __syncthreads();
    if (gridDim.y == 1) {
        for (int i = tid; i < MB * NC; i += kGemvThreads) {
            float s = red[i];
#pragma unroll
            for (int wi = 1; wi < kGemvWarps; wi++) s += red[wi * MB * NC + i];
            const int m = i / NC, cc = i % NC;
            if (m0 + m < M && n0 + cc < N) out[(size_t)(m0 + m) * N + n0 + cc] = s;
        }
        return;
    }
    // K split over the cluster.  Rank o owns columns [o * per, (o + 1) * per);
    // every rank stores its partial of those columns into slot `rank` of the
    // owner's buffer (distributed shared memory: remote stores pipeline, remote
    // loads would not), one release/acquire cluster barrier makes them
    // visible, and each owner sums its slots in rank order.  Every peer has
    // started (the arrive at entry) before the first remote store, and after
    // the barrier no CTA touches another's memory, so CTAs exit freely.
    cg::cluster_group cluster = cg::this_cluster();
    const int cs = (int)cluster.num_blocks(), rank = (int)cluster.block_rank();
    const int per = NC / cs;
    float* recv = part;  // [cs][MB][per]
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // peers started
    for (int i = tid; i < MB * NC; i += kGemvThreads) {
        float s = red[i];
#pragma unroll
        for (int wi = 1; wi < kGemvWarps; wi++) s += red[wi * MB * NC + i];
        const int m = i / NC, cc = i % NC, owner = cc / per;
        cluster.map_shared_rank(recv, owner)[(rank * MB + m) * per + cc % per] = s;
    }
    cluster.sync();
    for (int i = tid; i < MB * per; i += kGemvThreads) {
        const int m = i / per, cl = i % per, cc = rank * per + cl;
        float s = recv[m * per + cl];
        for (int rr = 1; rr < cs; rr++) s += recv[(rr * MB + m) * per + cl];
        if (m0 + m < M && n0 + cc < N) out[(size_t)(m0 + m) * N + n0 + cc] = s;
    }
}

// One warp per row: scale = max|row| / 127 (1 for an all-zero row), then
// q = round(w / scale), ties away from zero (std::round), IEEE division.
__global__ void quantize_rows_kernel(const float* __restrict__ w, int64_t rows, int64_t cols, int8_t* __restrict__ q,
                                     float* __restrict__ scales) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* src = w + row * cols;
    float mx = 0.0f;
    for (int64_t c = lane; c < cols; c += 32) mx = fmaxf(mx, fabsf(src[c]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float scale = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 1.0f;
    if (lane == 0) scales[row] = scale;
    int8_t* dst = q + row * cols;
    for (int64_t c = lane; c < cols; c += 32) dst[c] = (int8_t)(int)roundf(__fdiv_rn(src[c], scale));
}

struct GemvShape {
    int mb, cpl, cs, rows_per_cta, z;
    size_t smem;
};

template <int MB, int CPL>
int launch_gemv(const float* x, int M, int K, GemvGroup grp, const GemvShape& g, cudaStream_t stream) {
    auto kern = matmul_int8_kernel<MB, CPL>;
    static std::atomic<uint64_t> attrs_set{0};  // per device
    int st = once_per_device(attrs_set, [&] {
        S1KV_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        S1KV_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvSmemMax));
        return S1KV_OK;
    });
    if (st) return st;
    int tiles = 0;
    for (int i = 0; i < grp.n; i++) {
        GemvMat& m = grp.m[i];
        m.vec_loads = (m.N % CPL == 0) && ((reinterpret_cast<uintptr_t>(m.q) % CPL) == 0);
        m.tile0 = tiles;
        tiles += (m.N + 32 * CPL - 1) / (32 * CPL);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)tiles, (unsigned)g.cs, (unsigned)g.z);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = g.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = (unsigned)g.cs;
    attr[0].val.clusterDim.z = 1;
    // programmatic dependent launch: this grid may start while the previous
    // kernel of the stream finishes; it waits for it (griddepcontrol.wait)
    // before reading x
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    S1KV_CUDA(cudaLaunchKernelEx(&cfg, kern, x, M, K, grp, g.rows_per_cta));
    g_launches++;
    return S1KV_OK;
}

}  // namespace

// Shape of one launch (measured on B200 over the per-layer projections
// and the LM head, one to eight rows of x).
//   * Narrow matrices (N < 16384, the per-layer weights): 4 columns per
//     lane, so that a 1-3 MB matrix spreads over enough CTAs, and the K
//     split (the cluster size) that leaves at most 256 rows per CTA (384
//     with 8 rows of x).
//   * Wide matrices (the LM head): the widest load the rows of x allow (16
//     bytes for up to 2 rows, 8 for 4; 4 rows per slice beat 8 here) and
//     the fewest K splits, at most 512 rows per CTA: long row segments
//     stream best and there are CTAs enough.
static int gemv_shape(int M, int K, int N, int cap, GemvShape* g) {
    const bool wide = N >= 16384;
    g->mb = M >= 8 && !wide ? 8 : M >= 4 ? 4 : M >= 2 ? 2 : 1;
    g->z = (M + g->mb - 1) / g->mb;
    g->cpl = wide ? (g->mb <= 2 ? 16 : 8) : 4;
    const int rows_target = wide ? kMaxRowsCta : g->mb == 8 ? 384 : 256;
    int cs = 1;
    while (cs < cap && (K + cs - 1) / cs > rows_target) cs *= 2;
    while (cs < cap && (K + cs - 1) / cs > kMaxRowsCta) cs *= 2;
    if ((K + cs - 1) / cs > kMaxRowsCta)
        return set_error(S1KV_EINVAL, "matmul_int8: K = %d above %d", K, kMaxRowsCta * cap);
    g->cs = cs;
    const int nc = 32 * g->cpl;
    const int per_cta = (K + cs - 1) / cs;
    g->rows_per_cta = (per_cta + kGemvWarps - 1) / kGemvWarps * kGemvWarps;
    g->smem = sizeof(float) * ((size_t)g->mb * g->rows_per_cta + (size_t)(kGemvWarps + 1) * g->mb * nc);
    return S1KV_OK;
}

// Largest cluster along K this device co-schedules for the kernel: 16 (a
// non-portable size) where the occupancy query allows it, else 8.
static int gemv_cluster_cap(int dev) {
    static std::atomic<int> cap[64];  // 0 = not yet queried
    if (dev < 0 || dev >= 64) return 8;
    if (const int c = cap[dev].load(std::memory_order_acquire)) return c;
    auto kern = matmul_int8_kernel<8, 4>;
    int n = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess &&
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvSmemMax) == cudaSuccess) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(1, kMaxCluster, 1);
        cfg.blockDim = dim3(kGemvThreads);
        cfg.dynamicSmemBytes = kGemvSmemMax;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = kMaxCluster;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
    }
    cudaGetLastError();  // a refused query leaves no error behind
    const int c = n > 0 ? kMaxCluster : 8;
    cap[dev].store(c, std::memory_order_release);
    return c;
}

}  // namespace s1kv

using namespace s1kv;

extern "C" int s1kv_quantize_rows(const float* w, int64_t rows, int64_t cols, int8_t* q, float* scales, void* stream) {
    if (rows < 0 || cols < 0 || (rows > 0 && (!w || !q || !scales)))
        return set_error(S1KV_EINVAL, "quantize_rows: bad arguments");
    if (rows == 0) return S1KV_OK;
    const int warps = 8;
    quantize_rows_kernel<<<(unsigned)((rows + warps - 1) / warps), warps * 32, 0, (cudaStream_t)stream>>>(w, rows, cols, q,
                                                                                                        scales);
    g_launches++;
    S1KV_CUDA(cudaGetLastError());
    return S1KV_OK;
}

static int matmul_int8_group(const float* x, int64_t M, int64_t K, int32_t n, const int8_t* const* q,
                             const float* const* scales, const int64_t* N, float* const* out, cudaStream_t s) {
    if (n < 1 || n > kMaxGroup) return set_error(S1KV_EINVAL, "matmul_int8: 1 to %d matrices per launch", kMaxGroup);
    if (M < 0 || K < 0 || M > (1 << 30) || K > (1 << 30)) return set_error(S1KV_EINVAL, "matmul_int8: bad shape");
    GemvGroup grp = {};
    for (int i = 0; i < n; i++) {
        if (N[i] < 0 || N[i] > (1 << 30)) return set_error(S1KV_EINVAL, "matmul_int8: bad shape");
        if (M > 0 && N[i] > 0 && (!x || !q[i] || !scales[i] || !out[i]))
            return set_error(S1KV_EINVAL, "matmul_int8: null pointer");
        if (N[i] == 0) continue;  // nothing to compute for this one
        grp.m[grp.n].q = q[i];
        grp.m[grp.n].scales = scales[i];
        grp.m[grp.n].out = out[i];
        grp.m[grp.n].N = (int)N[i];
        grp.n++;
    }
    if (M == 0 || grp.n == 0) return S1KV_OK;
    if (K == 0) {
        for (int i = 0; i < grp.n; i++)
            S1KV_CUDA(cudaMemsetAsync(grp.m[i].out, 0, sizeof(float) * (size_t)M * (size_t)grp.m[i].N, s));
        return S1KV_OK;
    }
    int dev = 0;
    S1KV_CUDA(cudaGetDevice(&dev));
    GemvShape g;
    // the shape follows the group's widest matrix (narrow or wide loads)
    int widest = 0;
    for (int i = 0; i < grp.n; i++) widest = std::max(widest, grp.m[i].N);
    int st = gemv_shape((int)M, (int)K, widest, gemv_cluster_cap(dev), &g);
    if (st) return st;
    const int Mi = (int)M, Ki = (int)K;
#define S1KV_GEMV(MB_, CPL_) \
    if (g.mb == MB_ && g.cpl == CPL_) return launch_gemv<MB_, CPL_>(x, Mi, Ki, grp, g, s);
    S1KV_GEMV(1, 4) S1KV_GEMV(1, 8) S1KV_GEMV(1, 16)
    S1KV_GEMV(2, 4) S1KV_GEMV(2, 8) S1KV_GEMV(2, 16)
    S1KV_GEMV(4, 4) S1KV_GEMV(4, 8)
    S1KV_GEMV(8, 4)
#undef S1KV_GEMV
    return set_error(S1KV_EINVAL, "matmul_int8: no kernel for %d rows x %d columns per lane", g.mb, g.cpl);
}

extern "C" int s1kv_matmul_int8(const float* x, int64_t M, int64_t K, const int8_t* q, const float* scales, int64_t N,
                                float* out, void* stream) {
    return matmul_int8_group(x, M, K, 1, &q, &scales, &N, &out, (cudaStream_t)stream);
}

extern "C" int s1kv_matmul_int8_group(const float* x, int64_t M, int64_t K, int32_t n_mats, const int8_t* const* q,
                                      const float* const* scales, const int64_t* N, float* const* out, void* stream) {
    if (!q || !scales || !N || !out) return set_error(S1KV_EINVAL, "matmul_int8_group: null array");
    return matmul_int8_group(x, M, K, n_mats, q, scales, N, out, (cudaStream_t)stream);
}
