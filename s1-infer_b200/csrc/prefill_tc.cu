// prefill_tc.cu -- prefix-hit chunked-prefill attention on tcgen05.
//
// GQA_attention_paged (src/nn/attention.cpp:128-239 of s1-infer) for query
// chunks longer than one token over bf16 K/V: row i of a sequence's q_len
// new tokens attends to tokens 0 .. (kv_len - q_len) + i (:181).  This is a
// dense QK^T / PV contraction, so it runs on the 5th-generation tensor
// cores:
//   * CTA = (sequence, query chunk, kv head).  Its M = 128 accumulator rows
//     are (query, head) pairs: 128/G queries x the G query heads that share
//     the KV head, so every K/V tile feeds all heads of the group.
//   * Q (fp32 in global) is narrowed to bf16 into shared memory in the
//     128-byte-swizzled K-major layout UMMA reads.
//   * K/V tiles of 64 tokens = 4 blocks are fetched through the block table
//     by TMA (one 16-row x 64-element box per block and 128-byte half of a
//     row, 128B swizzle, no multicast), double buffered, completion on
//     mbarriers with bounded waits.
//   * S = Q K^T (M 128, N 64, K 128) and O += P V (M 128, N 128, K 64) are
//     tcgen05.mma kind::f16 with fp32 accumulators in TMEM: S double
//     buffered (2 x 64 columns) so the scores of tile t+1 are computed while
//     the threads run the softmax of tile t; O (128 columns) accumulates
//     across all tiles.  256 columns per CTA, 2 CTAs per SM.  One thread
//     issues; tcgen05.commit signals an mbarrier.
//   * Each thread owns one accumulator row: it reads S with tcgen05.ld,
//     applies the scale and the causal mask, runs the online softmax in the
//     exp2 domain and writes P (bf16) in the swizzled K-major layout for the
//     PV MMA into the current tile's K buffer (free once S is computed).
//     The reference max only moves when the row max outgrows it by 2^8, and
//     only then is the row of O in TMEM rescaled (tcgen05.ld/st), so the
//     common tile does no per-row O work at all.
// Every wait is bounded and decided for the whole CTA at once (a timeout
// sets the device error word); copies in flight are drained and TMEM is
// freed on every exit path.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <cmath>

#include "internal.h"

namespace s1kv {
namespace {

constexpr uint32_t kSpin = 1u << 22;
constexpr int kM = 128;          // accumulator rows per CTA
constexpr int kN = 64;           // tokens per K/V tile
constexpr int kD = 128;          // head dim (two 64-element swizzle atoms)
constexpr int kThreads = 128;    // one thread per accumulator row
constexpr int kTmemCols = 256;   // S[0] [0, 64), S[1] [64, 128), O [128, 256)
constexpr int kTmemS = 0, kTmemO = 128;
constexpr float kRescaleAt = 8.0f;  // log2 units: O is rescaled only when a row max grows by > 2^8

// shared memory layout (bytes, 1024-aligned pieces)
constexpr int kQBytes = 2 * kM * 128;          // 2 atoms x 128 rows x 128 B = 32 KB
constexpr int kKBytes = 2 * kN * 128;          // 2 atoms x 64 rows x 128 B  = 16 KB
constexpr int kVBytes = 2 * kN * 128;          // 2 d-atoms x 64 tokens x 128 B = 16 KB
constexpr int kPBytes = kM * 128;              // 1 atom (64 tokens) x 128 rows x 128 B = 16 KB, in K[buf]
static_assert(kPBytes == kKBytes, "P reuses the tile's K buffer");
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kQBytes;         // K[2] (P of the tile aliases K[tile & 1])
constexpr int kOffV = kOffK + 2 * kKBytes;     // V[2]
constexpr int kOffBar = kOffV + 2 * kVBytes;   // kv[2], s[2], o mbarriers + tmem slot
constexpr int kIdsCached = 256;                // block ids of the first 64 tiles (4096 tokens)
constexpr int kOffIds = kOffBar + 64;
constexpr int kSmem = kOffIds + kIdsCached * 4 + 1024;  // + slack for 1024 alignment of the base

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void bar_init(uint64_t* b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void bar_expect(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool bar_try(uint64_t* b, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(su32(b)), "r"(phase)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t phase) {
    for (uint32_t i = 0; i < kSpin; i++)
        if (bar_try(b, phase)) return true;
    return false;
}
__device__ __forceinline__ void tma4(void* dst, const CUtensorMap* m, uint64_t* b, int c0, int c1, int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];" ::"r"(su32(dst)),
        "l"(m), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(su32(b))
        : "memory");
}

// UMMA shared-memory descriptor, 128-byte swizzle (layout type 2), version 1.
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// kind::f16 instruction descriptor: bf16 A/B, fp32 D, M, N, majors.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, int a_mn_major, int b_mn_major) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn_major << 15) | ((uint32_t)b_mn_major << 16) |
           ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(b))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// Writes 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
        "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
        "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
        "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])),
        "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Byte offset of 16-byte chunk `c` (0..7) of row `r` inside a 128B-swizzled
// atom whose rows are 128 bytes: the chunk index is XORed with r mod 8.
__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

}  // namespace

// Queries per CTA: 128 rows / G heads.
template <int G>
__global__ void __launch_bounds__(kThreads, 2)
    prefill_tc_kernel(const __grid_constant__ PrefillParams p, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV) {
    constexpr int QT = kM / G;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sQ = smem + kOffQ;
    uint8_t* sK = smem + kOffK;
    uint8_t* sV = smem + kOffV;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);  // [0,1] kv, [2,3] s, [4] o
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + 48);

    const int tid = threadIdx.x, warp = tid >> 5;
    const int seq_i = blockIdx.x / p.max_chunks, chunk = blockIdx.x % p.max_chunks;
    const int h = blockIdx.y;
    const PrefillSeq sm = p.seqs[seq_i];
    const int q0 = chunk * QT;
    if (q0 >= sm.q_len) return;  // uniform: no TMEM allocated yet
    const int prefix = sm.kv_len - sm.q_len;
    // tokens the last query of the chunk may see
    const int kv_end = min(sm.kv_len, prefix + q0 + QT);
    const int n_tiles = (kv_end + kN - 1) / kN;

    // This thread's accumulator row: head g, query i of the chunk.
    const int r = tid;
    const int g = r / QT, qi = r % QT;
    const bool row_valid = q0 + qi < sm.q_len;
    const int row_limit = prefix + q0 + qi;  // last visible token

    // ---- set-up: TMEM, barriers ----
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int i = 0; i < 5; i++) bar_init(&bars[i], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // ---- Q: fp32 -> bf16, swizzled K-major ----
    {
        const float* qrow = p.q + ((int64_t)(sm.q_start + min(q0 + qi, sm.q_len - 1)) * p.Hq + h * G + g) * kD;
#pragma unroll 4
        for (int c = 0; c < 16; c++) {  // 16 chunks of 8 elements
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
            if (row_valid) {
                a = __ldg(reinterpret_cast<const float4*>(qrow + c * 8));
                b = __ldg(reinterpret_cast<const float4*>(qrow + c * 8 + 4));
            }
            uint4 w = make_uint4(pack_bf16(a.x, a.y), pack_bf16(a.z, a.w), pack_bf16(b.x, b.y), pack_bf16(b.z, b.w));
            *reinterpret_cast<uint4*>(sQ + (c >> 3) * (kM * 128) + swz(r, c & 7)) = w;
        }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int32_t* tab = p.table + (int64_t)sm.table_row * p.max_bps;

    // Block ids of the chunk's first kIdsCached blocks, looked up once.
    // Blocks past the sequence end are not looked up: a box that starts out
    // of range is zero-filled by TMA.
    int32_t* sIds = reinterpret_cast<int32_t*>(smem + kOffIds);
    auto lookup = [&](int i) -> int32_t {
        if (i * 16 >= sm.kv_len) return p.max_blocks;
        const int32_t blk = tab[i];
        if ((uint32_t)blk >= (uint32_t)p.max_blocks) {
            atomicOr(p.err, kErrBounds);
            return p.max_blocks;
        }
        return blk;
    };
    for (int i = tid; i < min(n_tiles * (kN / 16), kIdsCached); i += kThreads) sIds[i] = lookup(i);
    __syncthreads();

    auto issue_kv = [&](int t) {
        const int buf = t & 1;
        uint8_t* k = sK + buf * kKBytes;
        uint8_t* v = sV + buf * kVBytes;
        bar_expect(&bars[buf], kKBytes + kVBytes);
        for (int b = 0; b < kN / 16; b++) {
            const int i = t * (kN / 16) + b;
            const int32_t blk = i < kIdsCached ? sIds[i] : lookup(i);
            for (int a = 0; a < 2; a++) {
                tma4(k + a * (kN * 128) + b * 16 * 128, &tmK, &bars[buf], a * 64, h, blk * 16, p.layer);
                tma4(v + a * (kN * 128) + b * 16 * 128, &tmV, &bars[buf], a * 64, h, blk * 16, p.layer);
            }
        }
    };
    constexpr uint32_t idS = idesc_bf16(kM, kN, 0, 0);
    constexpr uint32_t idO = idesc_bf16(kM, kD, 0, 1);
    auto issue_s = [&](int t) {  // S[t&1] = Q K(t)^T
        tc_fence_after();
        const uint32_t qa = su32(sQ), ka = su32(sK + (t & 1) * kKBytes);
#pragma unroll
        for (int ks = 0; ks < kD / 16; ks++) {
            const uint32_t off = (ks & 3) * 32;  // 16 elements = 32 bytes inside the 128-byte atom row
            const uint64_t da = sdesc(qa + (ks >> 2) * (kM * 128) + off, 16, 1024);
            const uint64_t db = sdesc(ka + (ks >> 2) * (kN * 128) + off, 16, 1024);
            mma_bf16(tmem + kTmemS + (t & 1) * kN, da, db, idS, ks > 0);
        }
        mma_commit(&bars[2 + (t & 1)]);
    };
    auto issue_pv = [&](int t) {  // O += P(t) V(t); P(t) lives in K(t)'s buffer
        tc_fence_after();
        const uint32_t pa = su32(sK + (t & 1) * kKBytes), va = su32(sV + (t & 1) * kVBytes);
#pragma unroll
        for (int ks = 0; ks < kN / 16; ks++) {
            const uint64_t da = sdesc(pa + ks * 32, 16, 1024);
            const uint64_t db = sdesc(va + ks * 16 * 128, kN * 128, 1024);
            mma_bf16(tmem + kTmemO, da, db, idO, t > 0 || ks > 0);
        }
        mma_commit(&bars[4]);
    };

    // Issue schedule (thread 0): S(t+1) runs on the tensor core while the
    // threads do the softmax of tile t; PV(t) follows; K/V buffer t&1 is
    // refilled with tile t+2 once PV(t) has read P(t) and V(t).
    int kv_issued = 0, kv_waited = 0, s_issued = 0, pv_issued = 0, pv_waited = 0;
    bool issue_ok = true;
    if (tid == 0) {
        issue_kv(0);
        kv_issued = 1;
        if (n_tiles > 1) issue_kv(1), kv_issued = 2;
        issue_ok = bar_wait(&bars[0], 0);
        kv_waited = 1;
        if (issue_ok) issue_s(0), s_issued = 1;
        if (issue_ok && n_tiles > 1) {
            issue_ok = bar_wait(&bars[1], 0);
            kv_waited = 2;
            if (issue_ok) issue_s(1), s_issued = 2;
        }
    }

    float m = -INFINITY;  // running max actually used for p (lags the true max by < 2^8)
    float l = 0.0f;
    bool ok = true;
    int s_waited = 0;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;

    for (int t = 0; t < n_tiles; t++) {
        // 1. scores of tile t (PV(t-1) is complete too: thread 0 waited for it
        //    before arriving here)
        if (!__syncthreads_and(bar_wait(&bars[2 + (t & 1)], (uint32_t)((t >> 1) & 1)))) {
            ok = false;
            break;
        }
        s_waited = t + 1;
        tc_fence_after();
        // 2. online softmax of this row
        float sc[kN];
        tmem_ld32(tmem + lane_base + kTmemS + (t & 1) * kN, sc);
        tmem_ld32(tmem + lane_base + kTmemS + (t & 1) * kN + 32, sc + 32);
        const int base = t * kN;
        float mx = -INFINITY;
        if (base + kN - 1 <= prefix + q0) {  // whole tile visible to every row of the chunk
#pragma unroll
            for (int j = 0; j < kN; j++) {
                sc[j] *= p.scale_log2;
                mx = fmaxf(mx, sc[j]);
            }
        } else {
#pragma unroll
            for (int j = 0; j < kN; j++) {
                sc[j] = (base + j <= row_limit) ? sc[j] * p.scale_log2 : -INFINITY;
                mx = fmaxf(mx, sc[j]);
            }
        }
        // Raise the reference max only when the row max outgrows it by more
        // than 2^8; then O (in TMEM, complete up to tile t-1) and l are
        // rescaled.  Otherwise p = 2^(s - m) <= 2^8 stays well inside fp32
        // and bf16 range and the final O / l is unchanged.
        const bool raise = mx > m + kRescaleAt;
        float corr = 1.0f;
        if (raise) {
            corr = ex2f(m - mx);  // 0 on the first tile (m = -inf)
            m = mx;
            l *= corr;
        }
        if (t > 0 && __any_sync(0xffffffffu, raise)) {
#pragma unroll
            for (int c = 0; c < kD / 32; c++) {
                float ov[32];
                tmem_ld32(tmem + lane_base + kTmemO + c * 32, ov);
#pragma unroll
                for (int j = 0; j < 32; j++) ov[j] *= corr;
                tmem_st32(tmem + lane_base + kTmemO + c * 32, ov);
            }
        }
        const float mref = m == -INFINITY ? 0.0f : m;  // a row with nothing visible yet keeps p = 0
        float ls = 0.0f;
        uint8_t* sP = sK + (t & 1) * kKBytes;
#pragma unroll
        for (int c = 0; c < 8; c++) {
            float pv[8];
#pragma unroll
            for (int e = 0; e < 8; e++) {
                pv[e] = ex2f(sc[c * 8 + e] - mref);
                ls += pv[e];
            }
            uint4 w = make_uint4(pack_bf16(pv[0], pv[1]), pack_bf16(pv[2], pv[3]), pack_bf16(pv[4], pv[5]),
                                 pack_bf16(pv[6], pv[7]));
            *reinterpret_cast<uint4*>(sP + swz(r, c)) = w;
        }
        l += ls;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc_fence_before();
        __syncthreads();
        // 3. issue PV(t); then, once K(t+2)'s buffer is free, the next copy
        //    and the scores two tiles ahead
        if (tid == 0 && issue_ok) {
            issue_pv(t);
            pv_issued = t + 1;
            issue_ok = bar_wait(&bars[4], (uint32_t)(t & 1));
            pv_waited = t + 1;
            if (issue_ok && t + 2 < n_tiles) {
                issue_kv(t + 2);
                kv_issued = t + 3;
                issue_ok = bar_wait(&bars[(t + 2) & 1], (uint32_t)(((t + 2) >> 1) & 1));
                kv_waited = t + 3;
                if (issue_ok) issue_s(t + 2), s_issued = t + 3;
            }
        }
    }

    if (ok) {
        // the last PV was waited for by thread 0; make it visible to all
        ok = __syncthreads_and(issue_ok || tid != 0);
    } else if (tid == 0) {
        // Drain what is still in flight (bounded again) before TMEM and
        // shared memory are released.
        atomicOr(p.err, kErrTimeout);
        for (int i = s_waited; i < s_issued; i++) bar_wait(&bars[2 + (i & 1)], (uint32_t)((i >> 1) & 1));
        for (int i = pv_waited; i < pv_issued; i++) bar_wait(&bars[4], (uint32_t)(i & 1));
        for (int i = kv_waited; i < kv_issued; i++) bar_wait(&bars[i & 1], (uint32_t)((i >> 1) & 1));
    }
    if (ok) {
        tc_fence_after();
        const float inv = 1.0f / l;
        float* orow = p.out + ((int64_t)(sm.q_start + q0 + qi) * p.Hq + h * G + g) * kD;
#pragma unroll
        for (int c = 0; c < kD / 32; c++) {
            float ov[32];
            tmem_ld32(tmem + lane_base + kTmemO + c * 32, ov);
            if (row_valid) {
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<float4*>(orow + c * 32 + j) =
                        make_float4(ov[j] * inv, ov[j + 1] * inv, ov[j + 2] * inv, ov[j + 3] * inv);
            }
        }
    } else if (tid == 0) {
        atomicOr(p.err, kErrTimeout);
    }
    // ---- tear-down: every path frees TMEM ----
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

}  // namespace s1kv

namespace s1kv {

bool prefill_tc_supported(int dtype, int D, int G, int block_size) {
    return dtype == S1KV_DTYPE_BF16 && D == kD && block_size == 16 && (G == 1 || G == 2 || G == 4 || G == 8);
}

template <int G>
static int launch_prefill_g(const PrefillParams& p, const CUtensorMap& tk, const CUtensorMap& tv, cudaStream_t stream) {
    S1KV_CUDA(cudaFuncSetAttribute(prefill_tc_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    dim3 grid((unsigned)(p.n_seqs * p.max_chunks), (unsigned)p.Hkv);
    prefill_tc_kernel<G><<<grid, kThreads, kSmem, stream>>>(p, tk, tv);
    g_launches++;
    S1KV_CUDA(cudaGetLastError());
    return S1KV_OK;
}

int launch_prefill_tc(const PrefillParams& p, const CUtensorMap& tk, const CUtensorMap& tv, cudaStream_t stream) {
    const int G = p.Hq / p.Hkv;
    switch (G) {
        case 1: return launch_prefill_g<1>(p, tk, tv, stream);
        case 2: return launch_prefill_g<2>(p, tk, tv, stream);
        case 4: return launch_prefill_g<4>(p, tk, tv, stream);
        case 8: return launch_prefill_g<8>(p, tk, tv, stream);
        default: return set_error(S1KV_EINVAL, "prefill: unsupported group size %d", G);
    }
}

int prefill_queries_per_cta(int G) { return kM / G; }

}  // namespace s1kv
