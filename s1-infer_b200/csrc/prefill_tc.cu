// prefill_tc.cu -- prefix-hit chunked-prefill attention on tcgen05.
//
// GQA_attention_paged (src/nn/attention.cpp:128-239 of s1-infer) for query
// chunks longer than one token over bf16 K/V: row i of a sequence's q_len
// new tokens attends to tokens 0 .. (kv_len - q_len) + i (:181).  This is a
// dense QK^T / PV contraction, so it runs on the 5th-generation tensor
// cores, warp-specialised:
//   * CTA = (sequence, query chunk, kv head), two query tiles A and B.  The
//     M = 128 accumulator rows of a tile are (query, head) pairs: 128/G
//     queries x the G query heads that share the KV head, so every K/V tile
//     feeds all heads of the group, and both tiles share each K/V tile.
//   * Q (fp32 in global) arrives by TMA, one 128-row box per tile, in the
//     K/V ring before its first use, and is narrowed to bf16 in the
//     128-byte-swizzled K-major layout UMMA reads (rows query-major: row r =
//     query r / G, head r % G).  Finished rows of full chunks leave through
//     swizzled staging and TMA stores; partial chunks store directly.
//   * K/V tiles of 128 tokens = 8 blocks come through the block table by
//     TMA (one 16-row x 64-element box per block and 128-byte half of a
//     row, 128B swizzle, no multicast), issued by 16 lanes of the producer
//     warp in parallel into a 2-stage ring; completion on mbarriers.
//   * The MMA warp (one elected lane) issues S_X = Q_X K^T (M 128, N 128, K 128)
//     and O_X += P_X V (M 128, N 128, K 128, A read from TMEM) as
//     tcgen05.mma kind::f16 with fp32 accumulators in TMEM (512 columns:
//     S_A, S_B, O_A, O_B).  Order PV_A(t) S_A(t+1) PV_B(t) S_B(t+1): a
//     tile's next scores queue behind its PV, and one tile's softmax runs
//     while the other tile's MMAs execute.
//   * Two softmax warpgroups, one per tile; each thread owns one row: it
//     reads its 128 scores with tcgen05.ld, masks the causal edge, runs the
//     online softmax in the exp2 domain and writes P (bf16 pairs) back over
//     the first 64 columns of its S with tcgen05.st, where the PV MMA reads
//     it.  The reference max only moves when the row max outgrows it by
//     2^8, and only then is the row of O in TMEM rescaled, so the common
//     tile does no per-row O work.
// Every wait is bounded; a timeout raises a CTA-wide abort flag that every
// role polls, and the device error word.  Copies in flight are waited for
// (bounded) and TMEM is freed on every exit path.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <cmath>

#include "internal.h"

namespace s1kv {
namespace {

constexpr uint32_t kSpin = 1u << 22;
constexpr int kM = 128;          // accumulator rows per query tile (= TMEM lanes)
constexpr int kN = 128;          // tokens per K/V tile
constexpr int kBlocksPerTile = kN / 16;
constexpr int kD = 128;          // head dim (two 64-element swizzle atoms)
constexpr int kStages = 2;       // K/V ring depth
constexpr int kSoftmaxThreads = 256;  // two warpgroups, one per query tile
constexpr int kThreads = kSoftmaxThreads + 64;  // + TMA warp + MMA warp
constexpr int kTmemCols = 512;   // S_A [0,128) S_B [128,256) O_A [256,384) O_B [384,512)
constexpr int kColO = 256;
constexpr float kRescaleAt = 8.0f;  // log2 units: O is rescaled only when a row max grows by > 2^8
// shared memory layout (bytes, 1024-aligned pieces)
constexpr int kQBytes = 2 * kM * 128;          // one query tile: 2 atoms x 128 rows x 128 B = 32 KB
constexpr int kKBytes = 2 * kN * 128;          // 2 d-atoms x 128 tokens x 128 B = 32 KB
constexpr int kVBytes = 2 * kN * 128;
constexpr int kOffQ = 0;                        // Q_A, Q_B
constexpr int kOffK = kOffQ + 2 * kQBytes;      // K ring
constexpr int kOffV = kOffK + kStages * kKBytes;  // V ring
constexpr int kOffBar = kOffV + kStages * kVBytes;
// barriers: k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2], p_full[2], pv_done[2], drain, q_full,
// p_lo[2]
constexpr int kNumBars = 4 * kStages + 10;
// Q arrives as fp32 by TMA into the (still idle) K/V ring: one box of
// 128 (query, head) rows x 512 bytes per query tile
constexpr int kQStageBytes = kM * kD * 4;
static_assert(2 * kQStageBytes == kStages * (kKBytes + kVBytes), "Q staging must fill the K/V ring exactly");
constexpr int kOffMisc = kOffBar + kNumBars * 8;  // tmem slot, abort flag
constexpr int kIdsCached = 256;                   // block ids of the first 32 tiles (4096 tokens)
constexpr int kOffIds = (kOffMisc + 16 + 15) / 16 * 16;
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
// Non-blocking probe of a phase (mbarrier.test_wait); the waits below try it
// before the potentially suspending try_wait.
__device__ __forceinline__ bool bar_test(uint64_t* b, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
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
__device__ __forceinline__ void bar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ void tma4(void* dst, const CUtensorMap* m, uint64_t* b, int c0, int c1, int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];" ::"r"(su32(dst)),
        "l"(m), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(su32(b))
        : "memory");
}

__device__ __forceinline__ void tma3_load(void* dst, const CUtensorMap* m, uint64_t* b, int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
            su32(dst)),
        "l"(m), "r"(c0), "r"(c1), "r"(c2), "r"(su32(b))
        : "memory");
}
__device__ __forceinline__ void tma3_store(const CUtensorMap* m, uint32_t src, int c0, int c1, int c2) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(m), "r"(c0),
                 "r"(c1), "r"(c2), "r"(src)
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

// MMAs and commits are run by a whole warp, one elected lane issuing: the
// issuing warp stays converged, so its operands never leave the warp-uniform
// path.
// D (TMEM) (+)= A (shared) * B (shared)
__device__ __forceinline__ void mma_ss_w(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}
// D (TMEM) (+)= A (TMEM) * B (shared)
__device__ __forceinline__ void mma_ts_w(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc, bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(b), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}
__device__ __forceinline__ void mma_commit_w(uint64_t* b) {
    asm volatile(
        "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(su32(b))
        : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Loads 32 (or 128) consecutive fp32 columns of this thread's TMEM lane (one
// instruction) and waits for them.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, float* v) {
    uint32_t r[128];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x128.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79,%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95,%96,%97,%98,%99,%100,%101,%102,%103,%104,%105,%106,%107,%108,%109,%110,%111,%112,%113,%114,%115,%116,%117,%118,%119,%120,%121,%122,%123,%124,%125,%126,%127}, [%128];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]),
        "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]),
        "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]),
        "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]),
        "=r"(r[88]), "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]),
        "=r"(r[96]), "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]), "=r"(r[102]), "=r"(r[103]),
        "=r"(r[104]), "=r"(r[105]), "=r"(r[106]), "=r"(r[107]), "=r"(r[108]), "=r"(r[109]), "=r"(r[110]), "=r"(r[111]),
        "=r"(r[112]), "=r"(r[113]), "=r"(r[114]), "=r"(r[115]), "=r"(r[116]), "=r"(r[117]), "=r"(r[118]), "=r"(r[119]),
        "=r"(r[120]), "=r"(r[121]), "=r"(r[122]), "=r"(r[123]), "=r"(r[124]), "=r"(r[125]), "=r"(r[126]), "=r"(r[127])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 128; i++) v[i] = __uint_as_float(r[i]);
}

// Writes 32 (16) consecutive 32-bit columns of this thread's TMEM lane; the
// _nowait form leaves tcgen05.wait::st to the caller.
__device__ __forceinline__ void tmem_st32_nowait(uint32_t taddr, const float* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
        "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}
__device__ __forceinline__ void tmem_st16_nowait(uint32_t taddr, const float* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
        : "memory");
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

// Bounded wait that also gives up when another role of the CTA raised the
// abort flag; a timeout raises it.
__device__ __forceinline__ bool wait_or_abort(uint64_t* b, uint32_t phase, volatile int* abort_flag) {
    if (bar_test(b, phase)) return true;
    for (uint32_t i = 0; i < kSpin; i++) {
        if (bar_try(b, phase)) return true;
        if (*abort_flag) return false;
    }
    *abort_flag = 1;
    return false;
}

// The same, decided for the whole warp: a lane that saw the abort flag takes
// its warp with it (warp-collective tcgen05 instructions follow the waits).
__device__ __forceinline__ bool warp_wait(uint64_t* b, uint32_t phase, volatile int* abort_flag) {
    return __all_sync(0xffffffffu, wait_or_abort(b, phase, abort_flag));
}

}  // namespace

// Queries per query tile: 128 rows / G heads; a CTA takes two tiles.
template <int G>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ PrefillParams p, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmQ,
                      const __grid_constant__ CUtensorMap tmO) {
    constexpr int QT = kM / G;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
    uint64_t* k_full = bars;
    uint64_t* k_empty = bars + kStages;
    uint64_t* v_full = bars + 2 * kStages;
    uint64_t* v_empty = bars + 3 * kStages;
    uint64_t* s_full = bars + 4 * kStages;       // [2]
    uint64_t* p_full = bars + 4 * kStages + 2;   // [2]
    uint64_t* pv_done = bars + 4 * kStages + 4;  // [2]
    uint64_t* drain = bars + 4 * kStages + 6;
    uint64_t* q_full = bars + 4 * kStages + 7;
    uint64_t* p_lo = bars + 4 * kStages + 8;  // [2]: first half of P_X (tokens 0-63) is in TMEM
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);
    int32_t* sIds = reinterpret_cast<int32_t*>(smem + kOffIds);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int seq_i = blockIdx.x / p.max_chunks, chunk = blockIdx.x % p.max_chunks;
    const int h = blockIdx.y;
    const PrefillSeq sm = p.seqs[seq_i];
    const int q0 = chunk * 2 * QT;
    if (q0 >= sm.q_len) return;  // uniform: no TMEM allocated yet
    const int prefix = sm.kv_len - sm.q_len;
    const int kv_end = min(sm.kv_len, prefix + q0 + 2 * QT);  // tokens the last query may see
    const int n_tiles = (kv_end + kN - 1) / kN;
    // the last chunk of a sequence may hold no query of tile B: its MMAs and
    // softmax are skipped (uniform over the CTA)
    const bool two_tiles = q0 + QT < sm.q_len;
    const int32_t* tab = p.table + (int64_t)sm.table_row * p.max_bps;

    // ---- set-up ----
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        // each barrier initialised once; p_full takes one arrive per softmax warp
        for (int i = 0; i < kNumBars; i++) {
            const bool per_warp = i == 4 * kStages + 2 || i == 4 * kStages + 3 || i >= 4 * kStages + 8;  // p_full, p_lo
            bar_init(&bars[i], per_warp ? 4u : 1u);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        // both query tiles, fp32, rows (query, head) query-major; rows past
        // the end of q read as zeros
        bar_expect(q_full, 2 * kQStageBytes);
        for (int X = 0; X < 2; X++)
            tma3_load(smem + kOffK + X * kQStageBytes, &tmQ, q_full, 0, h * G, sm.q_start + q0 + X * QT);
    }
    auto lookup = [&](int i) -> int32_t {
        if (i * 16 >= sm.kv_len) return p.max_blocks;  // past the end: zero-filled box
        const int32_t blk = tab[i];
        if ((uint32_t)blk >= (uint32_t)p.max_blocks) {
            atomicOr(p.err, kErrBounds);
            return p.max_blocks;
        }
        return blk;
    };
    for (int i = tid; i < min(n_tiles * kBlocksPerTile, kIdsCached); i += kThreads) sIds[i] = lookup(i);
    // Q tiles: row r of tile X is query X*QT + r / G, head r % G.  Each
    // softmax warp narrows rows w, w + 8, ... from the fp32 staging (one
    // 512-byte row per warp access) to bf16 in the 128B-swizzled layout.
    __syncthreads();  // barrier initialisation visible before anyone waits
    if (tid < kSoftmaxThreads && warp_wait(q_full, 0, abort_flag)) {
        const uint8_t* stage = smem + kOffK;
        for (int R = warp; R < 2 * kM; R += kSoftmaxThreads / 32) {
            const int X = R >> 7, r = R & (kM - 1);
            const float4 a = *reinterpret_cast<const float4*>(stage + X * kQStageBytes + r * 512 + lane * 16);
            *reinterpret_cast<uint2*>(smem + kOffQ + X * kQBytes + (lane >> 4) * (kM * 128) + swz(r, (lane & 15) >> 1) +
                                      (lane & 1) * 8) = make_uint2(pack_bf16(a.x, a.y), pack_bf16(a.z, a.w));
        }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == kSoftmaxThreads / 32) {
        // ================= TMA producer: K/V ring, 16 lanes issue =================
        // lane L < 16 copies block L/2 of the tile, 64-element half L%2
        const int b = lane >> 1, a = lane & 1;
        int k_issued = 0, v_issued = 0;  // tiles whose K (V) copies were issued
        for (int t = 0; t < n_tiles; t++) {
            const int slot = t % kStages, use = t / kStages;
            if (t >= kStages && !warp_wait(&k_empty[slot], (uint32_t)((use - 1) & 1), abort_flag)) break;
            if (lane == 0) bar_expect(&k_full[slot], kKBytes);
            __syncwarp();
            const int i = t * kBlocksPerTile + b;
            const int32_t blk = lane < 16 ? (i < kIdsCached ? sIds[i] : lookup(i)) : 0;
            if (lane < 16)
                tma4(smem + kOffK + slot * kKBytes + a * (kN * 128) + b * 16 * 128, &tmK, &k_full[slot], a * 64, h,
                     blk * 16, p.layer);
            k_issued = t + 1;
            if (t >= kStages && !warp_wait(&v_empty[slot], (uint32_t)((use - 1) & 1), abort_flag)) break;
            if (lane == 0) bar_expect(&v_full[slot], kVBytes);
            __syncwarp();
            if (lane < 16)
                tma4(smem + kOffV + slot * kVBytes + a * (kN * 128) + b * 16 * 128, &tmV, &v_full[slot], a * 64, h,
                     blk * 16, p.layer);
            v_issued = t + 1;
        }
        // every copy issued has landed before the CTA may exit (bounded)
        for (int t = max(0, k_issued - kStages); t < k_issued; t++) bar_wait(&k_full[t % kStages], (uint32_t)((t / kStages) & 1));
        for (int t = max(0, v_issued - kStages); t < v_issued; t++) bar_wait(&v_full[t % kStages], (uint32_t)((t / kStages) & 1));
    } else if (warp == kSoftmaxThreads / 32 + 1) {
        // ================= MMA issuer =================
        // The whole warp runs the loop and its waits; one elected lane issues
        // each MMA and commit.
        {
            constexpr uint32_t idS = idesc_bf16(kM, kN, 0, 0);  // Q, K both K-major
            constexpr uint32_t idO = idesc_bf16(kM, kD, 0, 1);  // P from TMEM, V MN-major
            // Descriptors of every operand buffer, built once.  The start
            // address is the descriptor's low field (address / 16, 14 bits;
            // shared addresses stay below 2^18), so a K step's offset inside a
            // buffer is a constant added to the buffer's descriptor and the
            // issue loops below are the MMAs alone.
            static_assert(kStages == 2, "descriptors are selected by tile parity");
            const uint64_t dq0 = sdesc(su32(smem + kOffQ), 16, 1024), dq1 = sdesc(su32(smem + kOffQ + kQBytes), 16, 1024);
            const uint64_t dk0 = sdesc(su32(smem + kOffK), 16, 1024), dk1 = sdesc(su32(smem + kOffK + kKBytes), 16, 1024);
            const uint64_t dv0 = sdesc(su32(smem + kOffV), kN * 128, 1024);
            const uint64_t dv1 = sdesc(su32(smem + kOffV + kVBytes), kN * 128, 1024);
            auto issue_s = [&](int X, int t) {
                const uint64_t da = X ? dq1 : dq0, db = (t & 1) ? dk1 : dk0;
#pragma unroll
                for (int ks = 0; ks < kD / 16; ks++) {
                    // 16 elements = 32 bytes inside a 128-byte atom row; 64 elements per atom column
                    constexpr uint32_t kAtomA = kM * 128 / 16, kAtomB = kN * 128 / 16;
                    mma_ss_w(tmem + X * 128, da + (ks >> 2) * kAtomA + (ks & 3) * 2, db + (ks >> 2) * kAtomB + (ks & 3) * 2,
                           idS, ks > 0);
                }
                mma_commit_w(&s_full[X]);
            };
            // PV in two halves of 64 tokens: the first runs while the softmax
            // still computes the second half of P
            auto issue_pv_half = [&](int X, int t, int half) {
                const uint64_t db = (t & 1) ? dv1 : dv0;
#pragma unroll
                for (int k = 0; k < kN / 32; k++) {
                    const int ks = half * (kN / 32) + k;
                    // P: 16 tokens = 8 columns of bf16 pairs; V: 16 token rows = 2 KB
                    mma_ts_w(tmem + kColO + X * 128, tmem + X * 128 + ks * 8, db + ks * (16 * 128 / 16), idO, t > 0 || ks > 0);
                }
                if (half) mma_commit_w(&pv_done[X]);
            };
            bool ok = warp_wait(&k_full[0], 0, abort_flag);
            if (ok) {
                tc_fence_after();
                issue_s(0, 0);
                if (two_tiles) issue_s(1, 0);
                mma_commit_w(&k_empty[0]);
            }
            for (int t = 0; t < n_tiles && ok; t++) {
                const int slot = t % kStages;
                const bool more = t + 1 < n_tiles;
                const int ns = (t + 1) % kStages;
                ok = warp_wait(&p_lo[0], (uint32_t)(t & 1), abort_flag) &&
                     warp_wait(&v_full[slot], (uint32_t)((t / kStages) & 1), abort_flag);
                if (!ok) break;
                tc_fence_after();
                issue_pv_half(0, t, 0);
                ok = warp_wait(&p_full[0], (uint32_t)(t & 1), abort_flag);
                if (!ok) break;
                tc_fence_after();
                issue_pv_half(0, t, 1);
                if (more) {  // S_A(t+1) overwrites P_A(t): issued after PV_A(t), which reads it first
                    ok = warp_wait(&k_full[ns], (uint32_t)(((t + 1) / kStages) & 1), abort_flag);
                    if (!ok) break;
                    issue_s(0, t + 1);
                }
                if (two_tiles) {
                    ok = warp_wait(&p_lo[1], (uint32_t)(t & 1), abort_flag);
                    if (!ok) break;
                    tc_fence_after();
                    issue_pv_half(1, t, 0);
                    ok = warp_wait(&p_full[1], (uint32_t)(t & 1), abort_flag);
                    if (!ok) break;
                    tc_fence_after();
                    issue_pv_half(1, t, 1);
                }
                mma_commit_w(&v_empty[slot]);  // after the last MMA that reads the stage
                if (more) {
                    if (two_tiles) issue_s(1, t + 1);
                    mma_commit_w(&k_empty[ns]);
                }
            }
            // everything this warp issued has finished before TMEM is freed
            mma_commit_w(drain);
            bar_wait(drain, 0);
        }
    } else {
        // ================= softmax warpgroups =================
        const int X = tid >> 7, r = tid & 127;
        const int g = r % G, qi = X * QT + r / G;
        const bool valid = q0 + qi < sm.q_len;
        const int row_limit = prefix + q0 + qi;  // last visible token
        const uint32_t lane_base = (uint32_t)(32 * ((tid >> 5) & 3)) << 16;
        const uint32_t tS = tmem + lane_base + X * 128;  // S_X, P_X over its first 64 columns
        const uint32_t tO = tmem + lane_base + kColO + X * 128;
        float m = -INFINITY;  // reference max (lags the true max by < 2^8)
        float l = 0.0f;
        bool ok = true;
        const bool active = X == 0 || two_tiles;  // an empty tile B does nothing
        for (int t = 0; active && t < n_tiles; t++) {
            // S_X(t) done also means PV_X(t-1) done (tcgen05.commit tracks every
            // earlier MMA of the issuing thread): O_X and P_X are free.
            if (!warp_wait(&s_full[X], (uint32_t)(t & 1), abort_flag)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float sc[kN];
            tmem_ld128(tS, sc);
            const int base = t * kN;
            if (base + kN - 1 > prefix + q0) {  // tile crosses the causal edge of some row
#pragma unroll
                for (int j = 0; j < kN; j++)
                    if (base + j > row_limit) sc[j] = -INFINITY;
            }
            // Row max of the raw scores over eight independent chains (16 deep);
            // rounding is monotonic, so max(s) * scale equals max(s * scale)
            // exactly.
            float m8[8];
#pragma unroll
            for (int j = 0; j < 8; j++) m8[j] = sc[j];
#pragma unroll
            for (int j = 8; j < kN; j++) m8[j & 7] = fmaxf(m8[j & 7], sc[j]);
            const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                                   fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7]))) *
                             p.scale_log2;
            const bool raise = mx > m + kRescaleAt;
            float corr = 1.0f;
            if (raise) {
                corr = ex2f(m - mx);  // 0 on the first tile (m = -inf)
                m = mx;
                l *= corr;
            }
            const float mref = m == -INFINITY ? 0.0f : m;  // nothing visible yet: p = 0
            // p = 2^(s * scale - mref): one packed FFMA per pair, then ex2
            const float2 sc2 = make_float2(p.scale_log2, p.scale_log2), nm2 = make_float2(-mref, -mref);
            float2 ls2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
            const bool rescale = t > 0 && __any_sync(0xffffffffu, raise);  // warp-uniform
#pragma unroll
            for (int q = 0; q < 4; q++) {
                float pk[16];
#pragma unroll
                for (int e = 0; e < 16; e++) {
                    const int j = q * 32 + 2 * e;
                    const float2 x = __ffma2_rn(make_float2(sc[j], sc[j + 1]), sc2, nm2);
                    const float2 pv = make_float2(ex2f(x.x), ex2f(x.y));
                    ls2[e & 1] = __fadd2_rn(ls2[e & 1], pv);
                    pk[e] = __uint_as_float(pack_bf16(pv.x, pv.y));
                }
                tmem_st16_nowait(tS + q * 16, pk);
                if (q == 1 && !rescale) {
                    // first half of P (tokens 0-63) handed over: its PV half
                    // runs while the second half is computed
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) bar_arrive(&p_lo[X]);
                }
            }
            // Rescale O_X (the scores are dead by now: no register pressure).
            // A warp that rescales hands over both halves of P only after it,
            // since the first PV half accumulates into O.
            if (rescale) {
#pragma unroll 1
                for (int c = 0; c < kD / 32; c++) {
                    float ov[32];
                    tmem_ld32(tO + c * 32, ov);
#pragma unroll
                    for (int j = 0; j < 32; j++) ov[j] *= corr;
                    tmem_st32_nowait(tO + c * 32, ov);
                }
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            l += (ls2[0].x + ls2[1].x) + (ls2[0].y + ls2[1].y);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (rescale) bar_arrive(&p_lo[X]);
                bar_arrive(&p_full[X]);
            }
        }
        // last PV of this tile, then the output rows
        if (active && ok && warp_wait(&pv_done[X], (uint32_t)((n_tiles - 1) & 1), abort_flag)) {
            tc_fence_after();
            const float inv = 1.0f / l;
            if (q0 + 2 * QT <= sm.q_len) {
                // Full chunk: this warp's 32 rows (times 1/l) go through
                // 128B-swizzled staging (row r at r * 128 bytes of each
                // 32-float column block) and four TMA stores of {32 floats,
                // G heads, 32 / G queries}.  Every MMA that reads the staging
                // is done: tile A uses the Q buffers (their last reader, S_B,
                // was issued before PV_A), tile B the K/V ring (after the last
                // MMA).  The staging address is recomputed here from the
                // shared-memory symbol and stored through st.shared: a generic
                // pointer kept from the prologue costs the main loop spills.
                const uint32_t stage = ((su32(smem_raw) + 1023u) & ~1023u) + (X == 0 ? kOffQ : kOffK);
#pragma unroll 1
                for (int a = 0; a < kD / 32; a++) {
                    float ov[32];
                    tmem_ld32(tO + a * 32, ov);
#pragma unroll
                    for (int c = 0; c < 8; c++)
                        asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(stage + a * (kM * 128) + swz(r, c)),
                                     "f"(ov[4 * c] * inv), "f"(ov[4 * c + 1] * inv), "f"(ov[4 * c + 2] * inv),
                                     "f"(ov[4 * c + 3] * inv)
                                     : "memory");
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) {
                    const int wr = 32 * (warp & 3);  // first row of this warp
                    for (int a = 0; a < kD / 32; a++)
                        tma3_store(&tmO, stage + a * (kM * 128) + wr * 128, a * 32, h * G, sm.q_start + q0 + X * QT + wr / G);
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                }
                __syncwarp();
            } else {
                float* orow = p.out + ((int64_t)(sm.q_start + q0 + qi) * p.Hq + h * G + g) * kD;
#pragma unroll 1
                for (int c = 0; c < kD / 32; c++) {
                    float ov[32];
                    tmem_ld32(tO + c * 32, ov);
                    if (valid) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            *reinterpret_cast<float4*>(orow + c * 32 + j) =
                                make_float4(ov[j] * inv, ov[j + 1] * inv, ov[j + 2] * inv, ov[j + 3] * inv);
                    }
                }
            }
        }
    }

    // ---- tear-down: every path frees TMEM ----
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && *abort_flag) {
        atomicOr(p.err, kErrTimeout);
        bar_wait(q_full, 0);  // the Q copy has landed before the CTA exits (bounded)
    }
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

// Tensor maps over this call's q and out ([n_rows][Hq][128] fp32): q is
// read one query tile (128 rows of (query, head)) per box; out is written
// in 128B-swizzled boxes of {32 floats, G heads, 32 / G queries}.
static int encode_q_out_maps(const PrefillParams& p, int G, CUtensorMap* tq, CUtensorMap* to) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        S1KV_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !fn) return set_error(S1KV_ECUDA, "s1kv: cuTensorMapEncodeTiled unavailable");
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    cuuint64_t dims[3] = {(cuuint64_t)kD, (cuuint64_t)p.Hq, (cuuint64_t)p.n_rows};
    cuuint64_t strides[2] = {(cuuint64_t)kD * 4, (cuuint64_t)p.Hq * kD * 4};
    cuuint32_t estr[3] = {1, 1, 1};
    cuuint32_t box_q[3] = {(cuuint32_t)kD, (cuuint32_t)G, (cuuint32_t)(kM / G)};
    CUresult r = encode(tq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(p.q), dims, strides, box_q, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(S1KV_EINVAL, "prefill: tensor map over q rejected (%d)", (int)r);
    cuuint32_t box_o[3] = {32, (cuuint32_t)G, (cuuint32_t)(32 / G)};
    r = encode(to, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, p.out, dims, strides, box_o, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(S1KV_EINVAL, "prefill: tensor map over out rejected (%d)", (int)r);
    return S1KV_OK;
}

template <int G>
static int launch_prefill_g(const PrefillParams& p, const CUtensorMap& tk, const CUtensorMap& tv, cudaStream_t stream) {
    CUtensorMap tq, to;
    int st = encode_q_out_maps(p, G, &tq, &to);
    if (st) return st;
    S1KV_CUDA(cudaFuncSetAttribute(prefill_tc_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    dim3 grid((unsigned)(p.n_seqs * p.max_chunks), (unsigned)p.Hkv);
    prefill_tc_kernel<G><<<grid, kThreads, kSmem, stream>>>(p, tk, tv, tq, to);
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

int prefill_queries_per_cta(int G) { return 2 * (kM / G); }

}  // namespace s1kv
