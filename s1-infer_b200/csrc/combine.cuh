// combine.cuh -- merging the split-K partials of a decode row (device code
// shared by the decode kernels and the standalone combine kernel).
#pragma once

#include "internal.h"

namespace s1kv {

// out[row, h*G + g, :] = sum_s 2^(M_s - M) O_s / sum_s 2^(M_s - M) L_s over
// the n_split partials (max M_s in log2 units, sum L_s, unnormalised O_s)
// of query row `row` and KV head h; run by `nthreads` threads of one CTA.
// Partials written by other CTAs are read through L2 (__ldcg).
__device__ __forceinline__ void combine_partials(const AttnParams& p, int row, int h, int G, int D, int tid,
                                                 int nthreads) {
    const RowMeta rm = p.rows[row];
    for (int idx = tid; idx < G * D; idx += nthreads) {
        const int g = idx / D, d = idx % D;
        float M = -INFINITY;
        for (int s = 0; s < rm.n_split; s++) {
            const int64_t part = (int64_t)(rm.part_off + s) * p.Hkv + h;
            M = fmaxf(M, __ldcg(&p.part_ml[(part * G + g) * 2]));
        }
        float L = 0.0f, O = 0.0f;
        for (int s = 0; s < rm.n_split; s++) {
            const int64_t part = (int64_t)(rm.part_off + s) * p.Hkv + h;
            const float ms = __ldcg(&p.part_ml[(part * G + g) * 2]);
            float f = 0.0f;
            if (ms != -INFINITY) asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(f) : "f"(ms - M));
            L = fmaf(__ldcg(&p.part_ml[(part * G + g) * 2 + 1]), f, L);
            O = fmaf(__ldcg(&p.part_o[(part * G + g) * D + d]), f, O);
        }
        p.out[((int64_t)row * p.Hq + h * G + g) * D + d] = O / L;
    }
}

// Called by every CTA of a multi-split row once its partial is written:
// the last CTA to arrive on the (row, head) counter merges the row and sets
// the counter back to zero, so no separate combine launch is needed.
// `flag` is one int of the caller's shared memory.  Every CTA arrives, also
// after a timeout, so the counters always return to zero.
__device__ __forceinline__ void finish_split_row(const AttnParams& p, int row, int h, int n_split, int G, int D,
                                                 int* flag) {
    __threadfence();  // this CTA's partial is visible before its arrival
    __syncthreads();
    if (threadIdx.x == 0) {
        const int prev = atomicAdd(&p.counters[(int64_t)row * p.Hkv + h], 1);
        *flag = (prev == n_split - 1);
    }
    __syncthreads();
    if (*flag) {
        __threadfence();  // every other CTA's partial is visible to this one
        combine_partials(p, row, h, G, D, threadIdx.x, blockDim.x);
        if (threadIdx.x == 0) p.counters[(int64_t)row * p.Hkv + h] = 0;
    }
}

}  // namespace s1kv
