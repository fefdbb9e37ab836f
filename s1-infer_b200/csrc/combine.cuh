// combine.cuh -- merging the split-K partials of a decode row (device code
// shared by the decode kernels and the standalone combine kernel).
#pragma once

#include "internal.h"

namespace s1kv {

// Stores element d of (row, local head `head`) of the attention output.
// Exchange launches store it into this rank's slot and every peer's (NVLink)
// as one 64-bit word carrying the epoch beside the value: a single store of
// aligned 64 bits is seen whole or not at all, so a reader that polls the
// word until its epoch matches needs no fence, flag or counter from the
// writer (system scope: the readers run on other GPUs).
__device__ __forceinline__ void store_out(const AttnParams& p, int64_t row, int head, int d, int D, float v) {
    const int64_t i = (row * (p.out_stride > 0 ? p.out_stride : p.Hq) + p.out_head0 + head) * D + d;
    if (p.xout) {
        const uint64_t w = ((uint64_t)p.epoch << 32) | __float_as_uint(v);
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p.xout + i), "l"(w) : "memory");
        for (int k = 0; k < p.n_peers; k++)
            asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p.xpeer[k] + i), "l"(w) : "memory");
    } else {
        p.out[i] = v;
    }
}

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
        store_out(p, row, h * G + g, d, D, O / L);
    }
}

// Merges n partials of (row, KV head h) staged through shared memory (`sm`,
// at least 2 * (n + 1) * G floats): partial slots s0, s0 + stride, ...
// (split indices of the row, relative to its part_off).  The maxima,
// weights and normaliser are computed in parallel, then every (head, dim)
// output sums its n partials with eight loads in flight.  to_part: the
// result is written unnormalised as the partial of slot `dst` (its max
// and sum beside it; dst may be one of the sources: every element is read
// before the same thread writes it, and the maxima and sums are staged
// first); otherwise the normalised row is stored as the output.
__device__ __forceinline__ void merge_staged(const AttnParams& p, int row, int h, int G, int D, float* sm, int s0, int n,
                                             int stride, bool to_part, int dst) {
    const RowMeta rm = p.rows[row];
    const int tid = threadIdx.x, nt = blockDim.x;
    float* w = sm;           // [n][G]: max, then weight
    float* ls = sm + n * G;  // [n][G]: sums
    float* mg = ls + n * G;  // [G]: global max, then 1 / normaliser (or the sum)
    float* mx = mg + G;      // [G]: global max kept for a partial result
    for (int i = tid; i < n * G; i += nt) {
        const int s = s0 + (i / G) * stride, g = i % G;
        const int64_t part = (int64_t)(rm.part_off + s) * p.Hkv + h;
        w[i] = __ldcg(&p.part_ml[(part * G + g) * 2]);
        ls[i] = __ldcg(&p.part_ml[(part * G + g) * 2 + 1]);
    }
    __syncthreads();
    if (tid < G) {
        float M = -INFINITY;
        for (int j = 0; j < n; j++) M = fmaxf(M, w[j * G + tid]);
        mg[tid] = M;
        mx[tid] = M;
    }
    __syncthreads();
    for (int i = tid; i < n * G; i += nt) {
        const float m = w[i];
        float f = 0.0f;
        if (m != -INFINITY) asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(f) : "f"(m - mg[i % G]));
        w[i] = f;
    }
    __syncthreads();
    if (tid < G) {
        float L = 0.0f;
        for (int j = 0; j < n; j++) L = fmaf(ls[j * G + tid], w[j * G + tid], L);
        mg[tid] = to_part ? 1.0f : 1.0f / L;
        if (to_part) ls[tid] = L;  // the rows of ls were all read above
    }
    __syncthreads();
    const int64_t dpart = (int64_t)(rm.part_off + dst) * p.Hkv + h;
    const int64_t sstride = (int64_t)stride * p.Hkv * G * D;  // next source slot, same head
    auto put = [&](int g, int d, float o) {
        if (to_part) p.part_o[(dpart * G + g) * D + d] = o;
        else store_out(p, row, h * G + g, d, D, o);
    };
    if (D % 4 != 0) {
        for (int idx = tid; idx < G * D; idx += nt) {
            const int g = idx / D, d = idx % D;
            const float* po = p.part_o + ((int64_t)(rm.part_off + s0) * p.Hkv + h) * G * D + g * D + d;
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            int j = 0;
            for (; j + 8 <= n; j += 8) {
#pragma unroll
                for (int u = 0; u < 8; u++) acc[u] = fmaf(__ldcg(po + (j + u) * sstride), w[(j + u) * G + g], acc[u]);
            }
            for (; j < n; j++) acc[0] = fmaf(__ldcg(po + j * sstride), w[j * G + g], acc[0]);
            const float O = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
            put(g, d, O * mg[g]);
        }
    } else {
        // each thread sums 4 adjacent dims of one head (16-byte loads, eight
        // sources in flight): a merge is bound by the bytes this one CTA
        // keeps in flight
        const float4* base = reinterpret_cast<const float4*>(p.part_o + ((int64_t)(rm.part_off + s0) * p.Hkv + h) * G * D);
        const int64_t stride4 = sstride / 4;
        for (int c = tid; c < G * D / 4; c += nt) {
            const int g = (4 * c) / D, d = (4 * c) % D;
            const float4* po = base + c;
            float4 acc[8];
#pragma unroll
            for (int u = 0; u < 8; u++) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            int j = 0;
            for (; j + 8 <= n; j += 8) {
                float4 v[8];
#pragma unroll
                for (int u = 0; u < 8; u++) v[u] = __ldcg(po + (j + u) * stride4);
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    const float f = w[(j + u) * G + g];
                    acc[u] = make_float4(fmaf(v[u].x, f, acc[u].x), fmaf(v[u].y, f, acc[u].y),
                                         fmaf(v[u].z, f, acc[u].z), fmaf(v[u].w, f, acc[u].w));
                }
            }
            for (; j < n; j++) {
                const float4 v = __ldcg(po + j * stride4);
                const float f = w[j * G + g];
                acc[0] = make_float4(fmaf(v.x, f, acc[0].x), fmaf(v.y, f, acc[0].y), fmaf(v.z, f, acc[0].z),
                                     fmaf(v.w, f, acc[0].w));
            }
            const float r = mg[g];
            put(g, d + 0, (((acc[0].x + acc[1].x) + (acc[2].x + acc[3].x)) + ((acc[4].x + acc[5].x) + (acc[6].x + acc[7].x))) * r);
            put(g, d + 1, (((acc[0].y + acc[1].y) + (acc[2].y + acc[3].y)) + ((acc[4].y + acc[5].y) + (acc[6].y + acc[7].y))) * r);
            put(g, d + 2, (((acc[0].z + acc[1].z) + (acc[2].z + acc[3].z)) + ((acc[4].z + acc[5].z) + (acc[6].z + acc[7].z))) * r);
            put(g, d + 3, (((acc[0].w + acc[1].w) + (acc[2].w + acc[3].w)) + ((acc[4].w + acc[5].w) + (acc[6].w + acc[7].w))) * r);
        }
    }
    if (to_part && tid < G) {
        p.part_ml[(dpart * G + tid) * 2] = mx[tid];
        p.part_ml[(dpart * G + tid) * 2 + 1] = ls[tid];
    }
}

// Arrival of one CTA on counter `ctr` that `total` CTAs share; true in the
// last to arrive.  One thread fences for the CTA (the pattern of a grid
// barrier): the barrier orders every thread's stores before thread 0's
// fence, which is cumulative over them, so they are visible before the
// arrival; the last arriver fences again before it reads (__ldcg, L2) and
// the barrier passes that on.  A fence in every thread made each CTA's exit
// wait for all of its threads' fences.
__device__ __forceinline__ bool arrive_last(int32_t* ctr, int total, int* flag) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const int prev = atomicAdd(ctr, 1);
        const bool last = prev == total - 1;
        if (last) {
            __threadfence();
            *ctr = 0;  // no other CTA touches it again in this launch
        }
        *flag = last;
    }
    __syncthreads();
    return *flag != 0;
}

// Called by every CTA of a multi-split row once its partial (split `split`
// of n_split) is written.  Rows of up to kMergeGroup splits: the last CTA to
// arrive on the (row, head) counter merges all partials.  Longer rows merge
// in two levels, so no CTA reads more than kMergeGroup partials: the last
// arriver of each group of kMergeGroup consecutive splits merges the group
// into the group's first partial slot, then arrives on the row counter; the
// last group merges the groups' results into the output row.  Counters
// return to zero (each reset by its last arriver); every CTA arrives, also
// after a timeout.  `flag` is one int of the caller's shared memory and
// `scratch` (scratch_floats floats of free shared memory) stages the merge.
__device__ __forceinline__ void finish_split_row(const AttnParams& p, int row, int h, int split, int n_split, int G,
                                                 int D, int* flag, float* scratch, int scratch_floats) {
    int32_t* ctr = p.counters + ((int64_t)row * p.Hkv + h) * kCounterStride;
    if (n_split <= kMergeGroup) {
        if (!arrive_last(ctr, n_split, flag)) return;
        if (2 * (n_split + 1) * G + 2 * G <= scratch_floats)
            merge_staged(p, row, h, G, D, scratch, 0, n_split, 1, false, 0);
        else
            combine_partials(p, row, h, G, D, threadIdx.x, blockDim.x);
        return;
    }
    const int grp = split / kMergeGroup, n_groups = (n_split + kMergeGroup - 1) / kMergeGroup;
    const int first = grp * kMergeGroup, in_grp = min(kMergeGroup, n_split - first);
    if (!arrive_last(ctr + 1 + grp, in_grp, flag)) return;
    merge_staged(p, row, h, G, D, scratch, first, in_grp, 1, true, first);
    if (!arrive_last(ctr, n_groups, flag)) return;
    merge_staged(p, row, h, G, D, scratch, 0, n_groups, kMergeGroup, false, 0);
}

}  // namespace s1kv
