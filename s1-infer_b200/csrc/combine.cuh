// combine.cuh -- merging the split-K partials of a decode row (device code
// shared by the decode kernels and the standalone combine kernel).
#pragma once

#include "internal.h"

namespace s1kv {

// Stores element d of (row, local head `head`) of the attention output, and
// the same element of every peer's buffer (NVLink stores).
__device__ __forceinline__ void store_out(const AttnParams& p, int64_t row, int head, int d, int D, float v) {
    const int64_t i = (row * (p.out_stride > 0 ? p.out_stride : p.Hq) + p.out_head0 + head) * D + d;
    p.out[i] = v;
    for (int k = 0; k < p.n_peers; k++) p.peer_out[k][i] = v;
}

// Called by every thread of a CTA that has just stored a finished (row, KV
// head): when the launch's last such CTA arrives, this rank's flag on every
// rank is set to the epoch (release, system scope), after every store of the
// launch.  The barrier orders the CTA's stores before thread 0's system-scope
// fence, which is cumulative over them (the pattern of a grid barrier).
__device__ __forceinline__ void signal_done(const AttnParams& p) {
    if (!p.done) return;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        const uint32_t prev = atomicAdd(p.done, 1u);
        if (prev == (uint32_t)p.done_total - 1) {
            *p.done = 0;
            __threadfence_system();
            for (int r = 0; r < p.n_flags; r++)
                asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p.flag_dst[r]), "r"(p.epoch) : "memory");
        }
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

// The same merge with the splits' (max, sum) staged in shared memory
// (`sm`, at least 2 * (n_split + 1) * G floats): the maxima, weights and
// normaliser are computed in parallel, then every (head, dim) output sums
// its n_split partials with eight splits' loads in flight.  Long rows (64+
// splits per row) make the serial loop above latency-bound.
__device__ __forceinline__ void combine_partials_staged(const AttnParams& p, int row, int h, int G, int D, float* sm) {
    const RowMeta rm = p.rows[row];
    const int ns = rm.n_split, tid = threadIdx.x, nt = blockDim.x;
    float* w = sm;            // [ns][G]: max, then weight
    float* ls = sm + ns * G;  // [ns][G]: sums
    float* mg = ls + ns * G;  // [G]: global max, then 1 / normaliser
    for (int i = tid; i < ns * G; i += nt) {
        const int s = i / G, g = i % G;
        const int64_t part = (int64_t)(rm.part_off + s) * p.Hkv + h;
        w[i] = __ldcg(&p.part_ml[(part * G + g) * 2]);
        ls[i] = __ldcg(&p.part_ml[(part * G + g) * 2 + 1]);
    }
    __syncthreads();
    if (tid < G) {
        float M = -INFINITY;
        for (int s = 0; s < ns; s++) M = fmaxf(M, w[s * G + tid]);
        mg[tid] = M;
    }
    __syncthreads();
    for (int i = tid; i < ns * G; i += nt) {
        const float m = w[i];
        float f = 0.0f;
        if (m != -INFINITY) asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(f) : "f"(m - mg[i % G]));
        w[i] = f;
    }
    __syncthreads();
    if (tid < G) {
        float L = 0.0f;
        for (int s = 0; s < ns; s++) L = fmaf(ls[s * G + tid], w[s * G + tid], L);
        mg[tid] = 1.0f / L;
    }
    __syncthreads();
    if (D % 4 != 0) {
        for (int idx = tid; idx < G * D; idx += nt) {
            const int g = idx / D, d = idx % D;
            const float* po = p.part_o + ((int64_t)rm.part_off * p.Hkv + h) * G * D + g * D + d;
            const int64_t stride = (int64_t)p.Hkv * G * D;  // next split, same head
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            int s = 0;
            for (; s + 8 <= ns; s += 8) {
#pragma unroll
                for (int u = 0; u < 8; u++) acc[u] = fmaf(__ldcg(po + (s + u) * stride), w[(s + u) * G + g], acc[u]);
            }
            for (; s < ns; s++) acc[0] = fmaf(__ldcg(po + s * stride), w[s * G + g], acc[0]);
            const float O = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
            store_out(p, row, h * G + g, d, D, O * mg[g]);
        }
        return;
    }
    // Each thread sums 4 adjacent dims of one head (16-byte loads, eight
    // splits in flight): per element the same sums in the same order as the
    // scalar loop above, with 4x the bytes in flight.  A row's partials are
    // ns * G * D * 4 bytes (1.2 MB at 293 splits of 8 heads), read by this one
    // CTA, so its loads in flight set the merge time.
    const float4* base = reinterpret_cast<const float4*>(p.part_o + ((int64_t)rm.part_off * p.Hkv + h) * G * D);
    const int64_t stride4 = (int64_t)p.Hkv * G * D / 4;  // next split, same head
    for (int c = tid; c < G * D / 4; c += nt) {
        const int g = (4 * c) / D, d = (4 * c) % D;
        const float4* po = base + c;
        float4 acc[8];
#pragma unroll
        for (int u = 0; u < 8; u++) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        int s = 0;
        for (; s + 8 <= ns; s += 8) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) v[u] = __ldcg(po + (s + u) * stride4);
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const float f = w[(s + u) * G + g];
                acc[u] = make_float4(fmaf(v[u].x, f, acc[u].x), fmaf(v[u].y, f, acc[u].y), fmaf(v[u].z, f, acc[u].z),
                                     fmaf(v[u].w, f, acc[u].w));
            }
        }
        for (; s < ns; s++) {
            const float4 v = __ldcg(po + s * stride4);
            const float f = w[s * G + g];
            acc[0] = make_float4(fmaf(v.x, f, acc[0].x), fmaf(v.y, f, acc[0].y), fmaf(v.z, f, acc[0].z),
                                 fmaf(v.w, f, acc[0].w));
        }
        const float r = mg[g];
        const float o[4] = {
            (((acc[0].x + acc[1].x) + (acc[2].x + acc[3].x)) + ((acc[4].x + acc[5].x) + (acc[6].x + acc[7].x))) * r,
            (((acc[0].y + acc[1].y) + (acc[2].y + acc[3].y)) + ((acc[4].y + acc[5].y) + (acc[6].y + acc[7].y))) * r,
            (((acc[0].z + acc[1].z) + (acc[2].z + acc[3].z)) + ((acc[4].z + acc[5].z) + (acc[6].z + acc[7].z))) * r,
            (((acc[0].w + acc[1].w) + (acc[2].w + acc[3].w)) + ((acc[4].w + acc[5].w) + (acc[6].w + acc[7].w))) * r};
#pragma unroll
        for (int j = 0; j < 4; j++) store_out(p, row, h * G + g, d + j, D, o[j]);
    }
}

// Called by every CTA of a multi-split row once its partial is written:
// the last CTA to arrive on the (row, head) counter merges the row and sets
// the counter back to zero, so no separate combine launch is needed.
// `flag` is one int of the caller's shared memory; `scratch` (free shared
// memory of `scratch_floats` floats) stages the merge when it fits.  Every
// CTA arrives, also after a timeout, so the counters always return to zero.
__device__ __forceinline__ void finish_split_row(const AttnParams& p, int row, int h, int n_split, int G, int D,
                                                 int* flag, float* scratch, int scratch_floats) {
    // One thread fences for the CTA (the pattern of a grid barrier): the
    // barrier orders every thread's partial stores before thread 0's fence,
    // which is cumulative over them, so the partial is visible before the
    // arrival; the last arriver fences again before the merge reads (__ldcg,
    // L2) and the barrier passes that on.  A fence in every thread made each
    // CTA's exit wait for all of its threads' fences.
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const int prev = atomicAdd(&p.counters[(int64_t)row * p.Hkv + h], 1);
        const bool last = prev == n_split - 1;
        if (last) __threadfence();
        *flag = last;
    }
    __syncthreads();
    if (*flag) {
        if (2 * (n_split + 1) * G <= scratch_floats)
            combine_partials_staged(p, row, h, G, D, scratch);
        else
            combine_partials(p, row, h, G, D, threadIdx.x, blockDim.x);
        if (threadIdx.x == 0) p.counters[(int64_t)row * p.Hkv + h] = 0;
        signal_done(p);
    }
}

}  // namespace s1kv
