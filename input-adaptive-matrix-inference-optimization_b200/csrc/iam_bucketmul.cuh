// iam_bucketmul.cuh -- device building blocks of the bucketMul sparse GEMV on sm_100a.
//
// One bucketMul = cutoff search -> row selection -> accumulation (bucketMul.cl:68-497).
// On B200 the three phases run in ONE launch of thread-block clusters (iam_bucketmul.cu):
//   * every CTA recomputes the cutoff for its own use (4096 importance values held in
//     registers, one barrier per bisection step) -- no cutoff launch, no global round trip;
//   * the G CTAs of a cluster split the bucket rows into G input segments, select and
//     compact their segment (ascending row order -> deterministic), then rebalance the
//     selected rows evenly across the cluster through distributed shared memory counts;
//   * each cluster owns one column tile, so clusters never exchange data; the G partial
//     tiles of a cluster are summed through DSMEM in a fixed order (no global atomics).
#pragma once

#include <cooperative_groups.h>

#include "iam_common.cuh"

namespace iam {

namespace cg = cooperative_groups;

// ------------------------------------------------------------------ cutoff search

template <int NT>
struct CutoffShared {
    float mn[NT / 32];
    float mx[NT / 32];
    int cnt[2][NT / 32];
};

// Block-wide restatement of findCutoffBinarySearch (bucketMul.cl:68-214).  All threads of
// the block must call it; all receive the same cutoff.  The counts are exact integers and
// min/max are order independent, so any thread layout reproduces the reference's result
// bit for bit.  `target` = P - quantile (bucketMul.cl:81, bucket_mul.hpp:164).
template <int NT>
__device__ float block_find_cutoff(const float* __restrict__ x, const uint16_t* __restrict__ probes,
                                   int P, int target, CutoffShared<NT>& sm, int* iters_out) {
    constexpr int NW = NT / 32;
    constexpr int VPT = (kProbes + NT - 1) / NT;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    float v[VPT];
    float mn = INFINITY, mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const int i = tid + k * NT;
        if (i < P) {
            const float imp = importance(x[i], h2f(probes[i]));
            v[k] = imp;
            mn = fminf(mn, imp);
            mx = fmaxf(mx, imp);
        } else {
            v[k] = -1.0f;  // never counted: every tested mid is >= 0
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if (lane == 0) {
        sm.mn[warp] = mn;
        sm.mx[warp] = mx;
    }
    __syncthreads();
    mn = sm.mn[0];
    mx = sm.mx[0];
#pragma unroll
    for (int w = 1; w < NW; ++w) {
        mn = fminf(mn, sm.mn[w]);
        mx = fmaxf(mx, sm.mx[w]);
    }

    float lo = mn, hi = mx;
    float mid = __fmul_rn(__fadd_rn(lo, hi), 0.5f);  // (min+max)/2.0f, :139
    int min_count = P, max_count = 0;                // :142-143
    int it = 0;
    float result;
    for (;;) {
        int c = 0;
#pragma unroll
        for (int k = 0; k < VPT; ++k) c += (v[k] > mid) ? 1 : 0;  // ">" (:155)
        c = __reduce_add_sync(0xffffffffu, c);
        if (lane == 0) sm.cnt[it & 1][warp] = c;
        __syncthreads();
        int cnt = 0;
#pragma unroll
        for (int w = 0; w < NW; ++w) cnt += sm.cnt[it & 1][w];
        if (cnt < target) {
            hi = mid;
            max_count = cnt;
        } else {
            lo = mid;
            min_count = cnt;
        }
        const float next = __fmul_rn(__fadd_rn(lo, hi), 0.5f);
        ++it;
        if (cnt == target || __fsub_rn(hi, lo) < 1e-5f || abs(max_count - min_count) < 3) {
            result = mid;  // the mid that was tested (:198)
            break;
        }
        mid = next;
        if (it == kMaxIters) {
            result = mid;  // bounds[2] after the last update (:211-213)
            break;
        }
    }
    __syncthreads();  // sm.cnt may be reused by the caller
    if (iters_out) *iters_out = it;
    return result;
}

// ------------------------------------------------------------------ row selection

template <int NT>
struct ScanShared {
    int tot[2][NT / 32];
};

// prepareDispatch (bucketMul.cl:351-386) for inputs [i0, i1) of one expert: row
// row0 + 16*i + r is selected iff 1e5*|x[i]*stats[row][stride-1]| >= cutoff.  Selected
// rows are written to rows_out[0..n) in ascending order; returns n (same in all threads).
template <int NT>
__device__ int block_select(const float* __restrict__ x, const uint16_t* __restrict__ stats,
                            int stride, long long row0, int n_rows_valid, int i0, int i1,
                            float cutoff, int32_t* __restrict__ rows_out, ScanShared<NT>& sm) {
    constexpr int NW = NT / 32;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int base = 0, round = 0;
    for (int ib = i0; ib < i1; ib += NT, ++round) {
        const int i = ib + tid;
        unsigned mask = 0u;
        if (i < i1) {
            const float xi = x[i];
            const int rmax = min(16, n_rows_valid - i * 16);
            const uint16_t* sp = stats + (row0 + (long long)i * 16) * stride + (stride - 1);
            if (stride == 1 && rmax == 16 && ((reinterpret_cast<uintptr_t>(sp) & 15u) == 0)) {
                const uint4 a = *reinterpret_cast<const uint4*>(sp);
                const uint4 b = *reinterpret_cast<const uint4*>(sp + 8);
                const uint32_t wds[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
                for (int r = 0; r < 16; ++r) {
                    const uint32_t hb = (r & 1) ? (wds[r >> 1] >> 16) : (wds[r >> 1] & 0xffffu);
                    if (importance(xi, h2f(hb)) >= cutoff) mask |= 1u << r;  // ">=" (:380)
                }
            } else {
                for (int r = 0; r < rmax; ++r)
                    if (importance(xi, h2f(sp[r * stride])) >= cutoff) mask |= 1u << r;
            }
        }
        const int n = __popc(mask);
        int inc = n;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += t;
        }
        const int par = round & 1;
        if (lane == 31) sm.tot[par][warp] = inc;
        __syncthreads();
        int pre = 0, total = 0;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const int t = sm.tot[par][w];
            pre += (w < warp) ? t : 0;
            total += t;
        }
        int p = base + pre + inc - n;
        const int32_t rbase = (int32_t)(row0 + (long long)i * 16);
        while (mask) {
            const int r = __ffs(mask) - 1;
            mask &= mask - 1u;
            rows_out[p++] = rbase + r;
        }
        base += total;
    }
    __syncthreads();
    return base;
}

// ------------------------------------------------------------------ accumulation

template <int VEC>
struct VecLoad;
template <>
struct VecLoad<8> {
    using T = uint4;
    static IAM_DEV T load(const uint16_t* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
    static IAM_DEV uint32_t bits(const T& v, int k) {
        const uint32_t w = (k >> 1) == 0 ? v.x : (k >> 1) == 1 ? v.y : (k >> 1) == 2 ? v.z : v.w;
        return (k & 1) ? (w >> 16) : (w & 0xffffu);
    }
};
template <>
struct VecLoad<4> {
    using T = uint2;
    static IAM_DEV T load(const uint16_t* p) { return __ldg(reinterpret_cast<const uint2*>(p)); }
    static IAM_DEV uint32_t bits(const T& v, int k) {
        const uint32_t w = (k >> 1) == 0 ? v.x : v.y;
        return (k & 1) ? (w >> 16) : (w & 0xffffu);
    }
};
template <>
struct VecLoad<1> {
    using T = uint32_t;
    static IAM_DEV T load(const uint16_t* p) { return (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(p)); }
    static IAM_DEV uint32_t bits(const T& v, int) { return v; }
};

// Adds x * w_k into this lane's private slot accumulators acc[(slot*VEC + k) * 32].  The
// VEC addresses of one call are distinct (k differs), so all loads are issued before any
// store; successive calls may alias and stay in program order.
template <int VEC>
IAM_DEV void accumulate(float* __restrict__ acc, const typename VecLoad<VEC>::T& w, float x) {
    int off[VEC];
    float old[VEC];
#pragma unroll
    for (int k = 0; k < VEC; ++k) off[k] = ((int)((VecLoad<VEC>::bits(w, k) & 15u) * VEC + k)) << 5;
#pragma unroll
    for (int k = 0; k < VEC; ++k) old[k] = acc[off[k]];
#pragma unroll
    for (int k = 0; k < VEC; ++k) old[k] = fmaf(x, h2f(VecLoad<VEC>::bits(w, k)), old[k]);
#pragma unroll
    for (int k = 0; k < VEC; ++k) acc[off[k]] = old[k];
}

}  // namespace iam
