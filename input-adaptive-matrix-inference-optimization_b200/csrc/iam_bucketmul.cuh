// iam_bucketmul.cuh -- device building blocks of the bucketMul sparse GEMV on sm_100a:
// the cutoff search (bucketMul.cl:68-214), the row-selection predicate (:351-386) with a
// compacting scan, input providers that fuse the layer glue into the matmul prologue, and
// the per-slot accumulation of bucketMul (:392-447).  The fused kernel that strings them
// together is in iam_bucketmul.cu.
#pragma once

#include <cooperative_groups.h>

#include <utility>

#include "iam_common.cuh"

namespace iam {

namespace cg = cooperative_groups;

// ------------------------------------------------------------------ cutoff search

template <int NT>
struct CutoffShared {
    float mn[NT / 32];
    float mx[NT / 32];
    int cnt[2][NT / 32];
    float result;
    int steps;
};

// fp32 (a + b) / 2 exactly as the reference computes its mids (bucketMul.cl:139, :190).
IAM_DEV float bisect_mid(float a, float b) { return __fmul_rn(__fadd_rn(a, b), 0.5f); }

// Block-wide restatement of findCutoffBinarySearch (bucketMul.cl:68-214).  All threads of
// the block must call it; all receive the same cutoff.  The counts are exact integers and
// min/max are order independent, so any thread layout reproduces the reference's result
// bit for bit.  `target` = P - quantile (bucketMul.cl:81, bucket_mul.hpp:164).
//
// NWC warps (one per SM sub-partition by default) hold the 4096 importance values in
// registers and run the bisection among themselves behind a named barrier: a step costs a
// handful of compares per lane plus one 32*NWC-thread barrier instead of a full-block one.
IAM_DEV void debug_stamp(long long* dbg, int k) {
    if (dbg) {
        long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        dbg[k] = t;
    }
}

struct NoSideTask {
    IAM_DEV void operator()() const {}
};

// side(): work for the warps outside the search (anything that does not need the cutoff),
// run while the NWC search warps bisect.
template <int NT, int NWC = 4, class XP, class Side = NoSideTask>
__device__ float block_find_cutoff(const XP& xp, const uint16_t* __restrict__ probes, int P,
                                   int target, CutoffShared<NT>& sm, int* iters_out,
                                   long long* dbg = nullptr, const Side& side = Side()) {
    static_assert(NWC * 32 <= NT, "cutoff warps exceed the block");
    constexpr int NCT = NWC * 32;
    constexpr int VPT = (kProbes + NCT - 1) / NCT;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (warp < NWC) {
        float v[VPT];
        unsigned mnb = 0x7f800000u, mxb = 0u;  // imp >= 0: float order == bit order
        // lane t of the NWC warps owns values [t*VPT, t*VPT + VPT): vector loads when the
        // full 4096 are in use and both arrays are 16-byte aligned
        const int i_base = tid * VPT;
        if (XP::kVectorizable && P == kProbes && VPT % 8 == 0 && xp.aligned16() &&
            ((reinterpret_cast<uintptr_t>(probes) & 15u) == 0)) {
#pragma unroll
            for (int k = 0; k < VPT; k += 8) {
                const uint4 pb = __ldg(reinterpret_cast<const uint4*>(probes + i_base + k));
                float xv[8];
                xp.load8(i_base + k, xv);
                const uint32_t pw[4] = {pb.x, pb.y, pb.z, pb.w};
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const uint32_t hb = (e & 1) ? (pw[e >> 1] >> 16) : (pw[e >> 1] & 0xffffu);
                    v[k + e] = importance(xv[e], h2f(hb));
                }
            }
#pragma unroll
            for (int k = 0; k < VPT; ++k) {
                mnb = min(mnb, __float_as_uint(v[k]));
                mxb = max(mxb, __float_as_uint(v[k]));
            }
        } else {
#pragma unroll
            for (int k = 0; k < VPT; ++k) {
                const int i = i_base + k;
                if (i < P) {
                    v[k] = importance(xp(i), h2f(__ldg(probes + i)));
                    mnb = min(mnb, __float_as_uint(v[k]));
                    mxb = max(mxb, __float_as_uint(v[k]));
                } else {
                    v[k] = -1.0f;  // never counted: every tested mid is >= 0
                }
            }
        }
        mnb = __reduce_min_sync(0xffffffffu, mnb);
        mxb = __reduce_max_sync(0xffffffffu, mxb);
        if (lane == 0) {
            sm.mn[warp] = __uint_as_float(mnb);
            sm.mx[warp] = __uint_as_float(mxb);
        }
        asm volatile("bar.sync 1, %0;" ::"n"(NCT));
        debug_stamp(dbg, 0);
        float mn = sm.mn[0], mx = sm.mx[0];
#pragma unroll
        for (int w = 1; w < NWC; ++w) {
            mn = fminf(mn, sm.mn[w]);
            mx = fmaxf(mx, sm.mx[w]);
        }
        float lo = mn, hi = mx;
        float mid = bisect_mid(lo, hi);    // (min+max)/2.0f, :139
        int min_count = P, max_count = 0;  // :142-143
        int it = 0;
        float result;
        for (;;) {
            int c4[4] = {0, 0, 0, 0};  // four short chains instead of one VPT-long chain
#pragma unroll
            for (int k = 0; k < VPT; ++k) c4[k & 3] += (v[k] > mid) ? 1 : 0;  // ">" (:155)
            int c = __reduce_add_sync(0xffffffffu, (c4[0] + c4[1]) + (c4[2] + c4[3]));
            if (lane == 0) sm.cnt[it & 1][warp] = c;
            asm volatile("bar.sync 1, %0;" ::"n"(NCT));
            int cnt = 0;
#pragma unroll
            for (int w = 0; w < NWC; ++w) cnt += sm.cnt[it & 1][w];
            // the update of :150-213 with selects instead of branches
            const bool below = cnt < target;
            hi = below ? mid : hi;
            max_count = below ? cnt : max_count;
            lo = below ? lo : mid;
            min_count = below ? min_count : cnt;
            const float next = bisect_mid(lo, hi);
            ++it;
            const bool stop = (cnt == target) | (__fsub_rn(hi, lo) < 1e-5f) | (abs(max_count - min_count) < 3);
            result = stop ? mid : next;  // the mid that was tested (:198), else bounds[2] (:211-213)
            mid = stop ? mid : next;
            if (stop | (it == kMaxIters)) break;
        }
        if (tid == 0) {
            sm.result = result;
            sm.steps = it;
        }
        debug_stamp(dbg, 1);
    } else {
        side();
    }
    __syncthreads();
    const float result = sm.result;
    if (iters_out) *iters_out = sm.steps;
    __syncthreads();  // the shared state may be reused by the caller
    return result;
}

// ------------------------------------------------------------------ input providers
// The bucketMul input x is read through a provider so layer glue runs inside the matmul's
// prologue: every CTA evaluates the same function of the same bits, so all CTAs see
// bit-identical x and therefore compute the same cutoff and selection.

// Every provider also offers load8 (8 consecutive values, 16-byte aligned) for the cutoff's
// vector loads; kVectorizable says whether that path is worth taking.
// x = a plain fp32 vector.
struct XPlain {
    static constexpr bool kVectorizable = true;
    const float* x;
    IAM_DEV float operator()(int i) const { return __ldg(x + i); }
    IAM_DEV bool aligned16() const { return (reinterpret_cast<uintptr_t>(x) & 15u) == 0; }
    IAM_DEV void load8(int i, float* o) const {
        const float4 a = __ldg(reinterpret_cast<const float4*>(x + i));
        const float4 b = __ldg(reinterpret_cast<const float4*>(x + i + 4));
        o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
        o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
    }
};

// x = rmsNorm32fast(src) * gain (aux.cl:156-196 then mul16x32 aux.cl:434-440): the scale is
// computed once per CTA by block_rms_scale.
struct XRms {
    static constexpr bool kVectorizable = true;
    const float* src;
    const uint16_t* gain;
    float scale;
    IAM_DEV float operator()(int i) const {
        return __fmul_rn(h2f(__ldg(gain + i)), __fmul_rn(__ldg(src + i), scale));
    }
    IAM_DEV bool aligned16() const {
        return ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(gain)) & 15u) == 0;
    }
    IAM_DEV void load8(int i, float* o) const {
        const float4 a = __ldg(reinterpret_cast<const float4*>(src + i));
        const float4 b = __ldg(reinterpret_cast<const float4*>(src + i + 4));
        const uint4 gb = __ldg(reinterpret_cast<const uint4*>(gain + i));
        const float s8[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        const uint32_t gw[4] = {gb.x, gb.y, gb.z, gb.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const uint32_t hb = (e & 1) ? (gw[e >> 1] >> 16) : (gw[e >> 1] & 0xffffu);
            o[e] = __fmul_rn(h2f(hb), __fmul_rn(s8[e], scale));
        }
    }
};

// x = silu32(gate, up) = up * gate / (1 + exp(-gate)) (matrix.cl:27-32).
struct XSilu {
    static constexpr bool kVectorizable = true;
    const float* gate;
    const float* up;
    static IAM_DEV float f(float gv, float uv) { return __fdiv_rn(__fmul_rn(uv, gv), __fadd_rn(1.0f, expf(-gv))); }
    IAM_DEV float operator()(int i) const { return f(__ldg(gate + i), __ldg(up + i)); }
    IAM_DEV bool aligned16() const {
        return ((reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(up)) & 15u) == 0;
    }
    IAM_DEV void load8(int i, float* o) const {
        const float4 g0 = __ldg(reinterpret_cast<const float4*>(gate + i));
        const float4 g1 = __ldg(reinterpret_cast<const float4*>(gate + i + 4));
        const float4 u0 = __ldg(reinterpret_cast<const float4*>(up + i));
        const float4 u1 = __ldg(reinterpret_cast<const float4*>(up + i + 4));
        const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const float uv[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = f(gv[e], uv[e]);
    }
};

// rsqrt(sum(x^2)/n + eps) with the reduction order of rmsNorm32fast (aux.cl:165-190) when
// n is a multiple of 256 (256 contiguous runs, then a halving tree), else sequential.
// Every thread returns the same value.  red must hold 256 floats.  The run loads are issued
// together (float4 when aligned); the tree levels 16..1 pair the same elements through warp
// shuffles (lane t + s is thread t + s of warp 0), so the sums are bit-identical.
template <int NT>
__device__ float block_rms_scale(const float* __restrict__ x, int n, float eps, float* red) {
    static_assert(NT >= 256, "rms scale needs >= 256 threads");
    const int tid = threadIdx.x;
    if (n >= 256 && n % 256 == 0) {
        if (tid < 256) {
            const int e = n / 256;
            const float* xr = x + (size_t)tid * e;
            float s = 0.0f;
            if (e % 16 == 0 && ((reinterpret_cast<uintptr_t>(x) & 15u) == 0)) {
                for (int b = 0; b < e; b += 16) {
                    float4 q[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) q[k] = __ldg(reinterpret_cast<const float4*>(xr + b) + k);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        s = __fadd_rn(s, __fmul_rn(q[k].x, q[k].x));
                        s = __fadd_rn(s, __fmul_rn(q[k].y, q[k].y));
                        s = __fadd_rn(s, __fmul_rn(q[k].z, q[k].z));
                        s = __fadd_rn(s, __fmul_rn(q[k].w, q[k].w));
                    }
                }
            } else {
                for (int i = 0; i < e; ++i) {
                    const float v = __ldg(xr + i);
                    s = __fadd_rn(s, __fmul_rn(v, v));
                }
            }
            red[tid] = s;
        }
        __syncthreads();
        for (int s = 128; s >= 32; s >>= 1) {
            if (tid < s) red[tid] = __fadd_rn(red[tid], red[tid + s]);
            __syncthreads();
        }
        if (tid < 32) {
            float v = red[tid];
#pragma unroll
            for (int s = 16; s > 0; s >>= 1) v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, s));
            if (tid == 0) red[0] = v;
        }
        __syncthreads();
    } else {
        if (tid == 0) {
            float s = 0.0f;
            for (int i = 0; i < n; ++i) {
                const float v = __ldg(x + i);
                s = __fadd_rn(s, __fmul_rn(v, v));
            }
            red[0] = s;
        }
        __syncthreads();
    }
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(red[0], (float)n), eps)));
    __syncthreads();
    return scale;
}

// ------------------------------------------------------------------ row selection

template <int NT>
struct ScanShared {
    int tot[2][NT / 32];
};

// The 16 row importances 1e5*|x[i]*stats[row]| of one input (-1 for rows past
// n_rows_valid: never selected, every cutoff is >= 0).
template <class XP>
IAM_DEV void input_importances(const XP& xp, const uint16_t* __restrict__ stats, int stride, long long row0,
                               int n_rows_valid, int i, float* imp) {
    const float xi = xp(i);
    const int rmax = min(16, n_rows_valid - i * 16);
    const uint16_t* sp = stats + (row0 + (long long)i * 16) * stride + (stride - 1);
    if (stride == 1 && rmax == 16 && ((reinterpret_cast<uintptr_t>(sp) & 15u) == 0)) {
        const uint4 a = __ldg(reinterpret_cast<const uint4*>(sp));
        const uint4 b = __ldg(reinterpret_cast<const uint4*>(sp + 8));
        const uint32_t wds[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int r = 0; r < 16; ++r) imp[r] = importance(xi, h2f((r & 1) ? (wds[r >> 1] >> 16) : (wds[r >> 1] & 0xffffu)));
    } else {
#pragma unroll
        for (int r = 0; r < 16; ++r) imp[r] = r < rmax ? importance(xi, h2f(__ldg(sp + r * stride))) : -1.0f;
    }
}

// prepareDispatch predicate (bucketMul.cl:351-386) for inputs [i0, i1) of one expert: bit r
// of masks[i - i0] is set iff row row0 + 16*i + r is selected, i.e.
// 1e5*|x[i]*stats[row][stride-1]| >= cutoff.  Returns the number of selected rows (same in
// all threads).  The importances of inputs [i0, i0 + npre) were computed beforehand (by the
// warps outside the cutoff search, during the search): thread 128 + t holds input i0 + t in
// pimp when pin >= 0.  Inputs past i0 + npre are done here by every thread.
template <int NT, class XP>
__device__ int block_masks_pre(const XP& xp, const uint16_t* __restrict__ stats, int stride, long long row0,
                               int n_rows_valid, int i0, int i1, int npre, float cutoff, int pin,
                               const float* pimp, uint16_t* __restrict__ masks, ScanShared<NT>& sm) {
    constexpr int NW = NT / 32;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int cnt = 0;
    if (pin >= 0) {
        unsigned mask = 0u;
#pragma unroll
        for (int r = 0; r < 16; ++r) mask |= (pimp[r] >= cutoff) ? (1u << r) : 0u;  // ">=" (:380)
        masks[pin - i0] = (uint16_t)mask;
        cnt += __popc(mask);
    }
    for (int i = i0 + npre + tid; i < i1; i += NT) {
        float imp[16];
        input_importances(xp, stats, stride, row0, n_rows_valid, i, imp);
        unsigned mask = 0u;
#pragma unroll
        for (int r = 0; r < 16; ++r) mask |= (imp[r] >= cutoff) ? (1u << r) : 0u;
        masks[i - i0] = (uint16_t)mask;
        cnt += __popc(mask);
    }
    cnt = __reduce_add_sync(0xffffffffu, cnt);
    if (lane == 0) sm.tot[0][warp] = cnt;
    __syncthreads();
    int total = 0;
#pragma unroll
    for (int w = 0; w < NW; ++w) total += sm.tot[0][w];
    __syncthreads();
    return total;
}

// Writes the selected rows of inputs [i0, i1) (masks from block_masks_pre) as 16-bit offsets
// from row 16*i0 (ascending)
// into a shared-memory list (peers of the cluster read it through DSMEM).
template <int NT>
__device__ void block_write_rows_local(const uint16_t* __restrict__ masks, int i0, int i1,
                                       uint16_t* __restrict__ rows_out, ScanShared<NT>& sm) {
    constexpr int NW = NT / 32;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int base = 0, round = 0;
    for (int ib = i0; ib < i1; ib += NT, ++round) {
        const int i = ib + tid;
        unsigned mask = (i < i1) ? masks[i - i0] : 0u;
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
        const int rbase = (i - i0) * 16;
        while (mask) {
            const int r = __ffs(mask) - 1;
            mask &= mask - 1u;
            rows_out[p++] = (uint16_t)(rbase + r);
        }
        base += total;
    }
    __syncthreads();
}

// ------------------------------------------------------------------ accumulation

template <int VEC>
struct VecLoad;
template <>
struct VecLoad<8> {
    using T = uint4;
    static IAM_DEV T load(const uint16_t* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
    static IAM_DEV T zero() { return make_uint4(0u, 0u, 0u, 0u); }
    static IAM_DEV uint32_t word(const T& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }
    static IAM_DEV uint32_t bits(const T& v, int k) {
        const uint32_t w = (k >> 1) == 0 ? v.x : (k >> 1) == 1 ? v.y : (k >> 1) == 2 ? v.z : v.w;
        return (k & 1) ? (w >> 16) : (w & 0xffffu);
    }
};
template <>
struct VecLoad<4> {
    using T = uint2;
    static IAM_DEV T load(const uint16_t* p) { return __ldg(reinterpret_cast<const uint2*>(p)); }
    static IAM_DEV T zero() { return make_uint2(0u, 0u); }
    static IAM_DEV uint32_t word(const T& v, int i) { return i == 0 ? v.x : v.y; }
    static IAM_DEV uint32_t bits(const T& v, int k) {
        const uint32_t w = (k >> 1) == 0 ? v.x : v.y;
        return (k & 1) ? (w >> 16) : (w & 0xffffu);
    }
};
template <>
struct VecLoad<2> {
    using T = uint32_t;
    static IAM_DEV T load(const uint16_t* p) { return __ldg(reinterpret_cast<const unsigned int*>(p)); }
    static IAM_DEV T zero() { return 0u; }
    static IAM_DEV uint32_t word(const T& v, int) { return v; }
    static IAM_DEV uint32_t bits(const T& v, int k) { return (k & 1) ? (v >> 16) : (v & 0xffffu); }
};
template <>
struct VecLoad<1> {
    using T = uint32_t;
    static IAM_DEV T load(const uint16_t* p) { return (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(p)); }
    static IAM_DEV T zero() { return 0u; }
    static IAM_DEV uint32_t word(const T& v, int) { return v; }
    static IAM_DEV uint32_t bits(const T& v, int) { return v; }
};

// Adds x * w_k into this lane's private slot accumulators, addressed in the shared window:
// acc_lane = the lane's float in a per-warp region aligned to its size (16 slots x VEC x 32
// lanes x 4 B = 16 << SS bytes), slot s / column k at acc_lane + s * (1 << SS) + k * 128.  The
// slot (low 4 bits of the fp16 word) becomes an address with one shift and one LOP3:
// ((word << SS) & (15 << SS)) | acc_lane (low half) or ((word >> (16 - SS)) & ...) (high half).
template <int VEC>
struct SlotShift {
    static constexpr int value = VEC == 8 ? 10 : VEC == 4 ? 9 : VEC == 2 ? 8 : 7;  // log2(VEC * 128)
};

// Volatile asm keeps these in program order among themselves (a later row may hit the same
// slot); the accumulators are only touched elsewhere across __syncthreads().  The column
// offset OFF rides in the instruction's immediate.
template <int OFF>
IAM_DEV float lds_f32(uint32_t a) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1+%2];" : "=f"(v) : "r"(a), "n"(OFF));
    return v;
}
template <int OFF>
IAM_DEV void sts_f32(uint32_t a, float v) {
    asm volatile("st.shared.f32 [%0+%1], %2;" ::"r"(a), "n"(OFF), "f"(v));
}

template <int VEC, int K>
IAM_DEV uint32_t slot_addr(const typename VecLoad<VEC>::T& w, uint32_t acc_lane) {
    constexpr int SS = SlotShift<VEC>::value;
    constexpr uint32_t M = 15u << SS;
    const uint32_t word = VecLoad<VEC>::word(w, K >> 1);
    return ((K & 1) ? ((word >> (16 - SS)) & M) : ((word << SS) & M)) | acc_lane;
}

template <int VEC, int... K>
IAM_DEV void accumulate_sh_impl(uint32_t acc_lane, const typename VecLoad<VEC>::T& w, float x,
                                std::integer_sequence<int, K...>) {
    const uint32_t a[VEC] = {slot_addr<VEC, K>(w, acc_lane)...};
    float old[VEC] = {lds_f32<K * 128>(a[K])...};  // braced lists evaluate left to right
    ((old[K] = fmaf(x, h2f(VecLoad<VEC>::bits(w, K)), old[K])), ...);
    (sts_f32<K * 128>(a[K], old[K]), ...);
}

template <int VEC>
IAM_DEV void accumulate_sh(uint32_t acc_lane, const typename VecLoad<VEC>::T& w, float x) {
    accumulate_sh_impl<VEC>(acc_lane, w, x, std::make_integer_sequence<int, VEC>{});
}


}  // namespace iam
