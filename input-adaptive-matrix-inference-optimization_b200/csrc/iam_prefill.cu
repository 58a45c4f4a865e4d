// iam_prefill.cu -- layer glue of the batched prefill (see iam_prefill.h).
//
// The arithmetic follows the decode step token by token: the RMSNorm sums in the
// rmsNorm32fast order (256 contiguous runs, then a halving tree, aux.cl:165-186) with every
// product and sum rounded on its own, RoPE multiplies and adds separately rounded
// (aux.cl:244-246), SiLU is u * g / (1 + exp(-g)) (matrix.cl:31).  Attention uses a running
// maximum (online softmax) where the reference exponentiates the raw scores (aux.cl:204-225):
// the same value up to rounding.
#include <math.h>

#include <algorithm>

#include "iam_common.cuh"
#include "iam_prefill.h"

namespace iam {

namespace {

IAM_DEV void split_store(float v, uint16_t* hi, uint16_t* lo, size_t o) {
    const __half h = __float2half_rn(v);
    hi[o] = __half_as_ushort(h);
    lo[o] = __half_as_ushort(__float2half_rn(__fsub_rn(v, __half2float(h))));
}

__global__ void __launch_bounds__(256) embed_rows_kernel(const uint16_t* __restrict__ embed, int dim,
                                                          const int* __restrict__ tokens, float* __restrict__ h) {
    const int t = blockIdx.x;
    const uint16_t* e = embed + (size_t)tokens[t] * dim;
    float* o = h + (size_t)t * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) o[i] = h2f(e[i]);
}

IAM_DEV void split_store4(float4 v, uint16_t* hi, uint16_t* lo, size_t o) {  // o % 4 == 0
    const __half h0 = __float2half_rn(v.x), h1 = __float2half_rn(v.y), h2 = __float2half_rn(v.z),
                 h3 = __float2half_rn(v.w);
    uint2 hv, lv;
    hv.x = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
    hv.y = (uint32_t)__half_as_ushort(h2) | ((uint32_t)__half_as_ushort(h3) << 16);
    lv.x = (uint32_t)__half_as_ushort(__float2half_rn(__fsub_rn(v.x, __half2float(h0)))) |
           ((uint32_t)__half_as_ushort(__float2half_rn(__fsub_rn(v.y, __half2float(h1)))) << 16);
    lv.y = (uint32_t)__half_as_ushort(__float2half_rn(__fsub_rn(v.z, __half2float(h2)))) |
           ((uint32_t)__half_as_ushort(__float2half_rn(__fsub_rn(v.w, __half2float(h3)))) << 16);
    *reinterpret_cast<uint2*>(hi + o) = hv;
    *reinterpret_cast<uint2*>(lo + o) = lv;
}

// One CTA per row.  The sum of squares: 256 runs of dim/256 contiguous elements, then the
// halving tree (levels 128..32 in shared memory, 16..1 with shuffles: the same pairs).
__global__ void __launch_bounds__(256) rms_split_kernel(const float* __restrict__ h, int dim,
                                                         const uint16_t* __restrict__ gain, float eps,
                                                         uint16_t* __restrict__ hi, uint16_t* __restrict__ lo) {
    __shared__ float part[256];
    __shared__ float s_scale;
    const int t = blockIdx.x, tid = threadIdx.x;
    const float* x = h + (size_t)t * dim;
    if (dim % 256 == 0) {
        const int e = dim / 256;
        float s = 0.0f;
        if (e % 4 == 0) {
            const float4* xv = reinterpret_cast<const float4*>(x + tid * e);
            for (int i = 0; i < e / 4; ++i) {
                const float4 v = xv[i];
                s = __fadd_rn(s, __fmul_rn(v.x, v.x));
                s = __fadd_rn(s, __fmul_rn(v.y, v.y));
                s = __fadd_rn(s, __fmul_rn(v.z, v.z));
                s = __fadd_rn(s, __fmul_rn(v.w, v.w));
            }
        } else {
            for (int i = tid * e; i < tid * e + e; ++i) s = __fadd_rn(s, __fmul_rn(x[i], x[i]));
        }
        part[tid] = s;
        __syncthreads();
        for (int st = 128; st >= 32; st >>= 1) {
            if (tid < st) part[tid] = __fadd_rn(part[tid], part[tid + st]);
            __syncthreads();
        }
        if (tid < 32) {
            float v = part[tid];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, off));
            if (tid == 0) part[0] = v;
        }
    } else if (tid == 0) {  // small widths: one running sum, as the reference's scalar path
        float s = 0.0f;
        for (int i = 0; i < dim; ++i) s = __fadd_rn(s, __fmul_rn(x[i], x[i]));
        part[0] = s;
    }
    __syncthreads();
    if (tid == 0) s_scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(part[0], (float)dim), eps)));
    __syncthreads();
    const float scale = s_scale;
    if (dim % 4 == 0) {
        for (int i = tid * 4; i < dim; i += 256 * 4) {
            const float4 xv = *reinterpret_cast<const float4*>(x + i);
            float4 v = make_float4(__fmul_rn(xv.x, scale), __fmul_rn(xv.y, scale), __fmul_rn(xv.z, scale),
                                   __fmul_rn(xv.w, scale));
            if (gain) {
                const uint2 g = *reinterpret_cast<const uint2*>(gain + i);
                v.x = __fmul_rn(h2f(g.x & 0xffffu), v.x);
                v.y = __fmul_rn(h2f(g.x >> 16), v.y);
                v.z = __fmul_rn(h2f(g.y & 0xffffu), v.z);
                v.w = __fmul_rn(h2f(g.y >> 16), v.w);
            }
            split_store4(v, hi, lo, (size_t)t * dim + i);
        }
    } else {
        for (int i = tid; i < dim; i += 256) {
            const float v = __fmul_rn(x[i], scale);
            split_store(gain ? __fmul_rn(h2f(gain[i]), v) : v, hi, lo, (size_t)t * dim + i);
        }
    }
}

// Grid (tokens, n_heads + 2 n_kv): block y < n_heads rotates query head y in place, the next
// n_kv rotate the key heads into the cache, the last n_kv copy the value heads.  hd / 2 threads.
__global__ void rope_kv_kernel(float* __restrict__ qkv, int ld, int n_heads, int n_kv, int hd,
                               const float* __restrict__ rope, int pos0, uint16_t* __restrict__ k_cache,
                               uint16_t* __restrict__ v_cache, int max_ctx) {
    const int t = blockIdx.x, head = blockIdx.y, d = threadIdx.x, p = pos0 + t, half = hd / 2;
    float* base = qkv + (size_t)t * ld + (size_t)head * hd;  // k heads follow the q heads, v the k
    if (head < n_heads + n_kv) {
        const float c = rope[((size_t)p * half + d) * 2], s = rope[((size_t)p * half + d) * 2 + 1];
        const float m0 = base[d], m1 = base[d + half];
        const float o0 = __fsub_rn(__fmul_rn(m0, c), __fmul_rn(m1, s));
        const float o1 = __fadd_rn(__fmul_rn(m1, c), __fmul_rn(m0, s));
        if (head < n_heads) {
            base[d] = o0;
            base[d + half] = o1;
        } else {
            uint16_t* kr = k_cache + ((size_t)(head - n_heads) * max_ctx + p) * hd;
            kr[d] = __half_as_ushort(__float2half_rn(o0));
            kr[d + half] = __half_as_ushort(__float2half_rn(o1));
        }
    } else {
        uint16_t* vr = v_cache + ((size_t)(head - n_heads - n_kv) * max_ctx + p) * hd;
        vr[d] = __half_as_ushort(__float2half_rn(base[d]));
        vr[d + half] = __half_as_ushort(__float2half_rn(base[d + half]));
    }
}

template <int VD>
IAM_DEV void load_halves(const uint16_t* p, float (&f)[VD]) {
    if constexpr (VD == 8) {
        const uint4 u = *reinterpret_cast<const uint4*>(p);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            f[2 * i] = h2f(w[i] & 0xffffu);
            f[2 * i + 1] = h2f(w[i] >> 16);
        }
    } else if constexpr (VD == 4) {
        const uint2 u = *reinterpret_cast<const uint2*>(p);
        f[0] = h2f(u.x & 0xffffu);
        f[1] = h2f(u.x >> 16);
        f[2] = h2f(u.y & 0xffffu);
        f[3] = h2f(u.y >> 16);
    } else if constexpr (VD == 2) {
        const uint32_t u = *reinterpret_cast<const uint32_t*>(p);
        f[0] = h2f(u & 0xffffu);
        f[1] = h2f(u >> 16);
    } else {
        f[0] = h2f(*p);
    }
}

constexpr int kKeysPerStep = 4;  // keys whose dot products reduce together (shuffle latency overlap)

// One CTA per (kv head, token), one warp per query head of the group; lane owns VD dims.
template <int VD>
__global__ void prefill_attention_kernel(const float* __restrict__ qkv, int ldq, int n_heads, int n_kv,
                                         const uint16_t* __restrict__ k_cache, const uint16_t* __restrict__ v_cache,
                                         int max_ctx, int pos0, float* __restrict__ out, int ldo) {
    constexpr int HD = 32 * VD;
    const int kvh = blockIdx.x, t = blockIdx.y;
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = kvh * (n_heads / n_kv) + w;
    const int last = pos0 + t;
    float q[VD];
    const float* qp = qkv + (size_t)t * ldq + (size_t)h * HD + lane * VD;
#pragma unroll
    for (int i = 0; i < VD; ++i) q[i] = qp[i];
    const uint16_t* kb = k_cache + (size_t)kvh * max_ctx * HD + lane * VD;
    const uint16_t* vb = v_cache + (size_t)kvh * max_ctx * HD + lane * VD;
    const float inv_scale = sqrtf((float)HD);  // score = dot / sqrt(head_dim), aux.cl:537
    float mx = -INFINITY, l = 0.0f, acc[VD];
#pragma unroll
    for (int i = 0; i < VD; ++i) acc[i] = 0.0f;
    for (int j0 = 0; j0 <= last; j0 += kKeysPerStep) {
        float kf[kKeysPerStep][VD], vf[kKeysPerStep][VD], s[kKeysPerStep];
#pragma unroll
        for (int u = 0; u < kKeysPerStep; ++u) {
            const int j = min(j0 + u, last);  // keys past the last are loaded clamped and skipped
            load_halves<VD>(kb + (size_t)j * HD, kf[u]);
            load_halves<VD>(vb + (size_t)j * HD, vf[u]);
        }
#pragma unroll
        for (int u = 0; u < kKeysPerStep; ++u) {
            s[u] = 0.0f;
#pragma unroll
            for (int i = 0; i < VD; ++i) s[u] = fmaf(q[i], kf[u][i], s[u]);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
#pragma unroll
            for (int u = 0; u < kKeysPerStep; ++u) s[u] += __shfl_xor_sync(0xffffffffu, s[u], off);
#pragma unroll
        for (int u = 0; u < kKeysPerStep; ++u) {
            if (j0 + u <= last) {  // uniform over the warp
                const float sc = s[u] / inv_scale;
                const float mn = fmaxf(mx, sc);
                const float c = expf(mx - mn), pe = expf(sc - mn);
                l = l * c + pe;
#pragma unroll
                for (int i = 0; i < VD; ++i) acc[i] = acc[i] * c + pe * vf[u][i];
                mx = mn;
            }
        }
    }
    float* op = out + (size_t)t * ldo + (size_t)h * HD + lane * VD;
#pragma unroll
    for (int i = 0; i < VD; ++i) op[i] = acc[i] / l;
}

// Grid (column blocks of 4 x 256, tokens); ffn % 4 == 0.
__global__ void __launch_bounds__(256) silu_split_kernel(const float* __restrict__ gu, int ffn,
                                                          uint16_t* __restrict__ hi, uint16_t* __restrict__ lo) {
    const int t = blockIdx.y;
    const int i = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (i >= ffn) return;
    const float4 g = *reinterpret_cast<const float4*>(gu + (size_t)t * 2 * ffn + i);
    const float4 u = *reinterpret_cast<const float4*>(gu + (size_t)t * 2 * ffn + ffn + i);
    const float4 a = make_float4(__fdiv_rn(__fmul_rn(u.x, g.x), __fadd_rn(1.0f, expf(-g.x))),
                                 __fdiv_rn(__fmul_rn(u.y, g.y), __fadd_rn(1.0f, expf(-g.y))),
                                 __fdiv_rn(__fmul_rn(u.z, g.z), __fadd_rn(1.0f, expf(-g.z))),
                                 __fdiv_rn(__fmul_rn(u.w, g.w), __fadd_rn(1.0f, expf(-g.w))));
    split_store4(a, hi, lo, (size_t)t * ffn + i);
}

}  // namespace

int prefill_embed(const uint16_t* embed, int dim, const int* tokens, int n, float* h, cudaStream_t s) {
    if (n <= 0) return IAM_OK;
    embed_rows_kernel<<<n, 256, 0, s>>>(embed, dim, tokens, h);
    IAM_CUDA_TRY(cudaGetLastError());
    return IAM_OK;
}

int prefill_rms_split(const float* h, int n, int dim, const uint16_t* gain, float eps, uint16_t* hi, uint16_t* lo,
                      cudaStream_t s) {
    if (n <= 0) return IAM_OK;
    rms_split_kernel<<<n, 256, 0, s>>>(h, dim, gain, eps, hi, lo);
    IAM_CUDA_TRY(cudaGetLastError());
    return IAM_OK;
}

int prefill_rope_kv(float* qkv, int n, int ld, int n_heads, int n_kv, int hd, const float* rope, int pos0,
                    uint16_t* k_cache, uint16_t* v_cache, int max_ctx, cudaStream_t s) {
    if (n <= 0) return IAM_OK;
    if (hd % 2 || hd / 2 > 1024 || n > 65535) return fail(IAM_ERR_UNSUPPORTED, "prefill rope: head_dim / tokens");
    rope_kv_kernel<<<dim3(n, n_heads + 2 * n_kv), hd / 2, 0, s>>>(qkv, ld, n_heads, n_kv, hd, rope, pos0, k_cache,
                                                                 v_cache, max_ctx);
    IAM_CUDA_TRY(cudaGetLastError());
    return IAM_OK;
}

int prefill_attention(const float* qkv, int ldq, int n, int n_heads, int n_kv, int hd, const uint16_t* k_cache,
                      const uint16_t* v_cache, int max_ctx, int pos0, float* out, int ldo, cudaStream_t s) {
    if (n <= 0) return IAM_OK;
    const int gq = n_heads / n_kv;
    if (n_heads % n_kv != 0 || gq > 32) return fail(IAM_ERR_UNSUPPORTED, "prefill attention: query group size");
    const dim3 grid(n_kv, n), block(32 * gq);
    switch (hd) {
        case 32: prefill_attention_kernel<1><<<grid, block, 0, s>>>(qkv, ldq, n_heads, n_kv, k_cache, v_cache, max_ctx, pos0, out, ldo); break;
        case 64: prefill_attention_kernel<2><<<grid, block, 0, s>>>(qkv, ldq, n_heads, n_kv, k_cache, v_cache, max_ctx, pos0, out, ldo); break;
        case 128: prefill_attention_kernel<4><<<grid, block, 0, s>>>(qkv, ldq, n_heads, n_kv, k_cache, v_cache, max_ctx, pos0, out, ldo); break;
        case 256: prefill_attention_kernel<8><<<grid, block, 0, s>>>(qkv, ldq, n_heads, n_kv, k_cache, v_cache, max_ctx, pos0, out, ldo); break;
        default: return fail(IAM_ERR_UNSUPPORTED, "prefill attention: head_dim must be 32, 64, 128 or 256");
    }
    IAM_CUDA_TRY(cudaGetLastError());
    return IAM_OK;
}

int prefill_silu_split(const float* gu, int n, int ffn, uint16_t* hi, uint16_t* lo, cudaStream_t s) {
    if (n <= 0) return IAM_OK;
    if (ffn % 4 || n > 65535) return fail(IAM_ERR_UNSUPPORTED, "prefill silu: ffn % 4 / tokens");
    silu_split_kernel<<<dim3((ffn / 4 + 255) / 256, n), 256, 0, s>>>(gu, ffn, hi, lo);
    IAM_CUDA_TRY(cudaGetLastError());
    return IAM_OK;
}

}  // namespace iam
