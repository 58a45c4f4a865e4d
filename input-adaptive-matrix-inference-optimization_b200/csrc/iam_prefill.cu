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

constexpr int kAttnQ = 4;      // query tokens per CTA
constexpr int kAttnKT = 32;    // keys per shared-memory tile (one per lane in the score pass)

// One CTA per (kv head, block of kAttnQ query tokens): rows r = (token, query head of the
// group), RW rows per warp.  Per tile of 32 keys: the CTA stages K (rows padded to HD/2 + 1
// words: lane-per-key reads hit distinct banks) and V in shared memory; lane j scores key j
// against the warp's rows (no reductions inside the dot products); one max and one sum per
// row and tile update the running softmax; then each lane accumulates its VD dims of P V.
template <int VD, int RW>
__global__ void __launch_bounds__(256) prefill_attention_kernel(const float* __restrict__ qkv, int ldq, int n,
                                                                int n_heads, int n_kv,
                                                                const uint16_t* __restrict__ k_cache,
                                                                const uint16_t* __restrict__ v_cache, int max_ctx,
                                                                int pos0, float* __restrict__ out, int ldo) {
    constexpr int HD = 32 * VD;
    constexpr int KW = HD / 2 + 1;  // padded K row in 32-bit words
    extern __shared__ float sm[];
    const int gq = n_heads / n_kv;
    const int rows = kAttnQ * gq;
    float* s_q = sm;                                       // [rows][HD]
    uint32_t* s_k = reinterpret_cast<uint32_t*>(s_q + rows * HD);  // [KT][KW] half2 words
    uint32_t* s_v = s_k + kAttnKT * KW;                    // [KT][HD / 2] half2 words
    float* s_p = reinterpret_cast<float*>(s_v + kAttnKT * HD / 2);  // [warps][RW][KT]

    const int kvh = blockIdx.x, tb = blockIdx.y * kAttnQ;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nq = min(kAttnQ, n - tb);
    const int last_key = pos0 + tb + nq - 1;  // the block's last query sees keys [0, last_key]

    for (int e = threadIdx.x; e < rows * HD; e += blockDim.x) {
        const int r = e / HD, d = e % HD, ti = r / gq, g = r % gq;
        s_q[e] = ti < nq ? qkv[(size_t)(tb + ti) * ldq + (size_t)(kvh * gq + g) * HD + d] : 0.0f;
    }
    float mx[RW], l[RW], acc[RW][VD];
    int lastr[RW];
#pragma unroll
    for (int a = 0; a < RW; ++a) {
        const int r = warp * RW + a;
        mx[a] = -INFINITY;
        l[a] = 0.0f;
        lastr[a] = pos0 + tb + min(r / gq, nq - 1);
#pragma unroll
        for (int i = 0; i < VD; ++i) acc[a][i] = 0.0f;
    }
    const float inv_scale = sqrtf((float)HD);  // score = dot / sqrt(head_dim), aux.cl:537
    const uint16_t* kb = k_cache + (size_t)kvh * max_ctx * HD;
    const uint16_t* vb = v_cache + (size_t)kvh * max_ctx * HD;
    float* pw = s_p + warp * RW * kAttnKT;

    for (int k0 = 0; k0 <= last_key; k0 += kAttnKT) {
        __syncthreads();  // the previous tile is consumed (and s_q written, on the first pass)
        // stage K and V of keys [k0, k0 + 32) (rows past last_key read as zeros)
        for (int e = threadIdx.x; e < kAttnKT * HD / 8; e += blockDim.x) {
            const int j = e / (HD / 8), c = e % (HD / 8);
            uint4 kv4 = make_uint4(0, 0, 0, 0), vv4 = make_uint4(0, 0, 0, 0);
            if (k0 + j <= last_key) {
                kv4 = *reinterpret_cast<const uint4*>(kb + (size_t)(k0 + j) * HD + c * 8);
                vv4 = *reinterpret_cast<const uint4*>(vb + (size_t)(k0 + j) * HD + c * 8);
            }
            uint32_t* kr = s_k + j * KW + c * 4;
            kr[0] = kv4.x;
            kr[1] = kv4.y;
            kr[2] = kv4.z;
            kr[3] = kv4.w;
            *reinterpret_cast<uint4*>(s_v + j * (HD / 2) + c * 4) = vv4;
        }
        __syncthreads();
        if (warp * RW >= rows) continue;  // warps past the rows only help staging
        // scores: lane = key
        float sc[RW];
#pragma unroll
        for (int a = 0; a < RW; ++a) sc[a] = 0.0f;
        const uint32_t* kr = s_k + lane * KW;
        for (int w2 = 0; w2 < HD / 2; ++w2) {
            const uint32_t kw = kr[w2];
            const float k0f = h2f(kw & 0xffffu), k1f = h2f(kw >> 16);
#pragma unroll
            for (int a = 0; a < RW; ++a) {
                const float2 qv = *reinterpret_cast<const float2*>(s_q + (warp * RW + a) * HD + 2 * w2);
                sc[a] = fmaf(qv.x, k0f, sc[a]);
                sc[a] = fmaf(qv.y, k1f, sc[a]);
            }
        }
        const int key = k0 + lane;
#pragma unroll
        for (int a = 0; a < RW; ++a) {
            const float sv = key <= lastr[a] ? sc[a] / inv_scale : -INFINITY;
            float tm = sv;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, off));
            const float mn = fmaxf(mx[a], tm);  // finite: key 0 is in the first tile of every row
            const float c = expf(mx[a] - mn);
            const float pj = expf(sv - mn);
            float ps = pj;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
            l[a] = l[a] * c + ps;
            mx[a] = mn;
#pragma unroll
            for (int i = 0; i < VD; ++i) acc[a][i] *= c;
            pw[a * kAttnKT + lane] = pj;
        }
        __syncwarp();
        const int nk = min(kAttnKT, last_key - k0 + 1);
        for (int j = 0; j < nk; ++j) {
            float vf[VD];
            const uint32_t* vr = s_v + j * (HD / 2) + lane * (VD / 2);
#pragma unroll
            for (int i = 0; i < VD / 2; ++i) {
                vf[2 * i] = h2f(vr[i] & 0xffffu);
                vf[2 * i + 1] = h2f(vr[i] >> 16);
            }
#pragma unroll
            for (int a = 0; a < RW; ++a) {
                const float pj = pw[a * kAttnKT + j];
#pragma unroll
                for (int i = 0; i < VD; ++i) acc[a][i] = fmaf(pj, vf[i], acc[a][i]);
            }
        }
        __syncwarp();
    }
    if (warp * RW >= rows) return;
#pragma unroll
    for (int a = 0; a < RW; ++a) {
        const int r = warp * RW + a, ti = r / gq, g = r % gq;
        if (ti >= nq) continue;
        float* op = out + (size_t)(tb + ti) * ldo + (size_t)(kvh * gq + g) * HD + lane * VD;
#pragma unroll
        for (int i = 0; i < VD; ++i) op[i] = acc[a][i] / l[a];
    }
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

template <int VD, int RW>
int launch_attention_t(const float* qkv, int ldq, int n, int n_heads, int n_kv, const uint16_t* k_cache,
                       const uint16_t* v_cache, int max_ctx, int pos0, float* out, int ldo, cudaStream_t s) {
    constexpr int HD = 32 * VD;
    const int rows = kAttnQ * (n_heads / n_kv);
    const int warps = std::max(1, (rows + RW - 1) / RW);
    const size_t smem = (size_t)rows * HD * 4 + (size_t)kAttnKT * (HD / 2 + 1) * 4 + (size_t)kAttnKT * HD * 2 +
                        (size_t)warps * RW * kAttnKT * 4;
    if (warps > 8 || smem > 200 * 1024) return fail(IAM_ERR_UNSUPPORTED, "prefill attention: query group too large");
    auto kern = prefill_attention_kernel<VD, RW>;
    IAM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kern<<<dim3(n_kv, (n + kAttnQ - 1) / kAttnQ), 32 * warps, smem, s>>>(qkv, ldq, n, n_heads, n_kv, k_cache, v_cache,
                                                                         max_ctx, pos0, out, ldo);
    IAM_CUDA_TRY(cudaGetLastError());
    return IAM_OK;
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
    if (n_heads % n_kv != 0) return fail(IAM_ERR_UNSUPPORTED, "prefill attention: n_heads % n_kv_heads");
    if ((n + kAttnQ - 1) / kAttnQ > 65535) return fail(IAM_ERR_UNSUPPORTED, "prefill attention: tokens");
    // rows per warp: 8 warps when the block's rows fill them, else one row per warp
    const int rows = kAttnQ * (n_heads / n_kv);
    const bool two = rows % 16 == 0 && rows / 2 <= 8 * 2;
    switch (hd) {
        case 64:
            return two ? launch_attention_t<2, 2>(qkv, ldq, n, n_heads, n_kv, k_cache, v_cache, max_ctx, pos0, out, ldo, s)
                       : launch_attention_t<2, 1>(qkv, ldq, n, n_heads, n_kv, k_cache, v_cache, max_ctx, pos0, out, ldo, s);
        case 128:
            return two ? launch_attention_t<4, 2>(qkv, ldq, n, n_heads, n_kv, k_cache, v_cache, max_ctx, pos0, out, ldo, s)
                       : launch_attention_t<4, 1>(qkv, ldq, n, n_heads, n_kv, k_cache, v_cache, max_ctx, pos0, out, ldo, s);
        default:
            return fail(IAM_ERR_UNSUPPORTED, "prefill attention: head_dim must be 64 or 128");
    }
}

int prefill_silu_split(const float* gu, int n, int ffn, uint16_t* hi, uint16_t* lo, cudaStream_t s) {
    if (n <= 0) return IAM_OK;
    if (ffn % 4 || n > 65535) return fail(IAM_ERR_UNSUPPORTED, "prefill silu: ffn % 4 / tokens");
    silu_split_kernel<<<dim3((ffn / 4 + 255) / 256, n), 256, 0, s>>>(gu, ffn, hi, lo);
    IAM_CUDA_TRY(cudaGetLastError());
    return IAM_OK;
}

}  // namespace iam
