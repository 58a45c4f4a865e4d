// iam_layers.cu -- the decode-step kernels around bucketMul (sm_100a):
//   * embedding row gather (fetchRow16to32, aux.cl:442-452);
//   * decode attention: RoPE (rope_mx, aux.cl:227-248, with the host table of
//     attention.hpp:207-235), fp16 GQA KV-cache append (attention.hpp:281-309) and
//     split-K attention over the cache (dotSetScore2 / softmax / sumScores32,
//     aux.cl:497-540, :204-225, :370-384) for all query heads of one KV head at once;
//   * final RMSNorm * gain (aux.cl:156-196, :301-306), dense LM head GEMV (matmul16x32,
//     aux.cl:454-490) and the greedy argmax of the driver (test_generation.cpp:276).
// RMSNorm, SiLU and the residual adds live inside the bucketMul kernel (input providers and
// epilogue); see iam_bucketmul.cu.
#include <cfloat>

#include "iam_bucketmul.cuh"
#include "iam_layers.h"

namespace iam {

// ------------------------------------------------------------------ embedding

// x = float(embed[token]); token from `token_arg` or, when `token_key` is given, from the
// previous step's argmax key.  Also clears `argmax_key` for this step's LM head.
__global__ void embed_kernel(const uint16_t* __restrict__ embed, int dim, int token_arg,
                             const unsigned long long* token_key, const int* token_dev, float* __restrict__ x,
                             unsigned long long* argmax_key, int* token_used) {
    int token = token_arg;
    if (token_key) token = (int)(0xffffffffu - (unsigned)(*token_key & 0xffffffffull));
    else if (token_dev) token = *token_dev;
    const uint16_t* row = embed + (size_t)token * dim;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x) x[i] = h2f(row[i]);
    __syncthreads();
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        if (token_used) *token_used = token;
        if (argmax_key && token_key != argmax_key) *argmax_key = 0ull;
    }
}

// Clears the argmax slot (used when the embedding read its token from the same slot).
__global__ void clear_key_kernel(unsigned long long* key) { *key = 0ull; }

// ------------------------------------------------------------------ attention

// RoPE of one head (rotate-half, aux.cl:243-247) with separately rounded products.
IAM_DEV float rope_at(const float* m, const float* cs, int d, int half) {
    const int f = d % half;
    const float c = cs[2 * f], s = cs[2 * f + 1];
    if (d < half) return __fsub_rn(__fmul_rn(m[d], c), __fmul_rn(m[d + half], s));
    return __fadd_rn(__fmul_rn(m[d], c), __fmul_rn(m[d - half], s));
}

// grid = n_kv_heads * n_split, block = kAttnThreads.  CTA (kvh, s) handles context tokens
// [s*chunk, (s+1)*chunk) for the GQ query heads that share KV head kvh.
template <int GQ>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(AttnParams p) {
    extern __shared__ __align__(16) float sm[];
    const int hd = p.head_dim, half = hd / 2;
    const int kvh = blockIdx.x / p.n_split, s = blockIdx.x % p.n_split;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NWA = kAttnThreads / 32;
    const int pos = *p.pos_dev;
    const int n_tok = pos + 1;
    const int chunk = (n_tok + p.n_split - 1) / p.n_split;
    const int t0 = min(s * chunk, n_tok), t1 = min(t0 + chunk, n_tok);
    const int nt = t1 - t0;

    float* qr = sm;                  // [GQ][hd] roped queries
    float* knew = qr + GQ * hd;      // [hd] roped k at pos, rounded through fp16
    float* vnew = knew + hd;         // [hd] v at pos, rounded through fp16
    float* sc = vnew + hd;           // [GQ][chunk_cap] scores, then probabilities
    const float* cs = p.rope + (size_t)pos * hd;  // [hd/2][2]

    for (int e = tid; e < GQ * hd; e += kAttnThreads) {
        const int j = e / hd, d = e % hd;
        qr[e] = rope_at(p.q + (size_t)(kvh * GQ + j) * hd, cs, d, half);
    }
    for (int d = tid; d < hd; d += kAttnThreads) {
        knew[d] = __half2float(__float2half_rn(rope_at(p.k + (size_t)kvh * hd, cs, d, half)));
        vnew[d] = __half2float(__float2half_rn(p.v[(size_t)kvh * hd + d]));
    }
    uint16_t* kc = p.k_cache + (size_t)kvh * p.max_ctx * hd;
    uint16_t* vc = p.v_cache + (size_t)kvh * p.max_ctx * hd;
    __syncthreads();
    if (pos >= t0 && pos < t1) {  // the CTA whose chunk holds pos appends the new k/v
        for (int d = tid; d < hd; d += kAttnThreads) {
            kc[(size_t)pos * hd + d] = __half_as_ushort(__float2half_rn(knew[d]));
            vc[(size_t)pos * hd + d] = __half_as_ushort(__float2half_rn(vnew[d]));
        }
    }

    // scores: one warp per token, lanes split the head dimension
    const float inv = sqrtf((float)hd);
    for (int t = warp; t < nt; t += NWA) {
        const int tok = t0 + t;
        float dot[GQ];
#pragma unroll
        for (int j = 0; j < GQ; ++j) dot[j] = 0.0f;
        for (int d = lane; d < hd; d += 32) {
            const float kv = (tok == pos) ? knew[d] : h2f(kc[(size_t)tok * hd + d]);
#pragma unroll
            for (int j = 0; j < GQ; ++j) dot[j] = fmaf(qr[j * hd + d], kv, dot[j]);
        }
#pragma unroll
        for (int j = 0; j < GQ; ++j) {
            float v = dot[j];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) sc[j * p.chunk_cap + t] = __fdiv_rn(v, inv);  // q.k / sqrt(hd)
        }
    }
    __syncthreads();

    // per head: max, exp, sum (one warp per head)
    float* stat = p.part + ((size_t)(kvh * p.n_split + s) * GQ) * (hd + 2);
    for (int j = warp; j < GQ; j += NWA) {
        float m = -INFINITY;
        for (int t = lane; t < nt; t += 32) m = fmaxf(m, sc[j * p.chunk_cap + t]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float l = 0.0f;
        for (int t = lane; t < nt; t += 32) {
            const float e = nt ? expf(sc[j * p.chunk_cap + t] - m) : 0.0f;
            sc[j * p.chunk_cap + t] = e;
            l += e;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) {
            stat[j * (hd + 2)] = m;
            stat[j * (hd + 2) + 1] = l;
        }
    }
    __syncthreads();

    // unnormalised p.V for the chunk
    for (int e = tid; e < GQ * hd; e += kAttnThreads) {
        const int j = e / hd, d = e % hd;
        float o = 0.0f;
        for (int t = 0; t < nt; ++t) {
            const int tok = t0 + t;
            const float vv = (tok == pos) ? vnew[d] : h2f(vc[(size_t)tok * hd + d]);
            o = fmaf(sc[j * p.chunk_cap + t], vv, o);
        }
        stat[j * (hd + 2) + 2 + d] = o;
    }

    // last CTA of this KV head combines the splits in split order
    __threadfence();
    __syncthreads();
    __shared__ int last;
    if (tid == 0) last = (atomicAdd(p.ctr + kvh, 1) == p.n_split - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    const float* base = p.part + (size_t)kvh * p.n_split * GQ * (hd + 2);
    for (int e = tid; e < GQ * hd; e += kAttnThreads) {
        const int j = e / hd, d = e % hd;
        float M = -INFINITY;
        for (int r = 0; r < p.n_split; ++r) M = fmaxf(M, __ldcg(base + ((size_t)r * GQ + j) * (hd + 2)));
        float L = 0.0f, O = 0.0f;
        for (int r = 0; r < p.n_split; ++r) {
            const float* st = base + ((size_t)r * GQ + j) * (hd + 2);
            const float mr = __ldcg(st);
            if (mr == -INFINITY) continue;
            const float w = expf(mr - M);
            L = fmaf(w, __ldcg(st + 1), L);
            O = fmaf(w, __ldcg(st + 2 + d), O);
        }
        p.out[(size_t)(kvh * GQ + j) * hd + d] = __fdiv_rn(O, L);
    }
    if (tid == 0) p.ctr[kvh] = 0;  // ready for the next launch
}

// ------------------------------------------------------------------ LM head

// Orderable key of (logit, index): larger logit wins, then the smaller index.
IAM_DEV unsigned long long argmax_key(float v, int idx) {
    const unsigned u = __float_as_uint(v);
    const unsigned ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)ord << 32) | (unsigned long long)(0xffffffffu - (unsigned)idx);
}

// logits[r] = sum_c W[r][c] * xf[c], xf = rmsnorm(x) * gain; one warp per row, rows strided
// over the grid; also folds the greedy argmax into *argmax_key with atomicMax.
__global__ void __launch_bounds__(kHeadThreads) lm_head_kernel(LMHeadParams p) {
    extern __shared__ __align__(16) float xf[];
    __shared__ float red[256];
    __shared__ unsigned long long wbest[kHeadThreads / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NWH = kHeadThreads / 32;
    const float scale = block_rms_scale<kHeadThreads>(p.x, p.dim, p.eps, red);
    for (int i = tid; i < p.dim; i += kHeadThreads) xf[i] = __fmul_rn(__fmul_rn(p.x[i], scale), h2f(p.gain[i]));
    __syncthreads();
    unsigned long long best = 0ull;
    const int vec_ok = (p.dim % 256 == 0);
    for (int r = blockIdx.x * NWH + warp; r < p.rows; r += gridDim.x * NWH) {
        const uint16_t* w = p.W + (size_t)r * p.dim;
        float acc0 = 0.0f, acc1 = 0.0f;
        if (vec_ok) {
            for (int c = lane * 8; c < p.dim; c += 256) {
                const uint4 v = __ldcs(reinterpret_cast<const uint4*>(w + c));
                const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    acc0 = fmaf(h2f(wd[e] & 0xffffu), xf[c + 2 * e], acc0);
                    acc1 = fmaf(h2f(wd[e] >> 16), xf[c + 2 * e + 1], acc1);
                }
            }
        } else {
            for (int c = lane; c < p.dim; c += 32) acc0 = fmaf(h2f(w[c]), xf[c], acc0);
        }
        float v = acc0 + acc1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) {
            if (p.logits) p.logits[r] = v;
            const unsigned long long k = argmax_key(v, r);
            best = k > best ? k : best;
        }
    }
    if (lane == 0) wbest[warp] = best;
    __syncthreads();
    if (tid == 0 && p.argmax_key) {
        unsigned long long b = 0ull;
        for (int w2 = 0; w2 < NWH; ++w2) b = wbest[w2] > b ? wbest[w2] : b;
        atomicMax(p.argmax_key, b);
    }
}

// pos += 1 after a generated step, and the chosen token appended to tokens_out[*count].
__global__ void advance_kernel(int* pos, const unsigned long long* key, int* tokens_out, int* count) {
    if (tokens_out) tokens_out[*count] = (int)(0xffffffffu - (unsigned)(*key & 0xffffffffull));
    if (count) *count += 1;
    *pos += 1;
}

// ------------------------------------------------------------------ host launchers

int launch_embed(const uint16_t* embed, int dim, int token, const unsigned long long* token_key,
                 const int* token_dev, float* x, unsigned long long* argmax_key, int* token_used, cudaStream_t s) {
    embed_kernel<<<(dim + 1023) / 1024, 1024, 0, s>>>(embed, dim, token, token_key, token_dev, x, argmax_key,
                                                       token_used);
    IAM_CUDA_TRY(cudaGetLastError());
    if (argmax_key && token_key == argmax_key) {
        clear_key_kernel<<<1, 1, 0, s>>>(argmax_key);
        IAM_CUDA_TRY(cudaGetLastError());
    }
    return IAM_OK;
}

size_t attention_smem(const AttnParams& p, int gq) {
    return sizeof(float) * ((size_t)gq * p.head_dim + 2 * p.head_dim + (size_t)gq * p.chunk_cap);
}

int launch_attention(const AttnParams& p, int gq, cudaStream_t s) {
    const size_t smem = attention_smem(p, gq);
    const dim3 grid((unsigned)(p.n_kv_heads * p.n_split));
    switch (gq) {
#define IAM_ATTN_CASE(N)                                                                                   \
    case N:                                                                                                \
        if (smem > 48 * 1024)                                                                              \
            IAM_CUDA_TRY(cudaFuncSetAttribute(attention_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                              (int)smem));                                                 \
        attention_kernel<N><<<grid, kAttnThreads, smem, s>>>(p);                                           \
        break;
        IAM_ATTN_CASE(1)
        IAM_ATTN_CASE(2)
        IAM_ATTN_CASE(4)
        IAM_ATTN_CASE(8)
#undef IAM_ATTN_CASE
        default:
            return fail(IAM_ERR_UNSUPPORTED, "attention: n_heads / n_kv_heads must be 1, 2, 4 or 8");
    }
    IAM_CUDA_TRY(cudaGetLastError());
    return IAM_OK;
}

int launch_lm_head(const LMHeadParams& p, int grid, cudaStream_t s) {
    const size_t smem = sizeof(float) * (size_t)p.dim;
    if (smem > 48 * 1024)
        IAM_CUDA_TRY(cudaFuncSetAttribute(lm_head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    lm_head_kernel<<<grid, kHeadThreads, smem, s>>>(p);
    IAM_CUDA_TRY(cudaGetLastError());
    return IAM_OK;
}

int launch_advance(int* pos, const unsigned long long* key, int* tokens_out, int* count, cudaStream_t s) {
    advance_kernel<<<1, 1, 0, s>>>(pos, key, tokens_out, count);
    IAM_CUDA_TRY(cudaGetLastError());
    return IAM_OK;
}

}  // namespace iam
