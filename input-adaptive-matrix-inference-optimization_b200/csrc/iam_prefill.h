// iam_prefill.h -- layer glue of the batched (dense) prefill: the per-token operations of the
// decode step applied to a chunk of prompt tokens at once, around the tensor-core products of
// iam_dense.h.  Activations are row-major [token][feature] fp32.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace iam {

// h[t][:] = float(embed[tokens[t]][:])  (tokens on the device)
int prefill_embed(const uint16_t* embed, int dim, const int* tokens, int n, float* h, cudaStream_t s);
// RMSNorm of every row (rmsNorm32fast order, aux.cl:156-196, then the gain, aux.cl:434-440),
// written as fp16 hi / lo halves [n][dim] for the dense products.
int prefill_rms_split(const float* h, int n, int dim, const uint16_t* gain, float eps, uint16_t* hi, uint16_t* lo,
                      cudaStream_t s);
// RoPE (rotate-half, aux.cl:227-248) of the q and k heads of every row of qkv [n][ld] (q heads,
// then k heads, then v heads); q rotated in place, k and v appended to the fp16 caches
// [kv_head][max_ctx][hd] at positions pos0 + t.
int prefill_rope_kv(float* qkv, int n, int ld, int n_heads, int n_kv, int hd, const float* rope, int pos0,
                    uint16_t* k_cache, uint16_t* v_cache, int max_ctx, cudaStream_t s);
// Causal attention: row t (position pos0 + t) over cache positions [0, pos0 + t], GQA (query
// head h reads kv head h / (n_heads / n_kv)); out [n][ldo].
int prefill_attention(const float* qkv, int ldq, int n, int n_heads, int n_kv, int hd, const uint16_t* k_cache,
                      const uint16_t* v_cache, int max_ctx, int pos0, float* out, int ldo, cudaStream_t s);
// a = up * gate / (1 + exp(-gate)) (silu32, matrix.cl:27-32) of gu [n][2 ffn] (gate columns
// first), written as fp16 hi / lo [n][ffn].
int prefill_silu_split(const float* gu, int n, int ffn, uint16_t* hi, uint16_t* lo, cudaStream_t s);

}  // namespace iam
