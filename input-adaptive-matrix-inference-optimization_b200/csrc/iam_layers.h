// iam_layers.h -- launch descriptions of the decode-step kernels in iam_layers.cu.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "iam_tp.h"

namespace iam {

constexpr int kAttnThreads = 256;   // 16 half-warps
constexpr int kAttnTU = 2;          // tokens per half-warp in flight
constexpr int kAttnMinChunk = 32;   // context tokens per CTA at least (default of AttnParams::min_chunk)
constexpr int kAttnLaneMinCtx = 2048;   // default of AttnParams::lane_min_ctx
constexpr int kAttnLaneShortMax = 256;  // default of AttnParams::lane_short_max (8 warps x 32 tokens)
constexpr int kHeadThreads = 256;

struct AttnParams {
    const float* q;        // [n_heads][head_dim] pre-RoPE (bucketMul output)
    const float* k;        // [n_kv_heads][head_dim] pre-RoPE
    const float* v;        // [n_kv_heads][head_dim]
    uint16_t* k_cache;     // this layer: [n_kv_heads][max_ctx][head_dim] fp16, post-RoPE
    uint16_t* v_cache;     // this layer: [n_kv_heads][max_ctx][head_dim] fp16
    const float* rope;     // [max_ctx][head_dim/2][2] cos, sin
    const int* pos_dev;    // position of the token being decoded (context = pos + 1)
    int* pos_err;          // set when pos_dev holds max_ctx or more (the step is clamped), may be null
    float* out;            // [n_heads][head_dim]
    float* part;           // scratch [n_kv_heads][n_split][gq][head_dim + 2]
    int* ctr;              // [n_kv_heads] zero-initialised, self-resetting
    int n_kv_heads, head_dim, max_ctx, n_split;
    int min_chunk;         // context tokens per CTA at least
    int lane_min_ctx;      // contexts of this many tokens or more take the tensor-core layout,
    int lane_short_max;    // and so do contexts of at most this many (in one chunk per KV head)
    int tp_push;           // tensor parallel: head outputs at global index push_begin + i below
    int push_begin;        // push_limit also go to every peer's mailbox (kTpPushHeads)
    int push_limit;
    TpWindow tp;
};

struct LMHeadParams {
    const uint16_t* W;               // [rows][dim] fp16
    const float* x;                  // [dim] residual stream
    const uint16_t* gain;            // [dim] final norm gain
    float eps;
    int dim, rows;
    float* logits;                   // [rows] (may be null)
    unsigned long long* argmax_key;  // greedy argmax (may be null)
    int row0;                        // vocabulary index of row 0 (vocab-sharded LM head)
};

int launch_embed(const uint16_t* embed, int dim, int token, const unsigned long long* token_key,
                 const int* token_dev, float* x, unsigned long long* argmax_key, int* token_used, cudaStream_t s,
                 bool pdl = false);
size_t attention_smem(const AttnParams& p, int gq);
// pdl: launch with programmatic stream serialization (see launch_ex)
int launch_attention(const AttnParams& p, int gq, cudaStream_t s, bool pdl = false);
int launch_lm_head(const LMHeadParams& p, int grid, cudaStream_t s, bool pdl = false);
int launch_advance(int* pos, const unsigned long long* key, int* tokens_out, int* count, int max_ctx, cudaStream_t s,
                   bool pdl = false);

}  // namespace iam
