/*
 * iam_oracle.h -- CPU restatement of the reference's Effort-style bucketMul decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or calls this
 * code.  It is used by tests/ (as the parity checker), by __graft_entry__.smoke() (as the
 * checker) and by bench.py's cpu_baseline / --impl reference leg (as the timed CPU arm).
 *
 * Every function restates one piece of the reference (Guziuk/Input-Adaptive-Matrix-
 * Inference-Optimization) and cites the file:line it follows.  The reference's own code
 * for these steps is OpenCL C (bucketMul.cl, aux.cl, matrix.cl) and cannot be executed on
 * this image (no OpenCL headers, no ICD, no CPU OpenCL runtime), so this restatement is
 * the executable statement of the documented semantics.  Parity pinning:
 *   - the bucket layout (buckets / stats / probes) is pinned to the reference itself:
 *     tests/golden holds fixtures written by the reference's own Python function
 *     preprocess_layer_fixed_gpu.bucketize_fp16_packed, plus its verify_packing
 *     known-answer pairs;
 *   - the cutoff search, dispatch selection and accumulation are pinned only by this
 *     restatement and by an independent numpy restatement written into the same
 *     fixtures (tests/golden/make_golden.py): parity for those steps is "unpinned" against
 *     an executed reference, because none can run here.
 *
 * Generalisation beyond the reference (documented, never exercised by Mistral shapes):
 *   - probes_count = min(in_dim, 4096); the reference hard-codes 4096 and would read past
 *     the input for in_dim < 4096 (bucketMul.cl:106-110).
 */
#ifndef IAM_ORACLE_H
#define IAM_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORA_PROBES_COUNT 4096      /* bucketMul.cl:18, bucket_mul.hpp:101 */
#define ORA_CUTOFF_SCALE 100000.0f /* bucketMul.cl:17 */
#define ORA_MAX_ITERS 20           /* bucketMul.cl:148 */

/* ---- fp16 helpers (binary_loader.hpp:204-241) ---- */
float ora_half_to_float(uint16_t h);
uint16_t ora_float_to_half(float f); /* IEEE round-to-nearest-even */

/* ---- cutoff search (bucketMul.cl:68-214, bucket_mul.hpp:164) ---- */
int ora_probes_count(int in_dim);
int ora_target_count(float effort, int probes_count);
/* Returns the cutoff.  *iters (may be NULL) receives the number of bisection steps run. */
float ora_find_cutoff(const float* x, const uint16_t* probes, int probes_count, int target,
                      int* iters);

/* ---- dispatch selection (bucketMul.cl:351-386) ----
 * Selects bucket rows r in [row0, row0+expert_size) with r-row0 < 16*in_dim and
 * 1e5*|x[(r-row0)/16] * stats[r*stride + stride-1]| >= cutoff.  Rows are written in
 * ascending order (the reference's order is atomic-counter order; the SET is the same).
 * Returns the number of selected rows. */
long ora_prepare_dispatch(const float* x, const uint16_t* stats, int stats_stride, long row0,
                          long expert_size, int in_dim, float cutoff, int32_t* rows_out);

/* ---- bucketMul accumulation (bucketMul.cl:392-447) + integrate (:453-497) ----
 * out[c*16 + (w & 15)] += x[(row-row0)/16] * float(w), w = buckets[row*cols + c]
 * unmasked (the 4 slot bits stay in the multiplicand, bucketMul.cl:430-434).
 * out (16*cols floats) is overwritten.  nthreads > 1 splits columns over OpenMP threads
 * (per-output summation order is unchanged). */
void ora_bucket_mul(const uint16_t* buckets, int cols, const float* x, long row0,
                    const int32_t* rows, long count, float* out, int nthreads);

/* Whole operator (bucket_mul.hpp:254-267 fullMul).  rows_scratch holds expert_size ints.
 * Returns the selected row count; *cutoff_out (may be NULL) receives the cutoff. */
long ora_bucketmul_full(const float* x, const uint16_t* stats, int stats_stride,
                        const uint16_t* probes, const uint16_t* buckets, int expert_no,
                        int in_dim, int bucket_cols, long expert_size, float effort, float* out,
                        int32_t* rows_scratch, float* cutoff_out, int nthreads);

/* Dense fp64 GEMV on the original (unbucketed) fp16 weight W[M][N]: sanity reference. */
void ora_dense_gemv(const uint16_t* W, int M, int N, const float* x, double* out);

/* ---- layer glue (aux.cl, matrix.cl, attention.hpp) ---- */
/* rmsNorm32fast (aux.cl:156-196) followed by mul16x32 gain (aux.cl:434-440). */
void ora_rmsnorm(const float* x, int n, float eps, const uint16_t* gain, float* out);
/* RoPE table for one position (attention.hpp:207-235): cs[2*i]=cos, cs[2*i+1]=sin, i<hd/2 */
void ora_rope_table(int pos, int head_dim, double theta, float* cs);
/* rope_mx rotate-half (aux.cl:227-248) on n_heads contiguous heads. */
void ora_rope_apply(const float* in, int n_heads, int head_dim, const float* cs, float* out);
/* silu32 (matrix.cl:27-32): out = u * g / (1 + exp(-g)) */
void ora_silu_mul(const float* g, const float* u, int n, float* out);

typedef struct {
    int dim, n_layers, n_heads, n_kv_heads, head_dim, ffn_dim, vocab, max_ctx;
    float norm_eps;
    double rope_theta;
} ora_config;

typedef struct {
    const uint16_t* buckets; /* [16*in_dim][out_dim/16] */
    const uint16_t* stats;   /* [16*in_dim][stats_stride] */
    const uint16_t* probes;  /* [in_dim] */
    int in_dim, out_dim, stats_stride;
} ora_bm_weight;

typedef struct {
    const uint16_t* attn_norm; /* [dim] */
    const uint16_t* ffn_norm;  /* [dim] */
    ora_bm_weight wq, wk, wv, wo, w1, w2, w3; /* w1 = gate, w3 = up, w2 = down */
} ora_layer;

typedef struct {
    ora_config cfg;
    const uint16_t* embed;      /* [vocab][dim] */
    const uint16_t* final_norm; /* [dim] */
    const uint16_t* lm_head;    /* [vocab][dim]; equals embed when tied */
    const ora_layer* layers;
    uint16_t* k_cache; /* [n_layers][n_kv_heads][max_ctx][head_dim] fp16 */
    uint16_t* v_cache;
} ora_model;

/* Attention over the cache for one layer (attention.hpp:311-404; aux.cl:497-540 scores,
 * :204-225 softmax without max subtraction, :370-384 weighted V sum).  q is post-RoPE,
 * [n_heads][head_dim]; out is [n_heads][head_dim]. */
void ora_attention(const ora_config* cfg, const float* q, const uint16_t* k_layer,
                   const uint16_t* v_layer, int n_tokens, float* out);

/* matmul16x32 (aux.cl:454-490): logits[r] = sum_c W[r][c] * x[c]. */
void ora_lm_head(const uint16_t* W, int rows, int cols, const float* x, float* logits,
                 int nthreads);

/* One decode step, MistralModel::forward (model.hpp:152-231) with the layer order of
 * TransformerLayer::forward (transformer_layer.hpp:75-122).  Writes vocab logits and
 * returns the greedy argmax (first maximum, as std::max_element in test_generation.cpp:276).
 * sel_rows (may be NULL) accumulates the selected bucket rows of all 7*n_layers matmuls. */
int ora_model_forward(const ora_model* m, int token, int pos, float effort, float* logits,
                      long* sel_rows, int nthreads);

/* The same step with every bucket row of all 7*n_layers matmuls selected (no cutoff): the
 * product the dense tensor-core path computes (its prefill is checked against this, token by
 * token). */
int ora_model_forward_dense(const ora_model* m, int token, int pos, float* logits, int nthreads);

/* Size in floats of the scratch ora_model_forward allocates internally (for callers that
 * want to know the footprint). */
long ora_model_scratch_floats(const ora_config* cfg);

#ifdef __cplusplus
}
#endif

#endif /* IAM_ORACLE_H */
