/*
 * iam_b200.h -- C ABI of libiamb200.so, the B200 (sm_100a) implementation of the
 * Effort-style dynamic-sparse decode path of Guziuk/Input-Adaptive-Matrix-Inference-
 * Optimization.
 *
 * Conventions (all entry points):
 *   - every function returns an int status (IAM_OK = 0, else an IAM_ERR_* code);
 *     iam_last_error() returns a message for the calling thread's last failure;
 *   - pointers named *_dev are device pointers owned by the caller; nothing here
 *     frees or keeps them beyond the documented lifetime;
 *   - work is enqueued on the given cudaStream_t (passed as void*, 0 = legacy default)
 *     and is asynchronous; nothing synchronises unless documented;
 *   - a handle (iam_bucketmul_t, iam_model_t) owns its scratch memory, so one handle per
 *     stream is safe; a single handle is not re-entrant across streams (the reference's
 *     singleton BucketMul::shared is not re-entrant either, bucket_mul.hpp:119-122).
 *
 * Bucket weight layout (the reference's on-disk contract, preprocess_layer_fixed_gpu.py:
 * 110-282): for W[out_dim][in_dim] fp16, C = out_dim/16 bucket columns and R = 16*in_dim
 * bucket rows; buckets[R][C] u16 where row i*16+r holds the rank-r (|w| descending) value
 * of each 16-output bucket with its original slot in the low 4 mantissa bits; stats[R][4]
 * u16 fp16 mean |value| per bucket row (channel 3 is used, bucketMul.cl:372); probes[in_dim]
 * u16 fp16 mean |W[:,i]|.  stats_stride = 4 reads that file layout directly, 1 reads a
 * packed channel-3 array (iam_stats_pack).
 */
#ifndef IAM_B200_H
#define IAM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    IAM_OK = 0,
    IAM_ERR_ARG = 1,      /* invalid argument */
    IAM_ERR_IO = 2,       /* missing / truncated / malformed weight file */
    IAM_ERR_CUDA = 3,     /* CUDA runtime or launch error */
    IAM_ERR_NCCL = 4,     /* NCCL error */
    IAM_ERR_TIMEOUT = 5,  /* a bounded device-side wait gave up */
    IAM_ERR_UNSUPPORTED = 6,
    IAM_ERR_NOMEM = 7
};

#define IAM_PROBES_COUNT 4096 /* bucket_mul.hpp:101, bucketMul.cl:18 */

/* Library identity and last error of the calling host thread. */
const char* iam_version(void);
const char* iam_last_error(void);
/* Number of SMs and the sm_XY of `device`; fails with IAM_ERR_UNSUPPORTED off sm_100. */
int iam_device_info(int device, int* sm_count, int* cc_major, int* cc_minor);

/* Diagnostics: resident clusters of `cluster_size` CTAs for the fused bucketMul kernel with
 * vec-wide loads (8, 4 or 1) on the current device, and the plan chosen for one bucketMul of
 * bucket_cols columns and in_dim inputs: log2 of lanes per row slice, column tiles, and input
 * splits (clusters per column tile). */
int iam_bucketmul_plan_info(int vec, int cluster_size, int bucket_cols, int in_dim,
                            int* max_active_clusters, int* log2_lanes, int* n_tiles,
                            int* n_splits);

/* ------------------------------------------------------------------ bucketMul operator */
/* Replaces the BucketMul singleton (bucket_mul.hpp:99-268).  The handle owns what the
 * singleton owned (dispatch list, cutoff, counts), sized on demand. */
typedef struct iam_bucketmul_s* iam_bucketmul_t;

/* BucketMul::shared (bucket_mul.hpp:119-136). */
int iam_bucketmul_create(iam_bucketmul_t* out, int device);
int iam_bucketmul_destroy(iam_bucketmul_t h);

/* findCutoffBinarySearch alone (bucketMul.cl:68-214 with the quantile of bucket_mul.hpp:164):
 * writes the cutoff (fp32) to cutoff_dev[0] and the number of bisection steps to
 * iters_dev[0] (iters_dev may be NULL).  Uses x[0:min(in_dim,4096)] and
 * probes[expert_no*4096 + i]. */
int iam_bucketmul_cutoff(iam_bucketmul_t h, const float* x_dev, const uint16_t* probes_dev,
                         int expert_no, int in_dim, float effort, float* cutoff_dev,
                         int* iters_dev, void* stream);

/* BucketMul::calcDispatch (bucket_mul.hpp:147-191): cutoff + prepareDispatch
 * (bucketMul.cl:351-386) into the handle's dispatch list.  Rows are kept in ascending
 * row order (the reference's order is its atomic counter's; the selected SET is equal).
 * stats_stride is 4 for the file layout, 1 for a packed channel-3 array. */
int iam_bucketmul_calc_dispatch(iam_bucketmul_t h, const float* x_dev, const uint16_t* stats_dev,
                                int stats_stride, const uint16_t* probes_dev, int expert_no,
                                int in_dim, int bucket_cols, int expert_size, float effort,
                                void* stream);

/* Copies the current dispatch list out of the handle: rows_dev (capacity >= expert_size)
 * receives the selected bucket-row indices in ascending order, count_dev[0] their number,
 * cutoff_dev[0] the cutoff.  Any pointer may be NULL. */
int iam_bucketmul_read_dispatch(iam_bucketmul_t h, int32_t* rows_dev, int* count_dev,
                                float* cutoff_dev, void* stream);

/* BucketMul::mul (bucket_mul.hpp:193-252): bucketMul (bucketMul.cl:392-447) + integrate
 * (:453-497) over the handle's dispatch list.  out_dev receives 16*bucket_cols floats
 * (overwritten, not accumulated).  bucket_rows = rows of the full buckets tensor. */
int iam_bucketmul_mul(iam_bucketmul_t h, const uint16_t* buckets_dev, int bucket_rows,
                      int bucket_cols, float* out_dev, void* stream);

/* BucketMul::fullMul (bucket_mul.hpp:254-267) as ONE fused launch: cutoff, selection,
 * accumulation and integrate in the same kernel (one wave of at most one CTA per SM that
 * meets at a grid-wide barrier; nothing else may keep every SM of the device busy while it
 * runs).  count_dev (may be NULL) receives the number of selected bucket rows, cutoff_dev
 * (may be NULL) the cutoff. */
int iam_bucketmul_full(iam_bucketmul_t h, const float* x_dev, const uint16_t* stats_dev,
                       int stats_stride, const uint16_t* probes_dev, const uint16_t* buckets_dev,
                       int expert_no, int in_dim, int bucket_cols, int expert_size, float effort,
                       float* out_dev, int* count_dev, float* cutoff_dev, void* stream);
/* Synchronises the device; IAM_ERR_TIMEOUT when an iam_bucketmul_full launch of `h` gave up
 * waiting at its grid barrier (its outputs are then invalid), IAM_OK otherwise.  (No
 * counterpart in the reference.) */
int iam_bucketmul_status(iam_bucketmul_t h);

/* Diagnostics: every later iam_bucketmul_full of `h` writes the 16 trace slots (below) of
 * its first CTA to times_dev[0..15].  NULL turns it off. */
int iam_bucketmul_phase_times(iam_bucketmul_t h, long long* times_dev);

/* Diagnostics: every CTA c < capacity of later iam_bucketmul_full launches of `h` writes 16
 * int64 to trace_dev[16c .. 16c+15]: globaltimer stamps (ns) [0] start, [1] cutoff inputs
 * loaded, [8] bisection mids computed, [9] values binned, [10] suffix counts, [11] binned
 * steps replayed, [2] cutoff done, [3] row selection done, [4] accumulation done, [5] group
 * sums pushed to the cluster, [6] end; and counts [7] bucket rows of the CTA's input group,
 * [12] values of the last bisection bracket, [13] bisection steps.  NULL turns it off.
 * (No counterpart in the reference: phase and load-balance evidence for the kernel.) */
int iam_bucketmul_trace(iam_bucketmul_t h, long long* trace_dev, int capacity);

/* iam_bucketmul_full without any device allocation, for callers that cannot allocate device
 * memory (inside an allocator or memory-pool callback, or a plug-in whose host framework owns
 * every device allocation).  It has no counterpart in the reference, whose BucketMul
 * allocates its scratch in the singleton's constructor.  Same arguments and results as
 * iam_bucketmul_full minus the handle; its scratch is a ~1 MiB __device__ array built into
 * the library, held by every GPU that loads it until exit.
 * Limits: bucket_cols <= 1024 (out_dim <= 16384), else IAM_ERR_ARG.
 * Every call made outside a stream capture looks up that array's device address on the
 * current device (cudaGetSymbolAddress, which allocates nothing) and remembers it; a call made
 * while its stream is being captured uses the remembered address, so make the first call on
 * each device before any capture (a captured first call returns IAM_ERR_ARG).  After a
 * cudaDeviceReset the next call outside capture picks up the re-created array's address.
 * All calls share the one array: calls that overlap on the GPU (different streams, or
 * threads without ordering) race and corrupt each other's results; serialise them. */
int iam_bucketmul_full_noalloc(const float* x_dev, const uint16_t* stats_dev, int stats_stride,
                               const uint16_t* probes_dev, const uint16_t* buckets_dev, int expert_no,
                               int in_dim, int bucket_cols, int expert_size, float effort, float* out_dev,
                               int* count_dev, float* cutoff_dev, void* stream);

/* Packs channel 3 of a [rows][4] stats array into [rows] (stats_stride = 1 layout). */
int iam_stats_pack(const uint16_t* stats4_dev, long long rows, uint16_t* stats1_dev, void* stream);

/* Bucketize W[out_dim][in_dim] (fp16 bits, row-major, device) into the reference layout,
 * on the GPU: same result as preprocess_layer_fixed_gpu.py:110-242 (ties in |w| ordered
 * by lower original slot first).  buckets_dev [16*in_dim][out_dim/16], stats4_dev
 * [16*in_dim][4] (may be NULL), stats1_dev [16*in_dim] (may be NULL), probes_dev [in_dim]. */
int iam_bucketize(const uint16_t* w_dev, int out_dim, int in_dim, uint16_t* buckets_dev,
                  uint16_t* stats4_dev, uint16_t* stats1_dev, uint16_t* probes_dev, void* stream);

/* ------------------------------------------------------------------ dense tensor-core path */
/* Replaces the reference's dense GEMV kernels basicMul / basicMul2 (matrix.cl:80-127:
 * out[row] = sum_i v[i] * m[row][i], fp16 m, fp32 v) batched over tokens, on the tcgen05
 * tensor cores.  A handle owns the activation split (fp16 hi / lo) and split-K scratch for up
 * to max_tokens (<= 65535) x max_in_dim activations and max_out_dim outputs. */
typedef struct iam_dense_s* iam_dense_t;
int iam_dense_create(int max_tokens, int max_in_dim, int max_out_dim, int device, iam_dense_t* out);
int iam_dense_destroy(iam_dense_t h);
/* y[t][o] = residual[t][o] (when residual_dev is not NULL; it may equal y_dev)
 *           + sum_i W[o][i] * x[t][i]            for t < n_tokens, o < out_dim.
 * w_dev fp16 [out_dim][in_dim] (in_dim % 8 == 0, 16-byte aligned); x_dev fp32 [n_tokens][in_dim];
 * y_dev, residual_dev fp32 [n_tokens][out_dim].  precision 0: every activation enters as two
 * fp16 halves (hi + lo, ~22 significant bits, fp32 accumulation); 1: one fp16 (11 bits).
 * split_k 0 picks the K split from the SM count; >= 1 forces it (results are deterministic
 * for every split: the K slices are summed in order).  Asynchronous on `stream`. */
int iam_dense_gemm(iam_dense_t h, const uint16_t* w_dev, int out_dim, int in_dim, const float* x_dev,
                   int n_tokens, const float* residual_dev, float* y_dev, int precision, int split_k,
                   void* stream);
/* Synchronises the device; IAM_ERR_TIMEOUT when a pipeline wait of a GEMM on this handle gave
 * up since the last call (the flag is then cleared). */
int iam_dense_status(iam_dense_t h);
/* Dense fp16 matrix w_out [16*bucket_cols][in_dim] from the bucket layout
 * buckets [16*in_dim][bucket_cols]: each packed word (value with its slot in the low 4 bits,
 * preprocess_layer_fixed_gpu.py:196) returns to row 16*c + slot, column i.  This is the
 * matrix bucketMul multiplies by when every bucket row is selected (bucketMul.cl:430-434). */
int iam_dense_unpack(const uint16_t* buckets_dev, int in_dim, int bucket_cols, uint16_t* w_out_dev,
                     void* stream);

/* ------------------------------------------------------------------ decode model */
/* Replaces MistralModel (model.hpp:84-237), TransformerLayer (transformer_layer.hpp:55-162),
 * Attention (attention.hpp:71-404) and FeedForward (feedforward.hpp:89-183).  The model
 * owns its weights (bucket layout with packed stats), an fp16 GQA KV cache
 * [layer][kv_head][max_ctx][head_dim] (the reference's is fp32 and repeated per query head,
 * model.hpp:97-98), activations and scratch.  Vocabulary, dims, RoPE theta and RMSNorm eps
 * are parameters (the reference hard-codes them, model.hpp:25-30, attention.hpp:21-27). */
typedef struct {
    int dim, n_layers, n_heads, n_kv_heads, head_dim, ffn_dim, vocab, max_ctx;
    float norm_eps;         /* 1e-5 in aux.cl:190 */
    double rope_theta;      /* 1e6 in attention.hpp:27 */
    int tied_embeddings;    /* LM head = embedding matrix (else a separate lm_head) */
} iam_model_config;

typedef struct iam_model_s* iam_model_t;

/* Random-init model on `device`: every weight matrix i.i.d. N(0, 0.02) fp16 (a counter-based
 * generator seeded by `seed`), bucketized on the GPU; RMSNorm gains 1.0; embeddings N(0, 0.02). */
int iam_model_create_random(iam_model_t* out, const iam_model_config* cfg, unsigned long long seed,
                            int device);
/* Loads a model directory in the reference's file layout (MistralModel ctor, model.hpp:84-127):
 * embed_tokens.npy, norm_weight.npy, [lm_head.npy], layer{L}_input_layernorm.npy,
 * layer{L}_post_attention_layernorm.npy and layer{L}_{q,k,v,o,gate,up,down}_proj_bucketmul_fp16_
 * {meta.txt,buckets.bin,stats.bin,probes.bin} (preprocess_layer_fixed_gpu.py:245-333), with the
 * loader's validation (binary_loader.hpp:96-123): IAM_ERR_IO on missing or mis-sized files. */
int iam_model_load(iam_model_t* out, const char* weights_dir, const iam_model_config* cfg, int device);

/* Tensor parallelism over NCCL (one process per GPU, `world` ranks).  The reference runs one
 * GPU (model.hpp:84-231); this shards its decode step Megatron-style: q/k/v and gate/up are
 * column-parallel (rank r holds bucket columns [r*C/world, (r+1)*C/world), i.e. its heads and
 * its FFN slice), o and down are row-parallel (rank r holds the bucket rows of its inputs),
 * stats and probes are replicated so every rank computes the identical cutoff and selection,
 * and the LM head is vocab-sharded.  Per layer: an all-gather of the attention output, an
 * all-reduce of the o output, an all-gather of gate and up, an all-reduce of the down
 * output; per step a max all-reduce of the argmax key (and an all-gather of the logits when a
 * caller asks for them).  n_heads, n_kv_heads, the bucket columns of every matrix and vocab
 * must divide by `world`.
 *
 * iam_tp_unique_id fills the 128-byte NCCL id that rank 0 creates and the caller broadcasts
 * (any side channel: torch.distributed, MPI, a file). */
#define IAM_TP_ID_BYTES 128
int iam_tp_unique_id(unsigned char* id_out);
/* Shard layout of rank `rank` of `world` without a GPU: for each of the 7 matrices
 * (q, k, v, o, gate, up, down) four ints {first bucket column, bucket columns held, first
 * input, end input}, then {first vocab row, vocab rows held}: 30 ints in out. */
int iam_tp_shard_info(const iam_model_config* cfg, int rank, int world, int* out);
/* iam_model_create_random / iam_model_load for one rank of a tensor-parallel group: every rank
 * calls it at the same time (the NCCL communicator is created inside).  Random weights are
 * the same as iam_model_create_random's for the same seed, then sharded. */
int iam_model_create_random_tp(iam_model_t* out, const iam_model_config* cfg, unsigned long long seed,
                               int device, int rank, int world, const unsigned char* nccl_id);
int iam_model_load_tp(iam_model_t* out, const char* weights_dir, const iam_model_config* cfg, int device,
                      int rank, int world, const unsigned char* nccl_id);
int iam_model_destroy(iam_model_t m);
/* Writes the model to weights_dir in the reference's on-disk layout -- exactly what
 * iam_model_load and the reference's loader (binary_loader.hpp:141-193, model.hpp:84-127)
 * read: per matrix {_buckets,_stats,_probes}.bin and _meta.txt as written by
 * preprocess_layer_fixed_gpu.py:245-282 (stats with its 4 identical channels), fp16 .npy
 * files for the norms, the embedding and an untied LM head.  The directory must exist.
 * Single-GPU models only (IAM_ERR_UNSUPPORTED for a tensor-parallel rank). */
int iam_model_save(iam_model_t m, const char* weights_dir);
/* Synchronises the device and reports IAM_ERR_TIMEOUT when a tensor-parallel exchange of an
 * earlier step gave up waiting for a peer (its outputs are then invalid), IAM_ERR_ARG when a
 * decode step found its device position at or past max_ctx (the entry points refuse such
 * calls before launching; the kernels clamp to the last slot and flag it); IAM_OK otherwise.
 * (No counterpart in the reference: failure detection of the multi-GPU path.) */
int iam_model_status(iam_model_t m);
/* Self-test of the bounded device-side wait of the one-shot tensor-parallel exchanges, on ONE
 * GPU and with no peer process (no counterpart in the reference): builds a two-rank exchange
 * window on `device` whose second rank is a plain local buffer that never sends anything,
 * then runs the all-reduce of n floats twice with at most spin_limit polls per element.  The
 * first call's waits run out (the error word is set); the second returns without waiting.
 * *err_out (may be NULL) receives the error word, *first_ms / *second_ms (may be NULL) each
 * call's device time.  Returns IAM_ERR_TIMEOUT when the wait gave up as designed (what
 * iam_model_status reports for a model whose exchange timed out), IAM_OK if it did not. */
int iam_tp_wait_selftest(int device, int n, long long spin_limit, unsigned* err_out, float* first_ms,
                         float* second_ms);
/* MistralModel::reset_caches (model.hpp:233-237): zero the KV cache and the position. */
int iam_model_reset(iam_model_t m, void* stream);
/* MistralModel::forward (model.hpp:152-231): one decode step of `token` at `pos`; logits_dev
 * (vocab floats, may be NULL) receives the logits. */
int iam_model_forward(iam_model_t m, int token, int pos, float effort, float* logits_dev, void* stream);
/* Block-level entry points over one layer of a model (single-GPU models; IAM_ERR_UNSUPPORTED
 * for a tensor-parallel rank).  Vectors are device float arrays; the KV cache is the model's
 * own cache of that layer (iam_model_set_kv / iam_model_read_weight W_K_CACHE, W_V_CACHE), in
 * place of the caller-owned k_cache / v_cache buffers of the reference; the reference's
 * temporaries have no counterpart.  pos in [0, max_ctx), effort in (0, 1], else IAM_ERR_ARG.
 *
 * TransformerLayer::forward (transformer_layer.hpp:75-122): out = x + Attention(RMSNorm(x)),
 * then out += FeedForward(RMSNorm(out)), with the layer's gains; writes the layer's K/V at pos
 * and attends over [0, pos].  x_dev and out_dev hold dim floats (they may be the same array). */
int iam_layer_forward(iam_model_t m, int layer, const float* x_dev, int pos, float effort, float* out_dev,
                      void* stream);
/* Attention::forward (attention.hpp:135-202): h_dev (dim floats, already normalised) through
 * the q/k/v bucketMuls, RoPE, the fp16 K/V append at pos, attention over [0, pos] and the o
 * bucketMul into out_dev (dim floats); no residual. */
int iam_attention_forward(iam_model_t m, int layer, const float* h_dev, int pos, float effort, float* out_dev,
                          void* stream);
/* FeedForward::forward (feedforward.hpp:180): out = down(SiLU(gate(h)) * up(h)) for h_dev
 * (dim floats, already normalised) into out_dev (dim floats); no residual. */
int iam_feedforward_forward(iam_model_t m, int layer, const float* h_dev, float effort, float* out_dev,
                            void* stream);
/* Batched prefill on the dense tensor-core path: the n_tokens prompt tokens (host array) at
 * positions [start_pos, start_pos + n_tokens) go through every layer at once, with every bucket
 * row selected (the dense matmul of matrix.cl, basicMul :80-93, in place of bucketMul), and fill
 * the KV cache.  The reference feeds a prompt through forward() one token at a time
 * (test_generation.cpp:202-213); iam_model_forward does the same, at the chosen effort.
 * logits_dev (vocab floats, may be NULL) receives the last token's logits; *next_token (may be
 * NULL; the call then synchronises the stream) its greedy argmax.  The first call builds dense
 * fp16 copies of the weights (as large as the bucket weights) and prefill scratch.  The device
 * position becomes start_pos + n_tokens, so iam_model_generate with first_token < 0 continues
 * after the prompt from its greedy token.
 * Single-GPU models only (IAM_ERR_UNSUPPORTED for a tensor-parallel rank). */
int iam_model_prefill(iam_model_t m, const int* tokens_host, int n_tokens, int start_pos, float* logits_dev,
                      int* next_token, void* stream);
/* Greedy generation on the device (the decode loop of test_generation.cpp:239-291 without
 * host round trips): step 0 decodes first_token at start_pos, every later step decodes the
 * previous step's argmax; the n_tokens generated ids land in tokens_dev.  Steps after the
 * first replay one captured CUDA graph.  first_token < 0 continues from the device position
 * and the last argmax (start_pos is then ignored), replaying the graph for every step.
 * IAM_ERR_ARG, before anything is launched, when a step would decode at max_ctx or beyond
 * (the library tracks the position every entry point leaves on the device). */
int iam_model_generate(iam_model_t m, int first_token, int start_pos, int n_tokens, float effort,
                       int* tokens_dev, void* stream);
/* Diagnostics: decodes `steps` greedy tokens (continuing from the device position and the
 * last argmax) through one captured graph with a CUDA event between consecutive kernels.
 * kernel_ms[k] (capacity entries) receives the average device time of launch k of a step and
 * kinds[k] its IAM_KERNEL_* kind; *n_kernels the launches per step.  Advances the position. */
enum { IAM_KERNEL_EMBED = 0, IAM_KERNEL_BUCKETMUL = 1, IAM_KERNEL_ATTENTION = 2, IAM_KERNEL_LM_HEAD = 3,
       IAM_KERNEL_OTHER = 4, IAM_KERNEL_COLLECTIVE = 5 };
int iam_model_profile_steps(iam_model_t m, float effort, int steps, float* kernel_ms, int* kinds,
                            int capacity, int* n_kernels, void* stream);
/* KV cache contents of one layer: k/v [n_kv_heads][n_tokens][head_dim] fp16 (post-RoPE k).
 * Under tensor parallelism every rank takes the full arrays and keeps its own kv heads. */
int iam_model_set_kv(iam_model_t m, int layer, const uint16_t* k_dev, const uint16_t* v_dev,
                     int n_tokens, void* stream);
/* Fills positions [0, n_tokens) of every layer's K and V cache with N(0,1) fp16 (the same
 * values per kv head at every tensor-parallel width). */
int iam_model_fill_kv_random(iam_model_t m, int n_tokens, unsigned long long seed, void* stream);

enum {
    IAM_W_EMBED = 0, IAM_W_FINAL_NORM = 1, IAM_W_LM_HEAD = 2, IAM_W_ATTN_NORM = 3, IAM_W_FFN_NORM = 4,
    IAM_W_K_CACHE = 5, IAM_W_V_CACHE = 6, /* one layer: [n_kv_heads][max_ctx][head_dim] fp16 */
    /* IAM_W_MATRIX + 3*m + part: m in q,k,v,o,gate,up,down; part 0 buckets [16*in][cols],
     * 1 packed stats [16*in] (channel 3), 2 probes [in] */
    IAM_W_MATRIX = 16
};
/* Copies one weight tensor to host memory; *bytes_out receives its size (host_dst may be
 * NULL to query it).  Under tensor parallelism: this rank's shard (buckets, LM head rows, KV
 * heads); stats and probes are whole. */
int iam_model_read_weight(iam_model_t m, int layer, int which, void* host_dst, size_t capacity_bytes,
                          size_t* bytes_out);
/* Selected bucket rows summed over the 7*n_layers bucketMuls of the last step (under tensor
 * parallelism a collective call: every rank calls it and all get the whole-model total). */
int iam_model_selected_rows(iam_model_t m, long long* total);
/* Selected bucket rows of each bucketMul of the last step: counts[7*layer + m], m in q, k, v,
 * o, gate, up, down (this rank's rows under tensor parallelism: the whole selection for the
 * column-parallel matrices, its inputs' share for o and down).  capacity >= 7*n_layers. */
int iam_model_selected_rows_by_matrix(iam_model_t m, int* counts, int capacity);
/* Diagnostics (no counterpart in the reference): while a capture buffer is set, every decode
 * step records, for each layer, the input x of its bucketMuls exactly as the kernels computed
 * it (after the fused RMSNorm * gain or SiLU * up), their cutoffs and their outputs, so that
 * every bucketMul of a real step can be checked against a reference implementation on
 * identical inputs.  One record per layer, floats, with d = dim, a = n_heads * head_dim,
 * kv = n_kv_heads * head_dim, f = ffn_dim:
 *   x_qkv[d] q[a] k[kv] v[kv] x_o[a] res_o[d] out_o[d] x_gu[d] gate[f] up[f]
 *   x_down[f] res_down[d] out_down[d] cutoff[8] (q, k, v, o, gate, up, down, unused)
 * where out_o = res_o + o(x_o) and out_down = res_down + down(x_down).  buf_dev holds
 * iam_model_capture_floats floats; NULL turns capturing off.  Single-GPU models only. */
int iam_model_capture_floats(const iam_model_config* cfg, long long* floats);
int iam_model_capture(iam_model_t m, float* buf_dev, size_t capacity_floats);
/* Algorithmic bytes of the last step at KV length `context`: per bucketMul
 * 2|S|C + 2R + 4N + 2*min(N,4096) + 4M, plus K/V reads and the dense LM head (this rank's
 * share under tensor parallelism). */
int iam_model_step_bytes(iam_model_t m, int context, long long* bytes);

#ifdef __cplusplus
}
#endif

#endif /* IAM_B200_H */
