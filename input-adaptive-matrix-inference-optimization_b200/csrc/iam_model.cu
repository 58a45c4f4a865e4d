// iam_model.cu -- Mistral-style decode runtime over the fused bucketMul kernels.
//
// Replaces MistralModel (model.hpp:84-237) + TransformerLayer (transformer_layer.hpp:75-122)
// + Attention (attention.hpp:135-202) + FeedForward (feedforward.hpp:46-86).  One decode
// step is 2 + 5*n_layers launches:
//   embed -> per layer [qkv bucketMuls (RMSNorm*gain fused), attention (RoPE, fp16 KV
//   append, split-K), o bucketMul (+residual), gate/up bucketMuls (RMSNorm*gain fused),
//   down bucketMul (SiLU*up fused, +residual)] -> LM head (final RMSNorm*gain, argmax).
// Position and token live in device memory, so a step can be captured once as a CUDA graph
// and replayed for every generated token without host round trips.
#include <climits>
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <chrono>
#include <cstring>
#include <thread>
#include <fstream>
#include <sstream>
#include <string>
#include <vector>

#include <nccl.h>

#include "iam_bucketmul_group.h"
#include "iam_bucketmul_launch.h"
#include "iam_common.cuh"
#include "iam_dense.h"
#include "iam_layers.h"
#include "iam_prefill.h"
#include "iam_tp.h"

namespace iam {

enum { MQ = 0, MK, MV, MO, MG, MU, MD, NMAT };
static const char* kMatNames[NMAT] = {"q", "k", "v", "o", "gate", "up", "down"};

// Float offsets of one layer's record in a capture buffer (iam_model_capture).
struct CaptureLayout {
    size_t xqkv, q, k, v, xo, reso, outo, xgu, g, u, xd, resd, outd, cut, total;
};
inline CaptureLayout capture_layout(const iam_model_config& c) {
    const size_t d = c.dim, a = (size_t)c.n_heads * c.head_dim, kv = (size_t)c.n_kv_heads * c.head_dim, f = c.ffn_dim;
    CaptureLayout L{};
    size_t o = 0;
    L.xqkv = o; o += d;
    L.q = o;    o += a;
    L.k = o;    o += kv;
    L.v = o;    o += kv;
    L.xo = o;   o += a;
    L.reso = o; o += d;
    L.outo = o; o += d;
    L.xgu = o;  o += d;
    L.g = o;    o += f;
    L.u = o;    o += f;
    L.xd = o;   o += f;
    L.resd = o; o += d;
    L.outd = o; o += d;
    L.cut = o;  o += 8;
    L.total = o;
    return L;
}

struct Matrix {
    uint16_t* buckets = nullptr;  // [16*in][out/16] (column shard for column-parallel TP)
    uint16_t* stats = nullptr;    // [16*in] channel 3 of the stats (all rows, every rank)
    uint16_t* probes = nullptr;   // [in]
    int in_dim = 0, out_dim = 0;  // full matrix shape
    int cols = 0;                 // bucket columns held (out/16, or a shard of them)
    int in_begin = 0, in_end = 0; // inputs held (row-parallel shard) -- full range otherwise
    uint16_t* dense = nullptr;    // [out held][inputs held]: each weight at its output position,
                                  // its bucket row (rank) in the low 4 bits (high-effort decode)
};

struct Layer {
    uint16_t* attn_norm = nullptr;
    uint16_t* ffn_norm = nullptr;
    Matrix m[NMAT];
};

// Dense fp16 copies of a layer's matrices for the batched prefill (iam_dense_unpack layout:
// every bucket row selected), rows stacked per launch: q|k|v, o, gate|up, down.
struct DenseLayer {
    uint16_t *qkv = nullptr, *o = nullptr, *gu = nullptr, *down = nullptr;
};

// ------------------------------------------------------------------ tensor-parallel shards

// q, k, v, gate, up are column-parallel; o and down row-parallel (their inputs are the
// column-parallel outputs of the same rank, so no exchange is needed between the two halves).
inline bool column_parallel(int which) { return which != MO && which != MD; }

// Decode efforts from which the bucketMuls stream dense copies of the matrices (every weight,
// selected by rank: the same selection) instead of the selected bucket rows: above it the
// rows read are most of the matrix, and register accumulation beats the slot scatter.
constexpr float kDenseMinEffort = 0.8f;

// Input ranges of the row-parallel o and down bucketMuls, the same at every tensor-parallel
// degree (up to kTpMaxWorld) so that each rank holds whole ranges and the ranges' partials add
// up in the single-GPU order: 32 when in_dim allows, else fewer; 0 when no power of two of at
// least `world` divides in_dim (the shape is then chosen freely).
inline int row_parallel_ranges(int in_dim, int world) {
    for (int r = 32; r >= 1 && r >= world; r /= 2)
        if (in_dim % r == 0 && r % world == 0 && r % kTpMaxWorld == 0) return r;
    for (int r = 32; r >= 1 && r >= world; r /= 2)
        if (in_dim % r == 0 && r % world == 0) return r;
    return 0;
}

struct Shard {
    int col0, cols;  // bucket columns held
    int in0, in1;    // inputs held
};

inline void matrix_dims(const iam_model_config& c, int which, int* out_dim, int* in_dim) {
    const int qn = c.n_heads * c.head_dim, kvn = c.n_kv_heads * c.head_dim;
    const int outs[NMAT] = {qn, kvn, kvn, c.dim, c.ffn_dim, c.ffn_dim, c.dim};
    const int ins[NMAT] = {c.dim, c.dim, c.dim, qn, c.dim, c.dim, c.ffn_dim};
    *out_dim = outs[which];
    *in_dim = ins[which];
}

inline Shard shard_of(const iam_model_config& c, int which, int rank, int world) {
    int out_dim, in_dim;
    matrix_dims(c, which, &out_dim, &in_dim);
    const int C = out_dim / 16;
    if (world <= 1) return {0, C, 0, in_dim};
    if (column_parallel(which)) return {rank * (C / world), C / world, 0, in_dim};
    return {0, C, rank * (in_dim / world), (rank + 1) * (in_dim / world)};
}

int check_tp(const iam_model_config& c, int rank, int world) {
    if (world < 1 || rank < 0 || rank >= world) return fail(IAM_ERR_ARG, "tensor parallel: bad rank or world");
    if (world == 1) return IAM_OK;
    if (c.n_heads % world || c.n_kv_heads % world || c.vocab % world)
        return fail(IAM_ERR_UNSUPPORTED, "tensor parallel: n_heads, n_kv_heads and vocab must divide by world");
    for (int i = 0; i < NMAT; ++i) {
        int out_dim, in_dim;
        matrix_dims(c, i, &out_dim, &in_dim);
        if (column_parallel(i) ? (out_dim / 16) % world : in_dim % world)
            return fail(IAM_ERR_UNSUPPORTED, std::string("tensor parallel: ") + kMatNames[i] +
                                                 " does not split evenly over world");
    }
    return IAM_OK;
}

// splitmix64 -> two uniforms -> Box-Muller: a reproducible N(0,1) per (seed, tensor, index).
IAM_DEV unsigned long long mix64(unsigned long long z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

// Element i of the tensor is a function of (seed, tensor, i0 + i) only, so any slice of a
// tensor can be generated on its own (i0 even keeps the Box-Muller pairs aligned).
__global__ void init_normal_fp16(uint16_t* w, size_t n, unsigned long long seed, unsigned long long tensor,
                                 float stddev, size_t i0 = 0) {
    for (size_t j = blockIdx.x * (size_t)blockDim.x + threadIdx.x; j < n; j += (size_t)gridDim.x * blockDim.x) {
        const size_t i = i0 + j;
        const unsigned long long h = mix64(seed ^ mix64(tensor * 0x100000001b3ull + (i >> 1)));
        const float u1 = ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
        const float u2 = ((float)((h >> 16) & 0xffffffull) + 0.5f) * (1.0f / 16777216.0f);
        const float r = sqrtf(-2.0f * logf(u1));
        const float z = (i & 1) ? r * sinpif(2.0f * u2) : r * cospif(2.0f * u2);
        w[j] = __half_as_ushort(__float2half_rn(z * stddev));
    }
}

__global__ void fill_u16(uint16_t* w, size_t n, uint16_t v) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) w[i] = v;
}

__global__ void set_int_kernel(int* p, int v) {
    pdl_trigger();
    pdl_wait();
    *p = v;
}

// Copies columns [c0, c0+cols_out) of every row of a [rows][cols_in] u16 array.
__global__ void slice_cols_kernel(const uint16_t* src, int rows, int cols_in, int c0, int cols_out, uint16_t* dst) {
    const size_t n = (size_t)rows * cols_out;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / cols_out, c = i % cols_out;
        dst[i] = src[r * cols_in + c0 + c];
    }
}

}  // namespace iam

using namespace iam;

struct iam_model_s {
    iam_model_config cfg{};
    int device = 0;
    int sm_count = 148;
    int tp_rank = 0, tp_world = 1;
    ncclComm_t comm = nullptr;  // tensor-parallel group (world > 1)
    double tp_timeout_s = 300.0;
    int vocab0 = 0, vocab_local = 0;  // LM head rows held
    uint16_t* embed = nullptr;
    uint16_t* final_norm = nullptr;
    uint16_t* lm_head = nullptr;
    std::vector<Layer> layers;
    uint16_t* k_cache = nullptr;  // [L][kvh_local][max_ctx][hd]
    uint16_t* v_cache = nullptr;
    float* rope = nullptr;
    float *x = nullptr, *x1 = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr;
    float *g = nullptr, *u = nullptr, *logits = nullptr;
    int* pos = nullptr;
    int* pos_err = nullptr;  // set by a decode step whose device position was past the cache
    int host_pos = 0;        // the device position once the work enqueued so far has run
    int* token_used = nullptr;
    int* gen_count = nullptr;
    unsigned long long* key = nullptr;
    int* sel = nullptr;  // [L*7] selected rows of the last step
    // bucketMul scratch, one slot per problem of a batch
    float* partials[3] = {nullptr, nullptr, nullptr};
    int* ctr[3] = {nullptr, nullptr, nullptr};
    int* split_sel[3] = {nullptr, nullptr, nullptr};
    // attention scratch
    float* att_part = nullptr;
    int* att_ctr = nullptr;
    float dense_min_effort = kDenseMinEffort;  // decode efforts from here on stream the dense copies
    int att_split = 32, att_min_chunk = kAttnMinChunk, att_lane_min = kAttnLaneMinCtx,
        att_lane_short = kAttnLaneShortMax;
    // launch plans for the current effort
    std::vector<BMBatch> plans;   // 4 per layer (cluster-split kernel, IAM_BM_KERNEL=split)
    std::vector<BGBatch> gplans;  // 4 per layer (range kernel, the default)
    bool use_group = true;
    float* gpartials[3] = {nullptr, nullptr, nullptr};  // range-kernel partials, one slot per problem
    unsigned* bm_bar = nullptr;                          // range-kernel grid barrier words
    float* capture = nullptr;                            // diagnostics: per-layer bucketMul records
    float plan_effort = -1.0f;
    int vec = 4, G = 4;
    bool pdl = true;  // step kernels launched with programmatic stream serialization (IAM_PDL=0: off)
    // generation graph
    cudaGraphExec_t gen_graph = nullptr;
    float gen_effort = -1.0f;
    int gen_steps = 0;
    int* gen_tokens = nullptr;
    std::vector<void*> allocs;
    int n_heads_local = 0, n_kv_local = 0, ffn_local = 0;
    long long* tp_tmp = nullptr;  // 4 int64 of device scratch for host-side agreements
    // one-shot NVLink collectives (IAM_TP_COLL=nccl: NCCL instead)
    bool tp_p2p = true;
    bool tp_fused = true;       // o / down exchanges inside the bucketMul kernel (IAM_TP_FUSED=0: a launch after it)
    bool tp_push = true;        // heads and gate/up slices pushed by their producers (IAM_TP_PUSH=0: all-gathers)
    char* xwin = nullptr;         // this rank's window (exchanged activations, mailbox, flags)
    TpWindow win{};
    std::vector<void*> peer_maps;
    // batched dense prefill (built by the first iam_model_prefill)
    std::vector<DenseLayer> dense;
    int pf_cap = 0;  // tokens per prefill chunk
    int* pf_tok = nullptr;
    float *pf_h = nullptr, *pf_qkv = nullptr, *pf_att = nullptr, *pf_gu = nullptr, *pf_part = nullptr;
    uint16_t *pf_hi = nullptr, *pf_lo = nullptr;
    uint16_t *pf_hi2 = nullptr, *pf_lo2 = nullptr;  // SiLU(gate) * up as the down product's input
    bool pf_silu_fused = false;  // gate|up rows interleaved in 128-row blocks, SiLU in its epilogue
    unsigned* pf_err = nullptr;
};

namespace {

template <class T>
int dalloc(iam_model_s* m, T** p, size_t count) {
    void* ptr = nullptr;
    cudaError_t e = cudaMalloc(&ptr, count * sizeof(T) + 16);
    if (e != cudaSuccess) return cuda_fail(e, "model cudaMalloc");
    m->allocs.push_back(ptr);
    *p = reinterpret_cast<T*>(ptr);
    return IAM_OK;
}

int check_cfg(const iam_model_config* c) {
    if (!c) return fail(IAM_ERR_ARG, "model: null config");
    if (c->dim <= 0 || c->n_layers <= 0 || c->n_heads <= 0 || c->n_kv_heads <= 0 || c->head_dim <= 0 ||
        c->ffn_dim <= 0 || c->vocab <= 0 || c->max_ctx <= 0)
        return fail(IAM_ERR_ARG, "model: every dimension must be positive");
    if (c->n_heads % c->n_kv_heads) return fail(IAM_ERR_ARG, "model: n_heads must be a multiple of n_kv_heads");
    const int gq = c->n_heads / c->n_kv_heads;
    if (gq != 1 && gq != 2 && gq != 4 && gq != 8) return fail(IAM_ERR_UNSUPPORTED, "model: GQA group must be 1/2/4/8");
    if (c->head_dim != 64 && c->head_dim != 128 && c->head_dim != 256)
        return fail(IAM_ERR_UNSUPPORTED, "model: head_dim must be 64, 128 or 256");
    if (c->n_heads * c->head_dim % 16 || c->n_kv_heads * c->head_dim % 16 || c->dim % 16 || c->ffn_dim % 16)
        return fail(IAM_ERR_ARG, "model: every projection width must be a multiple of 16");
    if (c->dim % 8 || c->ffn_dim % 8) return fail(IAM_ERR_ARG, "model: dim and ffn_dim must be multiples of 8");
    return IAM_OK;
}

// RoPE table exactly as precompute_rope_cache (attention.hpp:210-226): freq in double then
// float, angle = float(pos) * freq, cosf / sinf.
std::vector<float> rope_table(const iam_model_config& c) {
    const int half = c.head_dim / 2;
    std::vector<float> t((size_t)c.max_ctx * c.head_dim);
    std::vector<float> freq(half);
    for (int i = 0; i < half; ++i) {
        const double exponent = (2.0 * i) / c.head_dim;
        freq[i] = (float)(1.0 / std::pow(c.rope_theta, exponent));
    }
    for (int p = 0; p < c.max_ctx; ++p)
        for (int i = 0; i < half; ++i) {
            const float angle = (float)p * freq[i];
            t[(size_t)p * c.head_dim + 2 * i] = std::cos(angle);
            t[(size_t)p * c.head_dim + 2 * i + 1] = std::sin(angle);
        }
    return t;
}

// Tensor-parallel inputs of o and down pushed by their producing kernels (NVLink exchanges,
// the range kernel with its exchange inside, IAM_TP_PUSH unset or not 0).
bool push_mode(const iam_model_s* m) {
    return m->tp_world > 1 && m->tp_p2p && m->use_group && m->tp_fused && m->tp_push;
}

int alloc_runtime(iam_model_s* m) {
    const iam_model_config& c = m->cfg;
    const int hd = c.head_dim;
    int rc;
    const size_t kv = (size_t)c.n_layers * m->n_kv_local * c.max_ctx * hd;
    if ((rc = dalloc(m, &m->k_cache, kv)) || (rc = dalloc(m, &m->v_cache, kv))) return rc;
    IAM_CUDA_TRY(cudaMemset(m->k_cache, 0, kv * 2));
    IAM_CUDA_TRY(cudaMemset(m->v_cache, 0, kv * 2));
    if ((rc = dalloc(m, &m->rope, (size_t)c.max_ctx * hd))) return rc;
    std::vector<float> rt = rope_table(c);
    IAM_CUDA_TRY(cudaMemcpy(m->rope, rt.data(), rt.size() * sizeof(float), cudaMemcpyHostToDevice));
    const int qn = c.n_heads * hd, kvn = c.n_kv_heads * hd;
    if (m->tp_world > 1 && m->tp_p2p) {
        // the exchanged activations live in one window that the peers map (iam_tp.h)
        size_t off = 0;
        auto take = [&](size_t bytes) {
            const size_t o = off;
            off += (bytes + 255) / 256 * 256;
            return o;
        };
        const size_t o_att = take((size_t)qn * 4), o_g = take((size_t)c.ffn_dim * 4), o_u = take((size_t)c.ffn_dim * 4);
        const size_t o_x1 = take((size_t)c.dim * 4), o_x = take((size_t)c.dim * 4), o_lg = take((size_t)c.vocab * 4);
        TpWindow& w = m->win;
        w.rank = m->tp_rank;
        w.world = m->tp_world;
        w.spin_limit = kTpSpinLimit;
        if (const char* v = getenv("IAM_TP_SPIN_LIMIT")) w.spin_limit = std::max(1LL, atoll(v));
        // the largest exchange: the o/down all-reduce (dim), the head all-gather, the gate+up
        // all-gather (2 x ffn_local) or the logits all-gather (vocab_local)
        w.mbox_floats = std::max(std::max(c.dim, qn / m->tp_world), std::max(2 * m->ffn_local, m->vocab_local));
        // the o / down range partials (tp_gather_reduce): ranges per rank x dim
        for (const int in : {qn, c.ffn_dim}) {
            const int r = row_parallel_ranges(in, m->tp_world);
            w.mbox_floats = std::max(w.mbox_floats, std::max(1, r / m->tp_world) * c.dim);
        }
        w.epoch_off = take(4 * kTpCtas);
        w.err_off = take(4);
        w.mbox_off = take((size_t)2 * m->tp_world * w.mbox_floats * 8);
        // the o / down range partials exchanged inside the bucketMul kernel: ranges per rank x dim
        // (the bucket path's fixed ranges or the dense stream's, whichever is more)
        w.fused_floats = 1;
        for (const int in : {qn, c.ffn_dim}) {
            const int r = std::max(row_parallel_ranges(in, m->tp_world), bg_dense_ranges(in, true));
            w.fused_floats = std::max(w.fused_floats, std::max(1, r / m->tp_world) * c.dim);
        }
        w.fused_off = take((size_t)2 * m->tp_world * w.fused_floats * 8);
        w.fused_epoch_off = take(4);
        w.xin_off = take(4 * kTpPushKinds);
        // pushed inputs (iam_tp_push.cuh): every head, and gate / up (the cutoff prefix of down)
        w.pmb_ffn = c.ffn_dim;
        w.pmb_off[kTpPushHeads] = take((size_t)qn * 8);
        w.pmb_off[kTpPushFfn] = take((size_t)2 * w.pmb_ffn * 8);
        if ((rc = dalloc(m, &m->xwin, off))) return rc;
        IAM_CUDA_TRY(cudaMemset(m->xwin, 0, off));
        w.base[m->tp_rank] = m->xwin;
        m->att = reinterpret_cast<float*>(m->xwin + o_att);
        m->g = reinterpret_cast<float*>(m->xwin + o_g);
        m->u = reinterpret_cast<float*>(m->xwin + o_u);
        m->x1 = reinterpret_cast<float*>(m->xwin + o_x1);
        m->x = reinterpret_cast<float*>(m->xwin + o_x);
        m->logits = reinterpret_cast<float*>(m->xwin + o_lg);
    } else if ((rc = dalloc(m, &m->x, c.dim)) || (rc = dalloc(m, &m->x1, c.dim)) || (rc = dalloc(m, &m->att, qn)) ||
               (rc = dalloc(m, &m->g, c.ffn_dim)) || (rc = dalloc(m, &m->u, c.ffn_dim)) ||
               (rc = dalloc(m, &m->logits, c.vocab))) {
        return rc;
    }
    if ((rc = dalloc(m, &m->q, qn)) || (rc = dalloc(m, &m->k, kvn)) || (rc = dalloc(m, &m->v, kvn)) ||
        (rc = dalloc(m, &m->pos, 4)) || (rc = dalloc(m, &m->pos_err, 1)) || (rc = dalloc(m, &m->token_used, 4)) || (rc = dalloc(m, &m->gen_count, 4)) ||
        (rc = dalloc(m, &m->key, 2)) || (rc = dalloc(m, &m->sel, (size_t)c.n_layers * NMAT)))
        return rc;
    IAM_CUDA_TRY(cudaMemset(m->pos, 0, 16));
    IAM_CUDA_TRY(cudaMemset(m->pos_err, 0, sizeof(int)));
    IAM_CUDA_TRY(cudaMemset(m->key, 0, 16));
    const int cols_max = std::max(std::max(qn, c.dim), c.ffn_dim) / 16;
    for (int s = 0; s < 3; ++s) {
        if ((rc = dalloc(m, &m->partials[s], (size_t)kMaxSplits * 16 * cols_max)) ||
            (rc = dalloc(m, &m->ctr[s], 4096)) || (rc = dalloc(m, &m->split_sel[s], kMaxSplits)) ||
            (rc = dalloc(m, &m->gpartials[s], bg_scratch_floats(kMaxRanges, cols_max))))
            return rc;
        IAM_CUDA_TRY(cudaMemset(m->ctr[s], 0, 4096 * sizeof(int)));
    }
    if ((rc = dalloc(m, &m->bm_bar, 4))) return rc;
    IAM_CUDA_TRY(cudaMemset(m->bm_bar, 0, 4 * sizeof(unsigned)));
    const int gq = c.n_heads / c.n_kv_heads;
    // chunks per KV head: about 2 CTAs per SM at long context with every KV head on one GPU
    // (short contexts use fewer: a chunk holds at least att_min_chunk tokens; 4 per SM and 4
    // tokens per half-warp in flight measured slower at 8192 tokens).  The count follows from
    // the model's KV heads, not this rank's, so a context is cut into the same chunks, and
    // summed in the same order, at every tensor-parallel degree.
    m->att_split = std::max(1, std::min(64, 2 * m->sm_count / std::max(1, c.n_kv_heads)));
    if (const char* v = getenv("IAM_ATTN_MIN_CHUNK")) m->att_min_chunk = std::max(1, atoi(v));
    if (const char* v = getenv("IAM_ATTN_LANE_MIN_CTX")) m->att_lane_min = std::max(1, atoi(v));
    if (const char* v = getenv("IAM_ATTN_LANE_SHORT_MAX")) m->att_lane_short = std::max(0, atoi(v));
    if (const char* v = getenv("IAM_DENSE_MIN_EFFORT")) m->dense_min_effort = (float)atof(v);
    if (gq > 4 || (hd != 64 && hd != 128)) {  // outside the tensor-core layout's shapes
        m->att_lane_min = INT_MAX;
        m->att_lane_short = 0;
    }
    {
        AttnParams probe{};
        probe.head_dim = hd;
        probe.n_split = m->att_split;
        if (attention_smem(probe, gq) > 227 * 1024) return fail(IAM_ERR_UNSUPPORTED, "model: head_dim too large for attention");
    }
    if ((rc = dalloc(m, &m->att_part, (size_t)m->n_kv_local * m->att_split * gq * (hd + 2))) ||
        (rc = dalloc(m, &m->att_ctr, m->n_kv_local)))
        return rc;
    IAM_CUDA_TRY(cudaMemset(m->att_ctr, 0, m->n_kv_local * sizeof(int)));
    return IAM_OK;
}

void free_model(iam_model_s* m) {
    if (m->gen_graph) cudaGraphExecDestroy(m->gen_graph);  // holds NCCL work: released first
    if (!m->peer_maps.empty()) {
        cudaDeviceSynchronize();
        for (void* p : m->peer_maps) cudaIpcCloseMemHandle(p);
        m->peer_maps.clear();
    }
    if (m->comm) {
        cudaDeviceSynchronize();
        ncclResult_t st = ncclSuccess;
        ncclCommGetAsyncError(m->comm, &st);
        if (st == ncclSuccess) ncclCommDestroy(m->comm);
        else ncclCommAbort(m->comm);
    }
    for (void* p : m->allocs) cudaFree(p);
    delete m;
}

// Waits (bounded) for a call on the non-blocking communicator to finish.
int nccl_done(iam_model_s* m, ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return IAM_OK;
    if (r != ncclInProgress) return fail(IAM_ERR_NCCL, std::string(what) + ": " + ncclGetErrorString(r));
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        ncclCommGetAsyncError(m->comm, &st);
        if (st == ncclSuccess) return IAM_OK;
        if (st != ncclInProgress) return fail(IAM_ERR_NCCL, std::string(what) + ": " + ncclGetErrorString(st));
        const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (el > m->tp_timeout_s) {
            ncclCommAbort(m->comm);
            m->comm = nullptr;
            return fail(IAM_ERR_TIMEOUT, std::string(what) + ": peers did not answer in time");
        }
        // an enqueue finishes in microseconds: spin first, sleep only on long waits (peers joining)
        if (el < 0.02) std::this_thread::yield();
        else std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
}

size_t woff(const iam_model_s* m, const float* p) {
    return (size_t)(reinterpret_cast<const char*>(p) - m->xwin);
}

int nccl_allgather(iam_model_s* m, float* buf, size_t per_rank, cudaStream_t s) {
    return nccl_done(m, ncclAllGather(buf + (size_t)m->tp_rank * per_rank, buf, per_rank, ncclFloat, m->comm, s),
                     "ncclAllGather");
}

int nccl_allreduce_sum(iam_model_s* m, float* buf, size_t n, cudaStream_t s) {
    return nccl_done(m, ncclAllReduce(buf, buf, n, ncclFloat, ncclSum, m->comm, s), "ncclAllReduce");
}

// Maps every peer's window (CUDA IPC handles exchanged over the NCCL communicator).  Called
// by every rank once all have built their shards.
int tp_map_peers(iam_model_s* m) {
    if (m->tp_world == 1 || !m->tp_p2p) return IAM_OK;
    if (m->tp_world > kTpMaxWorld) return fail(IAM_ERR_UNSUPPORTED, "tensor parallel: at most 8 ranks");
    cudaIpcMemHandle_t mine;
    IAM_CUDA_TRY(cudaIpcGetMemHandle(&mine, m->xwin));
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    unsigned char* dev = nullptr;
    IAM_CUDA_TRY(cudaMalloc(&dev, hb * m->tp_world));
    std::vector<unsigned char> all(hb * m->tp_world);
    cudaError_t e = cudaMemcpy(dev + hb * m->tp_rank, &mine, hb, cudaMemcpyHostToDevice);
    int rc = e == cudaSuccess ? IAM_OK : cuda_fail(e, "tp handle upload");
    if (!rc) rc = nccl_done(m, ncclAllGather(dev + hb * m->tp_rank, dev, hb, ncclUint8, m->comm, 0), "handle all-gather");
    if (!rc && (e = cudaMemcpy(all.data(), dev, all.size(), cudaMemcpyDeviceToHost)) != cudaSuccess)
        rc = cuda_fail(e, "tp handle download");
    cudaFree(dev);
    for (int p = 0; p < m->tp_world && !rc; ++p) {
        if (p == m->tp_rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, all.data() + hb * p, hb);
        void* ptr = nullptr;
        if ((e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess)) != cudaSuccess)
            rc = cuda_fail(e, "cudaIpcOpenMemHandle (peer window)");
        else {
            m->peer_maps.push_back(ptr);
            m->win.base[p] = static_cast<char*>(ptr);
        }
    }
    return rc;
}

// Every rank of the group learns whether all ranks got here with rc == IAM_OK (a rank that
// failed to build still takes part, so no rank waits on it in a later collective).
// The settings every rank of a group must share: which exchanges run and where (a rank that
// launched a different sequence of exchanges, or a different range layout, would wait for
// peers that never send).
long long tp_settings(const iam_model_s* m) {
    uint32_t dense_bits;
    std::memcpy(&dense_bits, &m->dense_min_effort, sizeof(dense_bits));
    return ((long long)dense_bits << 8) | (m->tp_p2p ? 1 : 0) | (m->tp_fused ? 2 : 0) | (m->tp_push ? 4 : 0) |
           (m->use_group ? 8 : 0);
}

int tp_agree(iam_model_s* m, int rc) {
    if (m->tp_world == 1) return rc;
    const long long mine = tp_settings(m);
    long long h[4] = {rc != IAM_OK ? 1 : 0, mine, -mine, 0};  // max of each: any failure, settings range
    IAM_CUDA_TRY(cudaMemcpy(m->tp_tmp, h, sizeof(h), cudaMemcpyHostToDevice));
    int r2 = nccl_done(m, ncclAllReduce(m->tp_tmp, m->tp_tmp, 3, ncclInt64, ncclMax, m->comm, 0), "status all-reduce");
    if (r2) return r2;
    IAM_CUDA_TRY(cudaMemcpy(h, m->tp_tmp, sizeof(h), cudaMemcpyDeviceToHost));
    if (rc) return rc;
    if (h[0]) return fail(IAM_ERR_UNSUPPORTED, "tensor parallel: another rank failed to build its shard");
    if (h[1] != mine || -h[2] != mine)
        return fail(IAM_ERR_ARG, "tensor parallel: the ranks were started with different exchange settings "
                                 "(IAM_TP_COLL, IAM_TP_FUSED, IAM_TP_PUSH, IAM_BM_KERNEL, IAM_DENSE_MIN_EFFORT)");
    return IAM_OK;
}

// Full matrix from (seed, tensor), bucketized whole (so stats, probes and the bucket layout
// are those of the unsharded model), then this rank's shard kept.
int make_matrix_random(iam_model_s* m, Matrix& mat, int which, unsigned long long seed, unsigned long long tensor,
                       uint16_t* wtmp, uint16_t* btmp) {
    int out_dim, in_dim;
    matrix_dims(m->cfg, which, &out_dim, &in_dim);
    const Shard sh = shard_of(m->cfg, which, m->tp_rank, m->tp_world);
    mat.in_dim = in_dim;
    mat.out_dim = out_dim;
    mat.cols = sh.cols;
    mat.in_begin = sh.in0;
    mat.in_end = sh.in1;
    int rc;
    if ((rc = dalloc(m, &mat.buckets, (size_t)16 * (sh.in1 - sh.in0) * sh.cols)) ||
        (rc = dalloc(m, &mat.stats, (size_t)16 * in_dim)) || (rc = dalloc(m, &mat.probes, (size_t)in_dim)))
        return rc;
    const size_t n = (size_t)out_dim * in_dim;
    init_normal_fp16<<<4 * m->sm_count, 256>>>(wtmp, n, seed, tensor, 0.02f);
    IAM_CUDA_TRY(cudaGetLastError());
    if (m->tp_world == 1) return bucketize_launch(wtmp, out_dim, in_dim, mat.buckets, nullptr, mat.stats, mat.probes, 0);
    if ((rc = bucketize_launch(wtmp, out_dim, in_dim, btmp, nullptr, mat.stats, mat.probes, 0))) return rc;
    const int C = out_dim / 16;
    if (column_parallel(which)) {
        slice_cols_kernel<<<4 * m->sm_count, 256>>>(btmp, 16 * in_dim, C, sh.col0, sh.cols, mat.buckets);
        IAM_CUDA_TRY(cudaGetLastError());
    } else {
        IAM_CUDA_TRY(cudaMemcpy(mat.buckets, btmp + (size_t)16 * sh.in0 * C, (size_t)16 * (sh.in1 - sh.in0) * C * 2,
                                cudaMemcpyDeviceToDevice));
    }
    return IAM_OK;
}

// ------------------------------------------------------------------ reference file format

struct Meta {
    long b0 = 0, b1 = 0, b2 = 0, s0 = 0, s1 = 0, s2 = 0, p0 = 0, p1 = 0, in_dim = 0, out_dim = 0, bsize = 0;
};

// binary_loader.hpp:59-102
int read_meta(const std::string& file, Meta& mt) {
    std::ifstream f(file);
    if (!f) return fail(IAM_ERR_IO, "Cannot open metadata file: " + file);
    std::string line;
    while (std::getline(f, line)) {
        if (line.empty() || line[0] == '#') continue;
        std::istringstream is(line);
        std::string key;
        is >> key;
        if (key == "buckets_shape:") is >> mt.b0 >> mt.b1 >> mt.b2;
        else if (key == "stats_shape:") is >> mt.s0 >> mt.s1 >> mt.s2;
        else if (key == "probes_shape:") is >> mt.p0 >> mt.p1;
        else if (key == "in_dim:") is >> mt.in_dim;
        else if (key == "out_dim:") is >> mt.out_dim;
        else if (key == "bsize:") is >> mt.bsize;
    }
    if (mt.in_dim == 0 || mt.out_dim == 0) return fail(IAM_ERR_IO, "Invalid metadata - missing dimensions: " + file);
    return IAM_OK;
}

// binary_loader.hpp:105-134: the file size must equal the metadata size.
int read_u16(const std::string& file, size_t n, std::vector<uint16_t>& out) {
    std::ifstream f(file, std::ios::binary | std::ios::ate);
    if (!f) return fail(IAM_ERR_IO, "Cannot open binary file: " + file);
    const size_t size = (size_t)f.tellg();
    if (size != n * 2) {
        std::ostringstream os;
        os << "File size mismatch: " << file << " has " << size << " bytes, expected " << n * 2;
        return fail(IAM_ERR_IO, os.str());
    }
    f.seekg(0);
    out.resize(n);
    if (!f.read(reinterpret_cast<char*>(out.data()), (std::streamsize)size)) return fail(IAM_ERR_IO, "Failed to read " + file);
    return IAM_OK;
}

// model.hpp:54-81: fp16 payload after the .npy header.
int read_npy_u16(const std::string& file, size_t n, std::vector<uint16_t>& out) {
    std::ifstream f(file, std::ios::binary | std::ios::ate);
    if (!f) return fail(IAM_ERR_IO, "Cannot open: " + file);
    const size_t size = (size_t)f.tellg();
    f.seekg(0);
    char hdr[10];
    if (size < 10 || !f.read(hdr, 10) || std::memcmp(hdr, "\x93NUMPY", 6) != 0) return fail(IAM_ERR_IO, "not a .npy file: " + file);
    const size_t hlen = (unsigned char)hdr[8] | ((size_t)(unsigned char)hdr[9] << 8);
    if (size < 10 + hlen || size - 10 - hlen != n * 2) {
        std::ostringstream os;
        os << "npy payload mismatch: " << file << " expected " << n << " fp16 values";
        return fail(IAM_ERR_IO, os.str());
    }
    f.seekg((std::streamoff)(10 + hlen));
    out.resize(n);
    if (!f.read(reinterpret_cast<char*>(out.data()), (std::streamsize)(n * 2))) return fail(IAM_ERR_IO, "Failed to read " + file);
    return IAM_OK;
}

int upload(iam_model_s* m, uint16_t** dst, const std::vector<uint16_t>& src) {
    int rc = dalloc(m, dst, src.size());
    if (rc) return rc;
    IAM_CUDA_TRY(cudaMemcpy(*dst, src.data(), src.size() * 2, cudaMemcpyHostToDevice));
    return IAM_OK;
}

int load_matrix(iam_model_s* m, const std::string& dir, int layer, int which, int out_dim, int in_dim, Matrix& mat) {
    const std::string prefix = dir + "/layer" + std::to_string(layer) + "_" + kMatNames[which] + "_proj_bucketmul_fp16";
    Meta mt;
    int rc = read_meta(prefix + "_meta.txt", mt);
    if (rc) return rc;
    if (mt.in_dim != in_dim || mt.out_dim != out_dim || mt.b1 != 16L * in_dim || mt.b2 != out_dim / 16 ||
        mt.s1 != 16L * in_dim || mt.p1 != in_dim)
        return fail(IAM_ERR_IO, "weight shape differs from the model config: " + prefix);
    std::vector<uint16_t> b, s, p;
    if ((rc = read_u16(prefix + "_buckets.bin", (size_t)(mt.b0 * mt.b1 * mt.b2), b)) ||
        (rc = read_u16(prefix + "_stats.bin", (size_t)(mt.s0 * mt.s1 * mt.s2), s)) ||
        (rc = read_u16(prefix + "_probes.bin", (size_t)(mt.p0 * mt.p1), p)))
        return rc;
    std::vector<uint16_t> s1((size_t)mt.s1);
    for (size_t r = 0; r < s1.size(); ++r) s1[r] = s[r * (size_t)mt.s2 + (size_t)(mt.s2 - 1)];  // channel 3
    const Shard sh = shard_of(m->cfg, which, m->tp_rank, m->tp_world);
    mat.in_dim = in_dim;
    mat.out_dim = out_dim;
    mat.cols = sh.cols;
    mat.in_begin = sh.in0;
    mat.in_end = sh.in1;
    if (m->tp_world > 1) {  // keep this rank's shard of the bucket rows / columns
        const size_t C = (size_t)out_dim / 16;
        std::vector<uint16_t> part((size_t)16 * (sh.in1 - sh.in0) * sh.cols);
        for (size_t r = 0; r < (size_t)16 * (sh.in1 - sh.in0); ++r)
            std::memcpy(&part[r * sh.cols], &b[((size_t)16 * sh.in0 + r) * C + sh.col0], (size_t)sh.cols * 2);
        b.swap(part);
    }
    if ((rc = upload(m, &mat.buckets, b)) || (rc = upload(m, &mat.stats, s1))) return rc;
    p.resize((size_t)in_dim);
    return upload(m, &mat.probes, p);
}

// ------------------------------------------------------------------ step

void fill_problem(iam_model_s* m, BMProblem& p, const Matrix& mat, float effort, float* out, int slot) {
    memset(&p, 0, sizeof(p));
    p.buckets = mat.buckets;
    p.stats = mat.stats;
    p.stats_stride = 1;
    p.probes = mat.probes;
    p.row0 = 0;
    p.bucket_row0 = 16LL * mat.in_begin;
    p.in_begin = mat.in_begin;
    p.n_rows_valid = 16 * mat.in_end;
    p.n_inputs = mat.in_end;
    p.cols = mat.cols;
    p.P = std::min(mat.in_dim, IAM_PROBES_COUNT);
    p.target = bm_target(effort, p.P);
    p.out = out;
    p.partials = m->partials[slot];
    p.slice_ctr = m->ctr[slot];
    p.split_sel = m->split_sel[slot];
}

// Plans a batch for clusters of m->G CTAs; when that leaves more than a fifth of the SMs idle
// (column tiles x splits quantise badly, e.g. gate+up: 14 tiles) and clusters of 2 fill more,
// the batch is planned for clusters of 2 instead (IAM_BM_CLUSTER pins the size).
void plan_batch(iam_model_s* m, BMBatch& b) {
    const BMBatch spec = b;
    bm_plan(b, m->vec, m->G, bm_max_active_clusters(m->vec, m->G));
    b.cluster = m->G;
    if (getenv("IAM_BM_CLUSTER") || m->G == 2) return;
    const int ctas = bm_total_clusters(b) * m->G;
    if (ctas >= 0.8 * m->sm_count) return;
    BMBatch alt = spec;
    bm_plan(alt, m->vec, 2, bm_max_active_clusters(m->vec, 2));
    if (bm_total_clusters(alt) * 2 > ctas) {
        b = alt;
        b.cluster = 2;
    }
}

int build_plans(iam_model_s* m, float effort) {
    if (m->plan_effort == effort && !m->plans.empty()) return IAM_OK;
    const iam_model_config& c = m->cfg;
    m->plans.assign((size_t)c.n_layers * 4, BMBatch{});
    for (int l = 0; l < c.n_layers; ++l) {
        const Layer& L = m->layers[l];
        int* sel = m->sel + l * NMAT;
        BMBatch& qkv = m->plans[l * 4 + 0];
        memset(&qkv, 0, sizeof(qkv));
        qkv.nprob = 3;
        qkv.mode = kModeFused;
        qkv.xmode = kXRms;
        float* outs[3] = {m->q, m->k, m->v};  // this rank's heads
        for (int i = 0; i < 3; ++i) {
            fill_problem(m, qkv.p[i], L.m[MQ + i], effort, outs[i], i);
            qkv.p[i].x = m->x;
            qkv.p[i].gain = L.attn_norm;
            qkv.p[i].norm_eps = c.norm_eps;
            qkv.p[i].norm_n = c.dim;
            qkv.p[i].count_out = sel + MQ + i;
        }
        plan_batch(m, qkv);

        BMBatch& o = m->plans[l * 4 + 1];
        memset(&o, 0, sizeof(o));
        o.nprob = 1;
        o.mode = kModeFused;
        o.xmode = kXPlain;
        fill_problem(m, o.p[0], L.m[MO], effort, m->x1, 0);
        o.p[0].x = m->att;  // every head (gathered under tensor parallelism)
        o.p[0].residual = m->tp_rank == 0 ? m->x : nullptr;  // added once; the all-reduce sums the ranks
        o.p[0].count_out = sel + MO;
        plan_batch(m, o);

        BMBatch& gu = m->plans[l * 4 + 2];
        memset(&gu, 0, sizeof(gu));
        gu.nprob = 2;
        gu.mode = kModeFused;
        gu.xmode = kXRms;
        const size_t f0 = (size_t)m->tp_rank * m->ffn_local;  // this rank's FFN slice
        float* gouts[2] = {m->g + f0, m->u + f0};
        for (int i = 0; i < 2; ++i) {
            fill_problem(m, gu.p[i], L.m[MG + i], effort, gouts[i], i);
            gu.p[i].x = m->x1;
            gu.p[i].gain = L.ffn_norm;
            gu.p[i].norm_eps = c.norm_eps;
            gu.p[i].norm_n = c.dim;
            gu.p[i].count_out = sel + MG + i;
        }
        plan_batch(m, gu);

        BMBatch& d = m->plans[l * 4 + 3];
        memset(&d, 0, sizeof(d));
        d.nprob = 1;
        d.mode = kModeFused;
        d.xmode = kXSilu;
        fill_problem(m, d.p[0], L.m[MD], effort, m->x, 0);
        d.p[0].x = m->g;
        d.p[0].x2 = m->u;
        d.p[0].residual = m->tp_rank == 0 ? m->x1 : nullptr;
        d.p[0].count_out = sel + MD;
        plan_batch(m, d);
    }
    // the same launches for the range kernel (the default): one wave of CTAs over column
    // tiles x input ranges of the inputs this rank holds
    m->gplans.assign(m->plans.size(), BGBatch{});
    static const int kMats[4][3] = {{MQ, MK, MV}, {MO, -1, -1}, {MG, MU, -1}, {MD, -1, -1}};
    for (int l = 0; l < c.n_layers; ++l)
        for (int bi = 0; bi < 4; ++bi) {
            const BMBatch& a = m->plans[l * 4 + bi];
            BGBatch& b = m->gplans[l * 4 + bi];
            memset(&b, 0, sizeof(b));
            b.nprob = a.nprob;
            b.xmode = a.xmode;
            b.barrier = m->bm_bar;
            for (int i = 0; i < a.nprob; ++i) {
                const Matrix& mat = m->layers[l].m[kMats[bi][i]];
                const BMProblem& sp = a.p[i];
                BGProblem& p = b.p[i];
                p.buckets = sp.buckets;
                p.stats = sp.stats;
                p.stats_stride = sp.stats_stride;
                p.probes = sp.probes;
                p.x = sp.x;
                p.x2 = sp.x2;
                p.gain = sp.gain;
                p.norm_eps = sp.norm_eps;
                p.norm_n = sp.norm_n;
                p.out = sp.out;
                p.residual = sp.residual;
                p.count_out = sp.count_out;
                p.partials = m->gpartials[i];
                p.row0 = 0;
                p.bucket_row0 = 16LL * mat.in_begin;
                p.n_rows_valid = 16 * mat.in_dim;
                p.in_begin = mat.in_begin;
                p.n_in = mat.in_end - mat.in_begin;
                p.cols = mat.cols;
                // the whole matrix (the sum order follows from it: identical at every TP degree)
                p.full_in = mat.in_dim;
                p.full_cols = mat.out_dim / 16;
                if (!column_parallel(kMats[bi][i])) p.fixed_ranges = row_parallel_ranges(mat.in_dim, m->tp_world);
                p.dense = mat.dense;
                p.P = sp.P;
                p.target = sp.target;
                if (m->capture) {  // diagnostics: the x each launch used and every cutoff
                    const CaptureLayout CL = capture_layout(c);
                    float* rec = m->capture + (size_t)l * CL.total;
                    const size_t xoff[4] = {CL.xqkv, CL.xo, CL.xgu, CL.xd};
                    if (i == 0) p.x_capture = rec + xoff[bi];
                    p.cutoff_out = rec + CL.cut + kMats[bi][i];
                }
            }
            // under the NVLink exchanges the o and down ranges of every rank are summed inside the
            // kernel (tp_fused; IAM_TP_FUSED=0: by a tp_gather_reduce launch after it)
            const bool rowp = m->tp_world > 1 && m->tp_p2p && m->use_group && (bi == 1 || bi == 3);
            b.tp_fused = (rowp && m->tp_fused) ? 1 : 0;
            b.partials_only = (rowp && !m->tp_fused) ? 1 : 0;
            if (b.tp_fused) {
                b.tp = m->win;
                b.p[0].residual = bi == 1 ? m->x : m->x1;  // every rank adds it: every rank sums all ranges
            }
            b.dense = effort >= m->dense_min_effort ? 1 : 0;
            for (int i = 0; i < b.nprob; ++i) {
                const BGProblem& p = b.p[i];
                if (!p.dense || bg_dense_ranges(p.full_in, p.fixed_ranges > 0) == 0) b.dense = 0;
            }
            bg_choose_shape(b);
            // the heads and the gate/up values of every rank that o and down read for their
            // cutoff (the first P inputs), pushed by the attention and gate/up launches into every
            // peer's mailbox; o and down read the ones other ranks made from their own mailbox
            if (push_mode(m) && bi >= 1) {
                b.tp = m->win;
                if (bi == 1) b.tp_wait = 1 + kTpPushHeads;
                if (bi == 3) b.tp_wait = 1 + kTpPushFfn;
                if (bi == 2) {
                    b.tp_push = 1 + kTpPushFfn;
                    b.push_limit = m->plans[(size_t)l * 4 + 3].p[0].P;  // down's cutoff prefix
                    for (int i = 0; i < b.nprob; ++i) b.p[i].out_begin = m->tp_rank * m->ffn_local;
                }
            }
        }
    m->plan_effort = effort;
    return IAM_OK;
}

// One bucketMul launch of the step: the group kernel, or the cluster-split kernel.
int launch_plan(iam_model_s* m, int idx, bool pdl, cudaStream_t s) {
    if (m->use_group) {
        m->gplans[idx].pdl = pdl;
        return bg_launch(m->gplans[idx], s);
    }
    m->plans[idx].pdl = pdl;
    return bm_launch(m->plans[idx], m->vec, m->plans[idx].cluster, s);
}

// Optional per-launch CUDA events (diagnostics): an event is recorded before every launch
// together with the kind of the launch that follows, and once after the last launch.
struct StepHooks {
    std::vector<cudaEvent_t> ev;
    std::vector<int> kinds;
};

int hook(StepHooks* h, int kind, cudaStream_t s) {
    if (!h) return IAM_OK;
    cudaEvent_t e;
    IAM_CUDA_TRY(cudaEventCreate(&e));
    h->ev.push_back(e);
    h->kinds.push_back(kind);
    // external record: inside a stream capture this becomes an event-record node that the
    // host can time after the graph ran (a plain record would only order the capture)
    IAM_CUDA_TRY(cudaEventRecordWithFlags(e, s, cudaEventRecordExternal));
    return IAM_OK;
}

// Decode attention of layer l over the layer's KV cache at the model's device position:
// q, k, v from the q/k/v bucketMuls, output into this rank's heads of m->att.
AttnParams attn_params(iam_model_s* m, int l) {
    const iam_model_config& c = m->cfg;
    AttnParams ap{};
    ap.q = m->q;
    ap.k = m->k;
    ap.v = m->v;
    const size_t layer_kv = (size_t)m->n_kv_local * c.max_ctx * c.head_dim;
    ap.k_cache = m->k_cache + (size_t)l * layer_kv;
    ap.v_cache = m->v_cache + (size_t)l * layer_kv;
    ap.rope = m->rope;
    ap.pos_dev = m->pos;
    ap.pos_err = m->pos_err;
    ap.out = m->att + (size_t)m->tp_rank * m->n_heads_local * c.head_dim;
    ap.part = m->att_part;
    ap.ctr = m->att_ctr;
    ap.n_kv_heads = m->n_kv_local;
    ap.head_dim = c.head_dim;
    ap.max_ctx = c.max_ctx;
    ap.n_split = m->att_split;
    ap.min_chunk = m->att_min_chunk;
    ap.lane_min_ctx = m->att_lane_min;
    ap.lane_short_max = m->att_lane_short;
    if (push_mode(m)) {  // every head goes to the peers (o's cutoff reads them all)
        ap.tp_push = 1;
        ap.tp = m->win;
        ap.push_begin = m->tp_rank * m->n_heads_local * c.head_dim;
        ap.push_limit = c.n_heads * c.head_dim;
    }
    return ap;
}

// Launch bi (0 q/k/v, 1 o, 2 gate/up, 3 down) of layer l for the block-level entry points:
// x read as given (no fused RMSNorm), no residual added, o and down written to `out`.
int launch_plain_plan(iam_model_s* m, int l, int bi, const float* x, float* out, cudaStream_t s) {
    BGBatch b = m->gplans[(size_t)l * 4 + bi];
    for (int i = 0; i < b.nprob; ++i) {
        BGProblem& p = b.p[i];
        if (bi == 0 || bi == 2) {
            p.x = x;
            p.gain = nullptr;
        }
        if (bi == 1 || bi == 3) {
            p.residual = nullptr;
            p.out = out;
        }
        p.x_capture = nullptr;
        p.cutoff_out = nullptr;
    }
    if (bi == 0 || bi == 2) b.xmode = kXPlain;
    b.pdl = 0;
    bg_choose_shape(b);
    return bg_launch(b, s);
}

// The NVLink exchange after the row-parallel o (bi 1) or down (bi 3) of layer l: the ranges'
// partials of every rank added in range order plus the residual (x for o, x1 for down) into
// x1 or x, as one GPU adds them (tp_gather_reduce); the split-CTA kernel's rank sums are
// all-reduced instead.
int o_down_exchange(iam_model_s* m, int l, int bi, cudaStream_t s, bool pdl) {
    const iam_model_config& c = m->cfg;
    float* out = bi == 1 ? m->x1 : m->x;
    if (!m->use_group) return tp_allreduce_sum(m->win, woff(m, out), c.dim, s, pdl);
    if (m->gplans[(size_t)l * 4 + bi].tp_fused) return IAM_OK;  // done inside the kernel
    const BGBatch& b = m->gplans[(size_t)l * 4 + bi];
    const BGProblem& p = b.p[0];
    return tp_gather_reduce(m->win, p.partials, c.dim, p.n_ranges, bi == 1 ? m->x : m->x1, out,
                            m->sel + l * NMAT + (bi == 1 ? MO : MD), s, pdl);
}

// The launches of decoder layer l (transformer_layer.hpp:75-122): RMSNorm-fused q/k/v
// bucketMuls, attention with the RoPE'd fp16 KV append, o (+ the residual), RMSNorm-fused
// gate/up, SiLU-fused down (+ the residual), with the tensor-parallel exchanges between them.
// Reads m->x at the model's device position; leaves the layer's output in m->x.
int enqueue_layer(iam_model_s* m, int l, bool pdl, cudaStream_t s, StepHooks* hk) {
    const iam_model_config& c = m->cfg;
    const int gq = c.n_heads / c.n_kv_heads;
    int rc = IAM_OK;
    if ((rc = hook(hk, IAM_KERNEL_BUCKETMUL, s))) return rc;
    if ((rc = launch_plan(m, l * 4 + 0, pdl, s))) return rc;
    if (m->capture) {  // q, k, v of this layer (before attention rotates them)
        const CaptureLayout CL = capture_layout(c);
        float* rec = m->capture + (size_t)l * CL.total;
        const size_t qn = (size_t)c.n_heads * c.head_dim, kvn = (size_t)c.n_kv_heads * c.head_dim;
        IAM_CUDA_TRY(cudaMemcpyAsync(rec + CL.q, m->q, qn * 4, cudaMemcpyDeviceToDevice, s));
        IAM_CUDA_TRY(cudaMemcpyAsync(rec + CL.k, m->k, kvn * 4, cudaMemcpyDeviceToDevice, s));
        IAM_CUDA_TRY(cudaMemcpyAsync(rec + CL.v, m->v, kvn * 4, cudaMemcpyDeviceToDevice, s));
    }
    const AttnParams ap = attn_params(m, l);
    if ((rc = hook(hk, IAM_KERNEL_ATTENTION, s))) return rc;
    if ((rc = launch_attention(ap, gq, s, pdl))) return rc;
    for (int b = 1; b < 4; ++b) {
        if (m->tp_world > 1 && m->tp_p2p) {
            // the exchange in front of launch b (NVLink one-shot); none after a fused o launch,
            // which summed every rank's ranges itself, and none of the pushed heads and slices
            if (!(b == 2 && m->gplans[(size_t)l * 4 + 1].tp_fused) && !(b != 2 && push_mode(m))) {
                if ((rc = hook(hk, IAM_KERNEL_COLLECTIVE, s))) return rc;
                if (b == 1) rc = tp_allgather(m->win, woff(m, m->att), (size_t)-1, m->n_heads_local * c.head_dim, s, pdl);
                else if (b == 2) rc = o_down_exchange(m, l, 1, s, pdl);
                else rc = tp_allgather(m->win, woff(m, m->g), woff(m, m->u), m->ffn_local, s, pdl);
                if (rc) return rc;
            }
        } else if (m->tp_world > 1) {  // the exchange in front of launch b (NCCL)
            if ((rc = hook(hk, IAM_KERNEL_COLLECTIVE, s))) return rc;
            if (b == 1) rc = nccl_allgather(m, m->att, (size_t)m->n_heads_local * c.head_dim, s);
            else if (b == 2) rc = nccl_allreduce_sum(m, m->x1, c.dim, s);
            else {
                if ((rc = nccl_done(m, ncclGroupStart(), "ncclGroupStart"))) return rc;
                ncclAllGather(m->g + (size_t)m->tp_rank * m->ffn_local, m->g, m->ffn_local, ncclFloat, m->comm, s);
                ncclAllGather(m->u + (size_t)m->tp_rank * m->ffn_local, m->u, m->ffn_local, ncclFloat, m->comm, s);
                rc = nccl_done(m, ncclGroupEnd(), "ncclAllGather (gate, up)");
            }
            if (rc) return rc;
        }
        if ((rc = hook(hk, IAM_KERNEL_BUCKETMUL, s))) return rc;
        if (m->capture && b != 2)  // the residual this launch adds (o: x, down: x1)
            IAM_CUDA_TRY(cudaMemcpyAsync(m->capture + (size_t)l * capture_layout(c).total +
                                             (b == 1 ? capture_layout(c).reso : capture_layout(c).resd),
                                         b == 1 ? m->x : m->x1, (size_t)c.dim * 4, cudaMemcpyDeviceToDevice, s));
        if ((rc = launch_plan(m, l * 4 + b, pdl, s))) return rc;
        if (m->capture) {  // this launch's outputs
            const CaptureLayout CL = capture_layout(c);
            float* rec = m->capture + (size_t)l * CL.total;
            if (b == 1) IAM_CUDA_TRY(cudaMemcpyAsync(rec + CL.outo, m->x1, (size_t)c.dim * 4, cudaMemcpyDeviceToDevice, s));
            if (b == 2) {
                IAM_CUDA_TRY(cudaMemcpyAsync(rec + CL.g, m->g, (size_t)c.ffn_dim * 4, cudaMemcpyDeviceToDevice, s));
                IAM_CUDA_TRY(cudaMemcpyAsync(rec + CL.u, m->u, (size_t)c.ffn_dim * 4, cudaMemcpyDeviceToDevice, s));
            }
            if (b == 3) IAM_CUDA_TRY(cudaMemcpyAsync(rec + CL.outd, m->x, (size_t)c.dim * 4, cudaMemcpyDeviceToDevice, s));
        }
    }
    if (m->tp_world > 1 && !(m->tp_p2p && m->gplans[(size_t)l * 4 + 3].tp_fused)) {  // (down's: inside it)
        if ((rc = hook(hk, IAM_KERNEL_COLLECTIVE, s))) return rc;
        rc = m->tp_p2p ? o_down_exchange(m, l, 3, s, pdl) : nccl_allreduce_sum(m, m->x, c.dim, s);
        if (rc) return rc;
    }
    return IAM_OK;
}

// token: token_arg (>= 0), or the previous argmax when token_arg < 0.  pos: pos_arg (>= 0)
// is written to the device first, else the device value is used.
int enqueue_step(iam_model_s* m, int token_arg, int pos_arg, float effort, float* logits, cudaStream_t s,
                 StepHooks* hk = nullptr) {
    const iam_model_config& c = m->cfg;
    int rc = build_plans(m, effort);
    if (rc) return rc;
    // per-launch event hooks sit between the kernels, so they run without programmatic
    // serialization
    const bool pdl = m->pdl && !hk;
    if (pos_arg >= 0) IAM_CUDA_TRY(launch_ex(set_int_kernel, dim3(1), dim3(1), 0, s, pdl, m->pos, pos_arg));
    if ((rc = hook(hk, IAM_KERNEL_EMBED, s))) return rc;
    if ((rc = launch_embed(m->embed, c.dim, token_arg, token_arg < 0 ? m->key : nullptr, nullptr, m->x, m->key,
                           m->token_used, s, pdl)))
        return rc;
    for (int l = 0; l < c.n_layers; ++l)
        if ((rc = enqueue_layer(m, l, pdl, s, hk))) return rc;
    LMHeadParams hp{};
    hp.W = m->lm_head;  // this rank's vocabulary rows
    hp.x = m->x;
    hp.gain = m->final_norm;
    hp.eps = c.norm_eps;
    hp.dim = c.dim;
    hp.rows = m->vocab_local;
    hp.row0 = m->vocab0;
    // under the NVLink collectives the logits are gathered in the window, then copied out
    float* lg = (logits && m->tp_world > 1 && m->tp_p2p) ? m->logits : logits;
    hp.logits = lg ? lg + m->vocab0 : nullptr;
    hp.argmax_key = m->key;
    if ((rc = hook(hk, IAM_KERNEL_LM_HEAD, s))) return rc;
    if ((rc = launch_lm_head(hp, 2 * m->sm_count, s, pdl))) return rc;
    if (m->tp_world > 1 && m->tp_p2p) {
        if ((rc = hook(hk, IAM_KERNEL_COLLECTIVE, s))) return rc;
        if ((rc = tp_keymax(m->win, m->key, s, pdl))) return rc;
        if (logits) {
            if ((rc = tp_allgather(m->win, woff(m, m->logits), (size_t)-1, m->vocab_local, s, pdl))) return rc;
            if (logits != m->logits)
                IAM_CUDA_TRY(cudaMemcpyAsync(logits, m->logits, (size_t)c.vocab * 4, cudaMemcpyDeviceToDevice, s));
        }
    } else if (m->tp_world > 1) {  // the greedy token: max of the packed (logit, index) keys
        if ((rc = hook(hk, IAM_KERNEL_COLLECTIVE, s))) return rc;
        if ((rc = nccl_done(m, ncclAllReduce(m->key, m->key, 1, ncclUint64, ncclMax, m->comm, s), "argmax all-reduce")))
            return rc;
        if (logits && (rc = nccl_allgather(m, logits, m->vocab_local, s))) return rc;
    }
    return IAM_OK;
}

bool effort_ok(float e) { return std::isfinite(e) && e > 0.0f && e <= 1.0f; }

// Dense copies of every matrix and the chunk scratch of the prefill (once per model).
int build_prefill(iam_model_s* m, cudaStream_t s) {
    if (!m->dense.empty()) return IAM_OK;
    const iam_model_config& c = m->cfg;
    const int qn = c.n_heads * c.head_dim, kvn = c.n_kv_heads * c.head_dim, f = c.ffn_dim, d = c.dim;
    if (d % 8 || qn % 8 || f % 8) return fail(IAM_ERR_UNSUPPORTED, "prefill: dim, heads x head_dim and ffn_dim must be multiples of 8");
    int rc;
    std::vector<DenseLayer> dl(c.n_layers);
    for (int l = 0; l < c.n_layers; ++l) {
        DenseLayer& D = dl[l];
        const Layer& L = m->layers[l];
        if ((rc = dalloc(m, &D.qkv, (size_t)(qn + 2 * kvn) * d)) || (rc = dalloc(m, &D.o, (size_t)d * qn)) ||
            (rc = dalloc(m, &D.gu, (size_t)2 * f * d)) || (rc = dalloc(m, &D.down, (size_t)d * f)))
            return rc;
        // gate|up: with ffn a multiple of 128, blocks of 128 gate rows then the 128 up rows of
        // the same FFN columns (one 256-row product tile each: SiLU in the product's epilogue)
        const bool fused = f % (kDenseBW / 2) == 0;
        const int blk = fused ? kDenseBW / 2 : 0, pitch = fused ? kDenseBW : 0;
        struct Part { int which; uint16_t* dst; int rpb, pitch; };
        const Part parts[NMAT] = {{MQ, D.qkv, 0, 0},
                                  {MK, D.qkv + (size_t)qn * d, 0, 0},
                                  {MV, D.qkv + (size_t)(qn + kvn) * d, 0, 0},
                                  {MO, D.o, 0, 0},
                                  {MG, D.gu, blk, pitch},
                                  {MU, D.gu + (size_t)(fused ? blk : f) * d, blk, pitch},
                                  {MD, D.down, 0, 0}};
        for (const Part& p : parts) {
            const Matrix& mat = L.m[p.which];
            if ((rc = dense_unpack(mat.buckets, mat.in_dim, mat.cols, p.dst, mat.in_dim, s, p.rpb, p.pitch))) return rc;
        }
        m->pf_silu_fused = fused;
    }
    int cap = 256;
    if (const char* v = getenv("IAM_PREFILL_CHUNK")) cap = std::max(1, atoi(v));
    cap = std::min(cap, c.max_ctx);
    const size_t wide = (size_t)std::max(std::max(d, qn), f);
    if ((rc = dalloc(m, &m->pf_tok, (size_t)cap)) || (rc = dalloc(m, &m->pf_h, (size_t)cap * d)) ||
        (rc = dalloc(m, &m->pf_qkv, (size_t)cap * (qn + 2 * kvn))) || (rc = dalloc(m, &m->pf_att, (size_t)cap * qn)) ||
        (rc = dalloc(m, &m->pf_gu, (size_t)cap * 2 * f)) || (rc = dalloc(m, &m->pf_hi, (size_t)cap * wide)) ||
        (rc = dalloc(m, &m->pf_lo, (size_t)cap * wide)) || (rc = dalloc(m, &m->pf_hi2, (size_t)cap * f)) ||
        (rc = dalloc(m, &m->pf_lo2, (size_t)cap * f)) ||
        (rc = dalloc(m, &m->pf_part, dense_partial_floats(m->sm_count))) || (rc = dalloc(m, &m->pf_err, 1)))
        return rc;
    IAM_CUDA_TRY(cudaMemsetAsync(m->pf_err, 0, sizeof(unsigned), s));
    m->pf_cap = cap;
    m->dense.swap(dl);
    return IAM_OK;
}

// y[t][:] (+)= W x[t] with x given as the hi / lo halves [n][k] (default m->pf_hi / m->pf_lo).
int prefill_gemm(iam_model_s* m, const uint16_t* w, int out, int k, int n, float* y, const float* residual,
                 cudaStream_t s, const uint16_t* x_hi = nullptr, const uint16_t* x_lo = nullptr) {
    DenseProblem p{};
    p.w = w;
    p.m = out;
    p.k = k;
    p.ldw = k;
    p.x_hi = x_hi ? x_hi : m->pf_hi;
    p.x_lo = x_lo ? x_lo : m->pf_lo;
    p.n = n;
    p.y = y;
    p.ldy = out;
    p.residual = residual;
    p.ldr = out;
    p.partial = m->pf_part;
    p.split = dense_auto_split(out, k, n, m->sm_count);
    p.err = m->pf_err;
    return dense_gemm(p, s);
}

// Prompt tokens [c0, c0 + n) at positions pos0 + t through every layer; leaves the residual
// stream of its tokens in m->pf_h.
int prefill_chunk(iam_model_s* m, const int* tokens_host, int n, int pos0, cudaStream_t s) {
    const iam_model_config& c = m->cfg;
    const int qn = c.n_heads * c.head_dim, kvn = c.n_kv_heads * c.head_dim, f = c.ffn_dim, d = c.dim;
    const int ldq = qn + 2 * kvn;
    int rc;
    IAM_CUDA_TRY(cudaMemcpyAsync(m->pf_tok, tokens_host, (size_t)n * sizeof(int), cudaMemcpyHostToDevice, s));
    if ((rc = prefill_embed(m->embed, d, m->pf_tok, n, m->pf_h, s))) return rc;
    const size_t layer_kv = (size_t)c.n_kv_heads * c.max_ctx * c.head_dim;
    for (int l = 0; l < c.n_layers; ++l) {
        const Layer& L = m->layers[l];
        const DenseLayer& D = m->dense[l];
        uint16_t* kc = m->k_cache + (size_t)l * layer_kv;
        uint16_t* vc = m->v_cache + (size_t)l * layer_kv;
        if ((rc = prefill_rms_split(m->pf_h, n, d, L.attn_norm, c.norm_eps, m->pf_hi, m->pf_lo, s)) ||
            (rc = prefill_gemm(m, D.qkv, ldq, d, n, m->pf_qkv, nullptr, s)) ||
            (rc = prefill_rope_kv(m->pf_qkv, n, ldq, c.n_heads, c.n_kv_heads, c.head_dim, m->rope, pos0, kc, vc,
                                  c.max_ctx, s)) ||
            (rc = prefill_attention(m->pf_qkv, ldq, n, c.n_heads, c.n_kv_heads, c.head_dim, kc, vc, c.max_ctx, pos0,
                                    m->pf_att, qn, s)) ||
            (rc = dense_split(m->pf_att, n, qn, qn, m->pf_hi, m->pf_lo, s)) ||
            (rc = prefill_gemm(m, D.o, d, qn, n, m->pf_h, m->pf_h, s)) ||
            (rc = prefill_rms_split(m->pf_h, n, d, L.ffn_norm, c.norm_eps, m->pf_hi, m->pf_lo, s)))
            return rc;
        if (m->pf_silu_fused) {  // SiLU(gate) * up straight from the gate|up product's epilogue
            DenseProblem p{};
            p.w = D.gu;
            p.m = 2 * f;
            p.k = d;
            p.ldw = d;
            p.x_hi = m->pf_hi;
            p.x_lo = m->pf_lo;
            p.n = n;
            p.y = m->pf_gu;  // unused by this epilogue
            p.ldy = 2 * f;
            p.split = 1;
            p.err = m->pf_err;
            p.silu_out_hi = m->pf_hi2;
            p.silu_out_lo = m->pf_lo2;
            p.ld_silu = f;
            if ((rc = dense_gemm(p, s))) return rc;
        } else if ((rc = prefill_gemm(m, D.gu, 2 * f, d, n, m->pf_gu, nullptr, s)) ||
                   (rc = prefill_silu_split(m->pf_gu, n, f, m->pf_hi2, m->pf_lo2, s))) {
            return rc;
        }
        if ((rc = prefill_gemm(m, D.down, d, f, n, m->pf_h, m->pf_h, s, m->pf_hi2, m->pf_lo2))) return rc;
    }
    return IAM_OK;
}

// The dense copies the decode streams at efforts >= dense_min_effort (as much memory again as
// the bucket weights); skipped when that threshold is above 1.
int build_dense_copies(iam_model_s* m) {
    if (!(m->dense_min_effort <= 1.0f)) return IAM_OK;
    for (Layer& L : m->layers)
        for (Matrix& mat : L.m) {
            const int n_in = mat.in_end - mat.in_begin;
            int rc;
            if ((rc = dalloc(m, &mat.dense, (size_t)16 * mat.cols * n_in))) return rc;
            if ((rc = dense_unpack(mat.buckets, n_in, mat.cols, mat.dense, n_in, 0, 0, 0, true))) return rc;
        }
    return IAM_OK;
}

int finish_create(iam_model_s* m, iam_model_t* out) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        free_model(m);
        return cuda_fail(e, "model creation");
    }
    *out = m;
    return IAM_OK;
}

int init_common(iam_model_s* m, const iam_model_config* cfg, int device, int rank = 0, int world = 1,
                const unsigned char* nccl_id = nullptr) {
    int rc = check_cfg(cfg);
    if (rc) return rc;
    if ((rc = check_tp(*cfg, rank, world))) return rc;
    rc = iam_device_info(device, &m->sm_count, nullptr, nullptr);
    if (rc) return rc;
    IAM_CUDA_TRY(cudaSetDevice(device));
    m->cfg = *cfg;
    m->device = device;
    m->tp_rank = rank;
    m->tp_world = world;
    if (const char* v = getenv("IAM_PDL")) m->pdl = atoi(v) != 0;
    if (const char* v = getenv("IAM_BM_KERNEL")) m->use_group = std::string(v) != "split";
    if (const char* v = getenv("IAM_TP_TIMEOUT_S")) m->tp_timeout_s = atof(v);
    if (const char* v = getenv("IAM_TP_COLL")) m->tp_p2p = std::string(v) != "nccl";
    if (const char* v = getenv("IAM_TP_FUSED")) m->tp_fused = std::string(v) != "0";
    if (const char* v = getenv("IAM_TP_PUSH")) m->tp_push = std::string(v) != "0";
    m->n_heads_local = cfg->n_heads / world;
    m->n_kv_local = cfg->n_kv_heads / world;
    m->ffn_local = cfg->ffn_dim / world;
    m->vocab_local = cfg->vocab / world;
    m->vocab0 = rank * m->vocab_local;
    if (world > 1) {
        if (!nccl_id) return fail(IAM_ERR_ARG, "tensor parallel: null NCCL id");
        if ((rc = dalloc(m, &m->tp_tmp, 4))) return rc;
        ncclUniqueId id;
        std::memcpy(&id, nccl_id, sizeof(id));
        ncclConfig_t conf = NCCL_CONFIG_INITIALIZER;
        conf.blocking = 0;  // bounded wait for the peers instead of blocking forever
        if ((rc = nccl_done(m, ncclCommInitRankConfig(&m->comm, world, id, rank, &conf), "ncclCommInitRank")))
            return rc;
    }
    m->layers.assign(cfg->n_layers, Layer{});
    const char* g = getenv("IAM_BM_CLUSTER");
    m->G = g && *g ? atoi(g) : bm_default_cluster();
    const char* v = getenv("IAM_BM_VEC");
    m->vec = v && (atoi(v) == 8 || atoi(v) == 1) ? atoi(v) : 4;
    return IAM_OK;
}

int create_random(iam_model_t* out, const iam_model_config* cfg, unsigned long long seed, int device, int rank,
                  int world, const unsigned char* nccl_id) {
    if (!out) return fail(IAM_ERR_ARG, "iam_model_create_random: null out");
    *out = nullptr;
    iam_model_s* m = new iam_model_s();
    int rc = init_common(m, cfg, device, rank, world, nccl_id);
    if (rc) {
        free_model(m);
        return rc;
    }
    const iam_model_config& c = m->cfg;
    const int qn = c.n_heads * c.head_dim;
    const size_t wmax = (size_t)std::max(std::max(qn, c.dim), c.ffn_dim) * std::max(c.dim, c.ffn_dim);
    uint16_t *wtmp = nullptr, *btmp = nullptr;  // full matrix and, when sharding, its full buckets
    cudaError_t e = cudaMalloc(&wtmp, wmax * 2);
    if (e == cudaSuccess && world > 1) e = cudaMalloc(&btmp, wmax * 2);
    if (e != cudaSuccess) rc = cuda_fail(e, "model build scratch");
    const uint16_t one = 0x3c00;  // fp16 1.0: RMSNorm gains of the random-init benchmark model
    unsigned long long tensor = 1;
    for (int l = 0; l < c.n_layers && !rc; ++l) {
        Layer& L = m->layers[l];
        for (int i = 0; i < NMAT && !rc; ++i) rc = make_matrix_random(m, L.m[i], i, seed, tensor++, wtmp, btmp);
        if (!rc && !(rc = dalloc(m, &L.attn_norm, c.dim)) && !(rc = dalloc(m, &L.ffn_norm, c.dim))) {
            fill_u16<<<8, 256>>>(L.attn_norm, c.dim, one);
            fill_u16<<<8, 256>>>(L.ffn_norm, c.dim, one);
        }
    }
    if (!rc && !(rc = dalloc(m, &m->embed, (size_t)c.vocab * c.dim)) && !(rc = dalloc(m, &m->final_norm, c.dim))) {
        init_normal_fp16<<<4 * m->sm_count, 256>>>(m->embed, (size_t)c.vocab * c.dim, seed, 0, 0.02f);
        fill_u16<<<8, 256>>>(m->final_norm, c.dim, one);
        m->lm_head = m->embed + (size_t)m->vocab0 * c.dim;  // tied embeddings (the random-init 32000-token model)
        if (!c.tied_embeddings && !(rc = dalloc(m, &m->lm_head, (size_t)m->vocab_local * c.dim)))
            init_normal_fp16<<<4 * m->sm_count, 256>>>(m->lm_head, (size_t)m->vocab_local * c.dim, seed, tensor++,
                                                       0.02f, (size_t)m->vocab0 * c.dim);
    }
    if (!rc) {
        e = cudaDeviceSynchronize();
        if (e != cudaSuccess) rc = cuda_fail(e, "model build");
    }
    cudaFree(wtmp);
    cudaFree(btmp);
    if (!rc) rc = alloc_runtime(m);
    if (!rc) rc = build_dense_copies(m);  // before the agreement: a rank that fails here stops every rank
    rc = tp_agree(m, rc);
    if (!rc) rc = tp_agree(m, tp_map_peers(m));
    if (rc) {
        free_model(m);
        return rc;
    }
    return finish_create(m, out);
}

int load_model(iam_model_t* out, const char* weights_dir, const iam_model_config* cfg, int device, int rank,
               int world, const unsigned char* nccl_id) {
    if (!out || !weights_dir) return fail(IAM_ERR_ARG, "iam_model_load: null argument");
    *out = nullptr;
    iam_model_s* m = new iam_model_s();
    int rc = init_common(m, cfg, device, rank, world, nccl_id);
    if (rc) {
        free_model(m);
        return rc;
    }
    const iam_model_config& c = m->cfg;
    const std::string dir(weights_dir);
    int dims_out[NMAT], dims_in[NMAT];
    for (int i = 0; i < NMAT; ++i) matrix_dims(c, i, &dims_out[i], &dims_in[i]);
    std::vector<uint16_t> buf;
    for (int l = 0; l < c.n_layers && !rc; ++l) {
        Layer& L = m->layers[l];
        for (int i = 0; i < NMAT && !rc; ++i) rc = load_matrix(m, dir, l, i, dims_out[i], dims_in[i], L.m[i]);
        const std::string lp = dir + "/layer" + std::to_string(l);
        if (!rc && !(rc = read_npy_u16(lp + "_input_layernorm.npy", c.dim, buf))) rc = upload(m, &L.attn_norm, buf);
        if (!rc && !(rc = read_npy_u16(lp + "_post_attention_layernorm.npy", c.dim, buf))) rc = upload(m, &L.ffn_norm, buf);
    }
    if (!rc && !(rc = read_npy_u16(dir + "/embed_tokens.npy", (size_t)c.vocab * c.dim, buf))) rc = upload(m, &m->embed, buf);
    if (!rc && !(rc = read_npy_u16(dir + "/norm_weight.npy", c.dim, buf))) rc = upload(m, &m->final_norm, buf);
    if (!rc) {
        if (c.tied_embeddings) {
            m->lm_head = m->embed + (size_t)m->vocab0 * c.dim;
        } else if (!(rc = read_npy_u16(dir + "/lm_head.npy", (size_t)c.vocab * c.dim, buf))) {
            std::vector<uint16_t> part(buf.begin() + (size_t)m->vocab0 * c.dim,
                                       buf.begin() + (size_t)(m->vocab0 + m->vocab_local) * c.dim);
            rc = upload(m, &m->lm_head, part);
        }
    }
    if (!rc) rc = alloc_runtime(m);
    if (!rc) rc = build_dense_copies(m);  // before the agreement: a rank that fails here stops every rank
    rc = tp_agree(m, rc);
    if (!rc) rc = tp_agree(m, tp_map_peers(m));
    if (rc) {
        free_model(m);
        return rc;
    }
    return finish_create(m, out);
}

}  // namespace

extern "C" {

int iam_tp_unique_id(unsigned char* id_out) {
    if (!id_out) return fail(IAM_ERR_ARG, "iam_tp_unique_id: null argument");
    static_assert(sizeof(ncclUniqueId) == IAM_TP_ID_BYTES, "NCCL id size");
    ncclUniqueId id;
    const ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) return fail(IAM_ERR_NCCL, std::string("ncclGetUniqueId: ") + ncclGetErrorString(r));
    std::memcpy(id_out, &id, sizeof(id));
    return IAM_OK;
}

int iam_tp_shard_info(const iam_model_config* cfg, int rank, int world, int* out) {
    if (!cfg || !out) return fail(IAM_ERR_ARG, "iam_tp_shard_info: null argument");
    int rc = check_cfg(cfg);
    if (rc || (rc = check_tp(*cfg, rank, world))) return rc;
    for (int i = 0; i < NMAT; ++i) {
        const Shard sh = shard_of(*cfg, i, rank, world);
        out[4 * i + 0] = sh.col0;
        out[4 * i + 1] = sh.cols;
        out[4 * i + 2] = sh.in0;
        out[4 * i + 3] = sh.in1;
    }
    out[4 * NMAT] = rank * (cfg->vocab / world);
    out[4 * NMAT + 1] = cfg->vocab / world;
    return IAM_OK;
}

int iam_model_create_random(iam_model_t* out, const iam_model_config* cfg, unsigned long long seed, int device) {
    return create_random(out, cfg, seed, device, 0, 1, nullptr);
}

int iam_model_create_random_tp(iam_model_t* out, const iam_model_config* cfg, unsigned long long seed, int device,
                               int rank, int world, const unsigned char* nccl_id) {
    return create_random(out, cfg, seed, device, rank, world, nccl_id);
}

int iam_model_load(iam_model_t* out, const char* weights_dir, const iam_model_config* cfg, int device) {
    return load_model(out, weights_dir, cfg, device, 0, 1, nullptr);
}

int iam_model_load_tp(iam_model_t* out, const char* weights_dir, const iam_model_config* cfg, int device, int rank,
                      int world, const unsigned char* nccl_id) {
    return load_model(out, weights_dir, cfg, device, rank, world, nccl_id);
}

int iam_model_destroy(iam_model_t m) {
    if (m) free_model(m);
    return IAM_OK;
}

int iam_model_reset(iam_model_t m, void* stream) {
    if (!m) return fail(IAM_ERR_ARG, "iam_model_reset: null model");
    const size_t kv = (size_t)m->cfg.n_layers * m->n_kv_local * m->cfg.max_ctx * m->cfg.head_dim * 2;
    IAM_CUDA_TRY(cudaMemsetAsync(m->k_cache, 0, kv, (cudaStream_t)stream));
    IAM_CUDA_TRY(cudaMemsetAsync(m->v_cache, 0, kv, (cudaStream_t)stream));
    IAM_CUDA_TRY(cudaMemsetAsync(m->pos, 0, sizeof(int), (cudaStream_t)stream));
    m->host_pos = 0;
    return IAM_OK;
}

int iam_model_forward(iam_model_t m, int token, int pos, float effort, float* logits_dev, void* stream) {
    if (!m) return fail(IAM_ERR_ARG, "iam_model_forward: null model");
    if (token < 0 || token >= m->cfg.vocab) return fail(IAM_ERR_ARG, "iam_model_forward: token out of range");
    if (pos < 0 || pos >= m->cfg.max_ctx) return fail(IAM_ERR_ARG, "iam_model_forward: pos out of range");
    if (!effort_ok(effort)) return fail(IAM_ERR_ARG, "iam_model_forward: effort must be in (0, 1]");
    const int rc = enqueue_step(m, token, pos, effort, logits_dev ? logits_dev : m->logits, (cudaStream_t)stream);
    if (!rc) m->host_pos = pos;
    return rc;
}

int iam_model_prefill(iam_model_t m, const int* tokens_host, int n_tokens, int start_pos, float* logits_dev,
                      int* next_token, void* stream) {
    if (!m || !tokens_host) return fail(IAM_ERR_ARG, "iam_model_prefill: null argument");
    if (m->tp_world > 1) return fail(IAM_ERR_UNSUPPORTED, "iam_model_prefill: single-GPU models only");
    const iam_model_config& c = m->cfg;
    if (n_tokens <= 0 || start_pos < 0 || (long long)start_pos + n_tokens > c.max_ctx)
        return fail(IAM_ERR_ARG, "iam_model_prefill: positions outside [0, max_ctx)");
    for (int i = 0; i < n_tokens; ++i)
        if (tokens_host[i] < 0 || tokens_host[i] >= c.vocab) return fail(IAM_ERR_ARG, "iam_model_prefill: token out of range");
    IAM_CUDA_TRY(cudaSetDevice(m->device));
    const cudaStream_t s = (cudaStream_t)stream;
    int rc = build_prefill(m, s);
    if (rc) return rc;
    int last_rows = 0;
    for (int c0 = 0; c0 < n_tokens; c0 += m->pf_cap) {
        last_rows = std::min(m->pf_cap, n_tokens - c0);
        if ((rc = prefill_chunk(m, tokens_host + c0, last_rows, start_pos + c0, s))) return rc;
    }
    IAM_CUDA_TRY(cudaMemsetAsync(m->key, 0, sizeof(unsigned long long), s));
    LMHeadParams hp{};
    hp.W = m->lm_head;
    hp.x = m->pf_h + (size_t)(last_rows - 1) * c.dim;
    hp.gain = m->final_norm;
    hp.eps = c.norm_eps;
    hp.dim = c.dim;
    hp.rows = m->vocab_local;
    hp.row0 = m->vocab0;
    hp.logits = logits_dev;
    hp.argmax_key = m->key;
    if ((rc = launch_lm_head(hp, 2 * m->sm_count, s, false))) return rc;
    // decoding continues after the prompt (iam_model_generate with first_token < 0 takes the
    // prefill's greedy token from the argmax slot and this position)
    IAM_CUDA_TRY(launch_ex(set_int_kernel, dim3(1), dim3(1), 0, s, false, m->pos, start_pos + n_tokens));
    m->host_pos = start_pos + n_tokens;
    if (next_token) {
        IAM_CUDA_TRY(cudaStreamSynchronize(s));
        unsigned err = 0;
        unsigned long long key = 0;
        IAM_CUDA_TRY(cudaMemcpy(&err, m->pf_err, sizeof(err), cudaMemcpyDeviceToHost));
        if (err) return fail(IAM_ERR_TIMEOUT, "iam_model_prefill: a dense-product pipeline wait gave up");
        IAM_CUDA_TRY(cudaMemcpy(&key, m->key, sizeof(key), cudaMemcpyDeviceToHost));
        *next_token = (int)(0xffffffffu - (unsigned)(key & 0xffffffffull));
    }
    return IAM_OK;
}

int iam_model_generate(iam_model_t m, int first_token, int start_pos, int n_tokens, float effort, int* tokens_dev,
                       void* stream) {
    if (!m || !tokens_dev) return fail(IAM_ERR_ARG, "iam_model_generate: null argument");
    const bool cont = first_token < 0;  // continue from the device position and last argmax
    if (first_token >= m->cfg.vocab) return fail(IAM_ERR_ARG, "iam_model_generate: bad token");
    if (n_tokens < 0) return fail(IAM_ERR_ARG, "iam_model_generate: negative n_tokens");
    if (!cont && (start_pos < 0 || (long long)start_pos + n_tokens > m->cfg.max_ctx))
        return fail(IAM_ERR_ARG, "iam_model_generate: positions exceed max_ctx");
    // continuing decodes at the device position, which the host tracks: refused before any
    // launch when the steps would run past the KV cache
    if (cont && (long long)m->host_pos + n_tokens > m->cfg.max_ctx)
        return fail(IAM_ERR_ARG, "iam_model_generate: continuing would decode past max_ctx");
    if (!effort_ok(effort)) return fail(IAM_ERR_ARG, "iam_model_generate: effort must be in (0, 1]");
    cudaStream_t s = (cudaStream_t)stream;
    if (n_tokens == 0) return IAM_OK;
    // step 0 from the given token (eager) unless continuing, then one captured step replayed
    // per token; each step appends its greedy token to tokens_dev[gen_count++] and advances
    // pos on the device
    IAM_CUDA_TRY(cudaMemsetAsync(m->gen_count, 0, sizeof(int), s));
    int rc = IAM_OK;
    int done = 0;
    if (!cont) {
        if ((rc = enqueue_step(m, first_token, start_pos, effort, m->tp_world > 1 ? nullptr : m->logits, s)))
            return rc;
        if ((rc = launch_advance(m->pos, m->key, tokens_dev, m->gen_count, m->cfg.max_ctx, s, m->pdl))) return rc;
        done = 1;
        if (n_tokens == 1) return IAM_OK;
    }
    if (!m->gen_graph || m->gen_effort != effort || m->gen_tokens != tokens_dev) {
        if (m->gen_graph) {
            cudaGraphExecDestroy(m->gen_graph);
            m->gen_graph = nullptr;
        }
        cudaStream_t cap;
        IAM_CUDA_TRY(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking));
        cudaGraph_t graph = nullptr;
        cudaError_t e = cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal);
        if (e == cudaSuccess) {
            // greedy generation needs only the argmax key: under tensor parallelism the
            // logits all-gather is left out
            rc = enqueue_step(m, -1, -1, effort, m->tp_world > 1 ? nullptr : m->logits, cap);
            if (!rc) rc = launch_advance(m->pos, m->key, tokens_dev, m->gen_count, m->cfg.max_ctx, cap, m->pdl);
            e = cudaStreamEndCapture(cap, &graph);
        }
        if (e == cudaSuccess && !rc) e = cudaGraphInstantiate(&m->gen_graph, graph, 0);
        if (graph) cudaGraphDestroy(graph);
        cudaStreamDestroy(cap);
        if (rc) return rc;
        if (e != cudaSuccess) return cuda_fail(e, "iam_model_generate: graph capture");
        m->gen_effort = effort;
        m->gen_tokens = tokens_dev;
    }
    for (int i = done; i < n_tokens; ++i) IAM_CUDA_TRY(cudaGraphLaunch(m->gen_graph, s));
    m->host_pos = (cont ? m->host_pos : start_pos) + n_tokens;
    return IAM_OK;
}

int iam_model_profile_steps(iam_model_t m, float effort, int steps, float* kernel_ms, int* kinds, int capacity,
                            int* n_kernels, void* stream) {
    if (!m || steps <= 0 || !n_kernels) return fail(IAM_ERR_ARG, "iam_model_profile_steps: bad arguments");
    if (!effort_ok(effort)) return fail(IAM_ERR_ARG, "iam_model_profile_steps: effort must be in (0, 1]");
    if ((long long)m->host_pos + steps > m->cfg.max_ctx)
        return fail(IAM_ERR_ARG, "iam_model_profile_steps: the steps would decode past max_ctx");
    cudaStream_t s = (cudaStream_t)stream;
    int rc = build_plans(m, effort);
    if (rc) return rc;
    StepHooks hk;
    cudaStream_t cap;
    IAM_CUDA_TRY(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking));
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    cudaError_t e = cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal);
    if (e == cudaSuccess) {
        rc = enqueue_step(m, -1, -1, effort, m->logits, cap, &hk);
        if (!rc) rc = hook(&hk, IAM_KERNEL_OTHER, cap);
        if (!rc) rc = launch_advance(m->pos, m->key, nullptr, nullptr, m->cfg.max_ctx, cap);
        if (!rc) rc = hook(&hk, IAM_KERNEL_OTHER, cap);
        e = cudaStreamEndCapture(cap, &graph);
    }
    if (e == cudaSuccess && !rc) e = cudaGraphInstantiate(&exec, graph, 0);
    const int nk = (int)hk.ev.size() - 1;
    std::vector<double> acc(nk > 0 ? nk : 0, 0.0);
    for (int it = 0; it < steps && e == cudaSuccess && !rc; ++it) {
        e = cudaGraphLaunch(exec, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        for (int k = 0; k < nk && e == cudaSuccess; ++k) {
            float ms = 0.0f;
            e = cudaEventElapsedTime(&ms, hk.ev[k], hk.ev[k + 1]);
            acc[k] += ms;
        }
    }
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    cudaStreamDestroy(cap);
    for (cudaEvent_t ev : hk.ev) cudaEventDestroy(ev);
    if (rc) return rc;
    if (e != cudaSuccess) return cuda_fail(e, "iam_model_profile_steps");
    m->host_pos += steps;
    *n_kernels = nk;
    for (int k = 0; k < nk && k < capacity; ++k) {
        if (kernel_ms) kernel_ms[k] = (float)(acc[k] / steps);
        if (kinds) kinds[k] = hk.kinds[k];
    }
    return IAM_OK;
}

int iam_model_set_kv(iam_model_t m, int layer, const uint16_t* k_dev, const uint16_t* v_dev, int n_tokens,
                     void* stream) {
    if (!m || !k_dev || !v_dev) return fail(IAM_ERR_ARG, "iam_model_set_kv: null argument");
    if (layer < 0 || layer >= m->cfg.n_layers || n_tokens < 0 || n_tokens > m->cfg.max_ctx)
        return fail(IAM_ERR_ARG, "iam_model_set_kv: bad layer or n_tokens");
    const size_t hd = m->cfg.head_dim, ctx = m->cfg.max_ctx;
    const size_t layer_kv = (size_t)m->n_kv_local * ctx * hd;
    const size_t h0 = (size_t)m->tp_rank * m->n_kv_local;  // this rank's first kv head
    for (int h = 0; h < m->n_kv_local; ++h) {
        uint16_t* kd = m->k_cache + layer * layer_kv + h * ctx * hd;
        uint16_t* vd = m->v_cache + layer * layer_kv + h * ctx * hd;
        IAM_CUDA_TRY(cudaMemcpyAsync(kd, k_dev + (h0 + h) * n_tokens * hd, n_tokens * hd * 2, cudaMemcpyDefault,
                                     (cudaStream_t)stream));
        IAM_CUDA_TRY(cudaMemcpyAsync(vd, v_dev + (h0 + h) * n_tokens * hd, n_tokens * hd * 2, cudaMemcpyDefault,
                                     (cudaStream_t)stream));
    }
    return IAM_OK;
}

int iam_model_fill_kv_random(iam_model_t m, int n_tokens, unsigned long long seed, void* stream) {
    if (!m || n_tokens < 0 || n_tokens > m->cfg.max_ctx) return fail(IAM_ERR_ARG, "iam_model_fill_kv_random: bad arguments");
    const size_t hd = m->cfg.head_dim, ctx = m->cfg.max_ctx;
    for (int l = 0; l < m->cfg.n_layers; ++l)
        for (int h = 0; h < m->n_kv_local; ++h) {
            const size_t off = ((size_t)l * m->n_kv_local + h) * ctx * hd;
            const unsigned long long hg = (unsigned long long)m->tp_rank * m->n_kv_local + h;  // global kv head
            const unsigned long long t = 0x4b560000ull + ((unsigned long long)l << 8) + hg;
            init_normal_fp16<<<m->sm_count, 256, 0, (cudaStream_t)stream>>>(m->k_cache + off, n_tokens * hd, seed, 2 * t, 1.0f);
            init_normal_fp16<<<m->sm_count, 256, 0, (cudaStream_t)stream>>>(m->v_cache + off, n_tokens * hd, seed, 2 * t + 1, 1.0f);
        }
    IAM_CUDA_TRY(cudaGetLastError());
    return IAM_OK;
}

int iam_model_read_weight(iam_model_t m, int layer, int which, void* host_dst, size_t capacity_bytes,
                          size_t* bytes_out) {
    if (!m) return fail(IAM_ERR_ARG, "iam_model_read_weight: null model");
    const iam_model_config& c = m->cfg;
    const void* src = nullptr;
    size_t bytes = 0;
    if (which == IAM_W_EMBED) {
        src = m->embed;
        bytes = (size_t)c.vocab * c.dim * 2;
    } else if (which == IAM_W_FINAL_NORM) {
        src = m->final_norm;
        bytes = (size_t)c.dim * 2;
    } else if (which == IAM_W_LM_HEAD) {
        src = m->lm_head;
        bytes = (size_t)m->vocab_local * c.dim * 2;
    } else {
        if (layer < 0 || layer >= c.n_layers) return fail(IAM_ERR_ARG, "iam_model_read_weight: bad layer");
        const Layer& L = m->layers[layer];
        if (which == IAM_W_ATTN_NORM) {
            src = L.attn_norm;
            bytes = (size_t)c.dim * 2;
        } else if (which == IAM_W_FFN_NORM) {
            src = L.ffn_norm;
            bytes = (size_t)c.dim * 2;
        } else if (which == IAM_W_K_CACHE || which == IAM_W_V_CACHE) {
            const size_t layer_kv = (size_t)m->n_kv_local * c.max_ctx * c.head_dim;
            src = (which == IAM_W_K_CACHE ? m->k_cache : m->v_cache) + layer * layer_kv;
            bytes = layer_kv * 2;
        } else if (which >= IAM_W_MATRIX && which < IAM_W_MATRIX + 3 * NMAT) {
            const Matrix& mt = L.m[(which - IAM_W_MATRIX) / 3];
            const int part = (which - IAM_W_MATRIX) % 3;
            const size_t rows = 16 * (size_t)(mt.in_end - mt.in_begin);
            src = part == 0 ? (const void*)mt.buckets : part == 1 ? (const void*)mt.stats : (const void*)mt.probes;
            bytes = part == 0 ? rows * mt.cols * 2 : part == 1 ? 16 * (size_t)mt.in_dim * 2 : (size_t)mt.in_dim * 2;
        } else {
            return fail(IAM_ERR_ARG, "iam_model_read_weight: unknown weight id");
        }
    }
    if (bytes_out) *bytes_out = bytes;
    if (!host_dst) return IAM_OK;
    if (capacity_bytes < bytes) return fail(IAM_ERR_ARG, "iam_model_read_weight: buffer too small");
    IAM_CUDA_TRY(cudaMemcpy(host_dst, src, bytes, cudaMemcpyDeviceToHost));
    return IAM_OK;
}

}  // extern "C"

namespace {

// NumPy .npy (format 1.0) of fp16 values: the header dict padded to a multiple of 64 bytes.
bool write_npy_f16(const std::string& path, const std::vector<uint16_t>& v, const std::vector<long>& shape) {
    std::string dict = "{'descr': '<f2', 'fortran_order': False, 'shape': (";
    for (size_t i = 0; i < shape.size(); ++i) dict += std::to_string(shape[i]) + (shape.size() == 1 ? "," : (i + 1 < shape.size() ? ", " : ""));
    dict += "), }";
    size_t total = 10 + dict.size() + 1;
    const size_t pad = (64 - total % 64) % 64;
    dict += std::string(pad, ' ') + "\n";
    std::ofstream f(path, std::ios::binary);
    if (!f) return false;
    const uint16_t hlen = (uint16_t)dict.size();
    f.write("\x93NUMPY\x01\x00", 8);
    f.put((char)(hlen & 0xff));
    f.put((char)(hlen >> 8));
    f.write(dict.data(), (std::streamsize)dict.size());
    f.write(reinterpret_cast<const char*>(v.data()), (std::streamsize)(v.size() * 2));
    return (bool)f;
}

bool write_u16(const std::string& path, const std::vector<uint16_t>& v) {
    std::ofstream f(path, std::ios::binary);
    if (!f) return false;
    f.write(reinterpret_cast<const char*>(v.data()), (std::streamsize)(v.size() * 2));
    return (bool)f;
}

int download(const uint16_t* src, size_t n, std::vector<uint16_t>& out) {
    out.resize(n);
    IAM_CUDA_TRY(cudaMemcpy(out.data(), src, n * 2, cudaMemcpyDeviceToHost));
    return IAM_OK;
}

}  // namespace

extern "C" {

int iam_model_save(iam_model_t m, const char* weights_dir) {
    if (!m || !weights_dir) return fail(IAM_ERR_ARG, "iam_model_save: null argument");
    if (m->tp_world > 1) return fail(IAM_ERR_UNSUPPORTED, "iam_model_save: a tensor-parallel rank holds a shard only");
    const iam_model_config& c = m->cfg;
    const std::string dir(weights_dir);
    std::vector<uint16_t> a, b;
    int rc = IAM_OK;
    for (int l = 0; l < c.n_layers && !rc; ++l) {
        const Layer& L = m->layers[l];
        for (int i = 0; i < NMAT && !rc; ++i) {
            const Matrix& mt = L.m[i];
            const std::string prefix = dir + "/layer" + std::to_string(l) + "_" + kMatNames[i] + "_proj_bucketmul_fp16";
            const size_t R = (size_t)16 * mt.in_dim;
            if ((rc = download(mt.buckets, R * mt.cols, a))) break;
            if (!write_u16(prefix + "_buckets.bin", a)) rc = fail(IAM_ERR_IO, "cannot write " + prefix + "_buckets.bin");
            if (rc || (rc = download(mt.stats, R, a))) break;
            b.resize(R * 4);  // the file keeps 4 identical channels per row (preprocess_layer_fixed_gpu.py:217-221)
            for (size_t r = 0; r < R; ++r) b[4 * r] = b[4 * r + 1] = b[4 * r + 2] = b[4 * r + 3] = a[r];
            if (!write_u16(prefix + "_stats.bin", b)) rc = fail(IAM_ERR_IO, "cannot write " + prefix + "_stats.bin");
            if (rc || (rc = download(mt.probes, (size_t)mt.in_dim, a))) break;
            if (!write_u16(prefix + "_probes.bin", a)) rc = fail(IAM_ERR_IO, "cannot write " + prefix + "_probes.bin");
            std::ofstream f(prefix + "_meta.txt");  // preprocess_layer_fixed_gpu.py:262-282
            f << "# BucketMul Weight Metadata\n# All arrays are FP16 (2 bytes per element)\n\n"
              << "buckets_shape: 1 " << R << " " << mt.cols << "\nstats_shape: 1 " << R << " 4\nprobes_shape: 1 " << mt.in_dim
              << "\nin_dim: " << mt.in_dim << "\nout_dim: " << mt.out_dim << "\nbsize: 16\ndtype: float16\n";
            if (!rc && !f) rc = fail(IAM_ERR_IO, "cannot write " + prefix + "_meta.txt");
        }
        const std::string lp = dir + "/layer" + std::to_string(l);
        if (!rc && !(rc = download(L.attn_norm, c.dim, a)) && !write_npy_f16(lp + "_input_layernorm.npy", a, {c.dim}))
            rc = fail(IAM_ERR_IO, "cannot write " + lp + "_input_layernorm.npy");
        if (!rc && !(rc = download(L.ffn_norm, c.dim, a)) && !write_npy_f16(lp + "_post_attention_layernorm.npy", a, {c.dim}))
            rc = fail(IAM_ERR_IO, "cannot write " + lp + "_post_attention_layernorm.npy");
    }
    if (!rc && !(rc = download(m->embed, (size_t)c.vocab * c.dim, a)) &&
        !write_npy_f16(dir + "/embed_tokens.npy", a, {c.vocab, c.dim}))
        rc = fail(IAM_ERR_IO, "cannot write " + dir + "/embed_tokens.npy");
    if (!rc && !(rc = download(m->final_norm, c.dim, a)) && !write_npy_f16(dir + "/norm_weight.npy", a, {c.dim}))
        rc = fail(IAM_ERR_IO, "cannot write " + dir + "/norm_weight.npy");
    if (!rc && !c.tied_embeddings && !(rc = download(m->lm_head, (size_t)c.vocab * c.dim, a)) &&
        !write_npy_f16(dir + "/lm_head.npy", a, {c.vocab, c.dim}))
        rc = fail(IAM_ERR_IO, "cannot write " + dir + "/lm_head.npy");
    return rc;
}

int iam_model_capture_floats(const iam_model_config* cfg, long long* floats) {
    if (!cfg || !floats) return fail(IAM_ERR_ARG, "iam_model_capture_floats: null argument");
    int rc = check_cfg(cfg);
    if (rc) return rc;
    *floats = (long long)capture_layout(*cfg).total * cfg->n_layers;
    return IAM_OK;
}

int iam_model_capture(iam_model_t m, float* buf_dev, size_t capacity_floats) {
    if (!m) return fail(IAM_ERR_ARG, "iam_model_capture: null model");
    if (buf_dev) {
        if (m->tp_world > 1) return fail(IAM_ERR_UNSUPPORTED, "iam_model_capture: single-GPU models only");
        if (!m->use_group) return fail(IAM_ERR_UNSUPPORTED, "iam_model_capture: needs the range bucketMul kernel");
        if (capacity_floats < capture_layout(m->cfg).total * (size_t)m->cfg.n_layers)
            return fail(IAM_ERR_ARG, "iam_model_capture: buffer smaller than iam_model_capture_floats");
    }
    m->capture = buf_dev;
    m->plan_effort = -1.0f;  // plans carry the capture pointers: rebuilt at the next step
    if (m->gen_graph) {
        cudaGraphExecDestroy(m->gen_graph);
        m->gen_graph = nullptr;
    }
    return IAM_OK;
}

int iam_model_selected_rows_by_matrix(iam_model_t m, int* counts, int capacity) {
    if (!m || !counts) return fail(IAM_ERR_ARG, "iam_model_selected_rows_by_matrix: null argument");
    const int n = m->cfg.n_layers * NMAT;
    if (capacity < n) return fail(IAM_ERR_ARG, "iam_model_selected_rows_by_matrix: capacity < 7 * n_layers");
    IAM_CUDA_TRY(cudaMemcpy(counts, m->sel, (size_t)n * sizeof(int), cudaMemcpyDeviceToHost));
    return IAM_OK;
}

int iam_model_status(iam_model_t m) {
    if (!m) return fail(IAM_ERR_ARG, "iam_model_status: null model");
    IAM_CUDA_TRY(cudaDeviceSynchronize());
    if (m->xwin) {
        uint32_t err = 0;
        IAM_CUDA_TRY(cudaMemcpy(&err, m->xwin + m->win.err_off, sizeof(err), cudaMemcpyDeviceToHost));
        if (err) return fail(IAM_ERR_TIMEOUT, "a tensor-parallel peer did not answer within the wait limit");
    }
    unsigned bar[4] = {0, 0, 0, 0};
    IAM_CUDA_TRY(cudaMemcpy(bar, m->bm_bar, sizeof(bar), cudaMemcpyDeviceToHost));
    if (bar[2]) return fail(IAM_ERR_TIMEOUT, "a bucketMul launch gave up waiting at its grid barrier");
    int perr = 0;
    IAM_CUDA_TRY(cudaMemcpy(&perr, m->pos_err, sizeof(perr), cudaMemcpyDeviceToHost));
    if (perr) return fail(IAM_ERR_ARG, "a decode step found its position at or past max_ctx (clamped to the last slot)");
    return IAM_OK;
}

int iam_model_selected_rows(iam_model_t m, long long* total) {
    if (!m || !total) return fail(IAM_ERR_ARG, "iam_model_selected_rows: null argument");
    std::vector<int> h((size_t)m->cfg.n_layers * NMAT);
    IAM_CUDA_TRY(cudaMemcpy(h.data(), m->sel, h.size() * sizeof(int), cudaMemcpyDeviceToHost));
    long long t = 0;
    for (size_t i = 0; i < h.size(); ++i) {
        // column-parallel matrices select the same rows on every rank: count them once
        if (m->tp_world > 1 && m->tp_rank != 0 && column_parallel((int)(i % NMAT))) continue;
        t += h[i];
    }
    if (m->tp_world > 1) {  // row-parallel selections are per rank: sum over the group
        IAM_CUDA_TRY(cudaMemcpy(m->tp_tmp, &t, sizeof(t), cudaMemcpyHostToDevice));
        int rc = nccl_done(m, ncclAllReduce(m->tp_tmp, m->tp_tmp, 1, ncclInt64, ncclSum, m->comm, 0), "selected rows");
        if (rc) return rc;
        IAM_CUDA_TRY(cudaMemcpy(&t, m->tp_tmp, sizeof(t), cudaMemcpyDeviceToHost));
    }
    *total = t;
    return IAM_OK;
}

// Algorithmic bytes of the last step (bucketMul selected weights, stats, x, probes, outputs,
// attention K/V reads, LM head) for the roofline accounting of a decode step.
int iam_model_step_bytes(iam_model_t m, int context, long long* bytes) {
    if (!m || !bytes) return fail(IAM_ERR_ARG, "iam_model_step_bytes: null argument");
    const iam_model_config& c = m->cfg;
    std::vector<int> h((size_t)c.n_layers * NMAT);
    IAM_CUDA_TRY(cudaMemcpy(h.data(), m->sel, h.size() * sizeof(int), cudaMemcpyDeviceToHost));
    long long t = 0;
    for (int l = 0; l < c.n_layers; ++l)
        for (int i = 0; i < NMAT; ++i) {
            const Matrix& mt = m->layers[l].m[i];  // this rank's shard
            const long long n_in = mt.in_end - mt.in_begin;
            t += 2LL * h[(size_t)l * NMAT + i] * mt.cols + 2 * 16 * n_in + 4LL * n_in +
                 2LL * std::min(mt.in_dim, IAM_PROBES_COUNT) + 4LL * 16 * mt.cols;
        }
    t += 2LL * c.n_layers * m->n_kv_local * (long long)context * c.head_dim * 2;  // K and V fp16
    t += 2LL * m->vocab_local * c.dim;                                          // LM head rows
    *bytes = t;
    return IAM_OK;
}

}  // extern "C"

// ------------------------------------------------------------------ block-level entry points

namespace {
int block_entry_check(iam_model_s* m, int layer, const void* in, const void* out, float effort, int pos) {
    if (!m || !in || !out) return fail(IAM_ERR_ARG, "layer entry: null argument");
    if (layer < 0 || layer >= m->cfg.n_layers) return fail(IAM_ERR_ARG, "layer entry: layer out of range");
    if (!effort_ok(effort)) return fail(IAM_ERR_ARG, "layer entry: effort must be in (0, 1]");
    if (pos < 0 || pos >= m->cfg.max_ctx) return fail(IAM_ERR_ARG, "layer entry: pos outside [0, max_ctx)");
    if (m->tp_world > 1) return fail(IAM_ERR_UNSUPPORTED, "layer entry: one GPU only (call iam_model_forward under TP)");
    IAM_CUDA_TRY(cudaSetDevice(m->device));
    return IAM_OK;
}
}  // namespace

extern "C" {

int iam_layer_forward(iam_model_t m, int layer, const float* x_dev, int pos, float effort, float* out_dev,
                      void* stream) {
    int rc = block_entry_check(m, layer, x_dev, out_dev, effort, pos);
    if (rc || (rc = build_plans(m, effort))) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    IAM_CUDA_TRY(launch_ex(set_int_kernel, dim3(1), dim3(1), 0, s, false, m->pos, pos));
    IAM_CUDA_TRY(cudaMemcpyAsync(m->x, x_dev, (size_t)m->cfg.dim * 4, cudaMemcpyDeviceToDevice, s));
    if ((rc = enqueue_layer(m, layer, false, s, nullptr))) return rc;
    IAM_CUDA_TRY(cudaMemcpyAsync(out_dev, m->x, (size_t)m->cfg.dim * 4, cudaMemcpyDeviceToDevice, s));
    m->host_pos = pos;
    return IAM_OK;
}

int iam_attention_forward(iam_model_t m, int layer, const float* h_dev, int pos, float effort, float* out_dev,
                          void* stream) {
    int rc = block_entry_check(m, layer, h_dev, out_dev, effort, pos);
    if (rc || (rc = build_plans(m, effort))) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    const iam_model_config& c = m->cfg;
    IAM_CUDA_TRY(launch_ex(set_int_kernel, dim3(1), dim3(1), 0, s, false, m->pos, pos));
    if ((rc = launch_plain_plan(m, layer, 0, h_dev, nullptr, s))) return rc;
    if ((rc = launch_attention(attn_params(m, layer), c.n_heads / c.n_kv_heads, s, false))) return rc;
    if ((rc = launch_plain_plan(m, layer, 1, m->att, out_dev, s))) return rc;
    m->host_pos = pos;
    return IAM_OK;
}

int iam_feedforward_forward(iam_model_t m, int layer, const float* h_dev, float effort, float* out_dev, void* stream) {
    int rc = block_entry_check(m, layer, h_dev, out_dev, effort, 0);
    if (rc || (rc = build_plans(m, effort))) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    if ((rc = launch_plain_plan(m, layer, 2, h_dev, nullptr, s))) return rc;
    return launch_plain_plan(m, layer, 3, nullptr, out_dev, s);
}

}  // extern "C"
