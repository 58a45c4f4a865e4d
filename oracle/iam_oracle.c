/*
 * iam_oracle.c -- CPU restatement of the reference's bucketMul decode path.
 * TEST INFRASTRUCTURE ONLY (see iam_oracle.h for what is pinned and how).
 *
 * Built with -ffp-contract=off so that every a*b+c below rounds twice, as written.
 */
#include "iam_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ fp16 helpers */

/* Exact fp16 -> fp32 (same result as binary_loader.hpp:204-230 fp16_to_float). */
float ora_half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    float f;
    if (exp == 0) {
        /* zero or subnormal: man * 2^-24 */
        f = ldexpf((float)man, -24);
        return sign ? -f : f;
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp - 15u + 127u) << 23) | (man << 13);
    }
    memcpy(&f, &bits, 4);
    return f;
}

/* IEEE fp32 -> fp16, round to nearest even, overflow to inf, NaN kept quiet. */
uint16_t ora_float_to_half(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) { /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    }
    if (ax >= 0x477ff000u) { /* >= 65520: rounds to inf */
        return (uint16_t)(sign | 0x7c00u);
    }
    if (ax < 0x38800000u) { /* below the smallest normal half: subnormal or zero */
        if (ax < 0x33000000u) return (uint16_t)sign; /* < 2^-25: rounds to zero */
        uint32_t e = ax >> 23;
        uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126u - e; /* value = m * 2^(e-150); half sub unit = 2^-24 */
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1u);
        if (rem > halfway || (rem == halfway && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (ax >> 23) - 127u + 15u;
    uint32_t m = ax & 0x7fffffu;
    uint32_t q = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return (uint16_t)(sign | q);
}

/* ------------------------------------------------------------------ cutoff search */

int ora_probes_count(int in_dim) { return in_dim < ORA_PROBES_COUNT ? in_dim : ORA_PROBES_COUNT; }

/* bucket_mul.hpp:164 quantile = int((PROBES_COUNT-1)*(1-effort)) in double;
 * bucketMul.cl:81 effort' = PROBES_COUNT - quantile is the target "above" count. */
int ora_target_count(float effort, int probes_count) {
    int quantile = (int)((double)(probes_count - 1) * (1.0 - (double)effort));
    return probes_count - quantile;
}

static float ora_importance(float x, float s) {
    /* bucketMul.cl:110 / :378: CUTOFF_SCALE * fabs(v * probe) */
    float p = x * s;
    return ORA_CUTOFF_SCALE * fabsf(p);
}

/* bucketMul.cl:68-214 findCutoffBinarySearch, restated for one work-group:
 *   imp_i = 1e5*|x_i*probe_i| for i < probes_count; global min / max;
 *   bounds = [min, max], mid = (min+max)/2, minCount = probes_count, maxCount = 0;
 *   up to 20 times: count = #(imp > mid);
 *     count < target -> max = mid, maxCount = count, else min = mid, minCount = count;
 *     next mid = (min+max)/2;
 *     stop on count == target, max-min < 1e-5f or |maxCount-minCount| < 3,
 *     returning the mid that was just TESTED (:195-199);
 *   after 20 steps return the updated mid (:211-213). */
float ora_find_cutoff(const float* x, const uint16_t* probes, int probes_count, int target,
                      int* iters) {
    float* imp = (float*)malloc(sizeof(float) * (size_t)(probes_count > 0 ? probes_count : 1));
    float gmin = 1e30f, gmax = -1e30f;
    for (int i = 0; i < probes_count; ++i) {
        imp[i] = ora_importance(x[i], ora_half_to_float(probes[i]));
        gmin = fminf(gmin, imp[i]);
        gmax = fmaxf(gmax, imp[i]);
    }
    float lo = gmin, hi = gmax;
    float mid = (lo + hi) / 2.0f;
    int min_count = probes_count, max_count = 0;
    for (int it = 0; it < ORA_MAX_ITERS; ++it) {
        int count = 0;
        for (int i = 0; i < probes_count; ++i) count += imp[i] > mid ? 1 : 0;
        if (count < target) {
            hi = mid;
            max_count = count;
        } else {
            lo = mid;
            min_count = count;
        }
        float next = (lo + hi) / 2.0f;
        int dc = max_count - min_count;
        if (dc < 0) dc = -dc;
        if (count == target || (hi - lo) < 0.00001f || dc < 3) {
            if (iters) *iters = it + 1;
            free(imp);
            return mid;
        }
        mid = next;
    }
    if (iters) *iters = ORA_MAX_ITERS;
    free(imp);
    return mid;
}

/* ------------------------------------------------------------------ dispatch */

long ora_prepare_dispatch(const float* x, const uint16_t* stats, int stats_stride, long row0,
                          long expert_size, int in_dim, float cutoff, int32_t* rows_out) {
    long n = 0;
    for (long r = 0; r < expert_size; ++r) {
        long input = r / 16; /* bucketMul.cl:374 */
        if (input >= in_dim) continue;
        long row = row0 + r;
        float s = ora_half_to_float(stats[row * stats_stride + (stats_stride - 1)]);
        if (ora_importance(x[input], s) >= cutoff) rows_out[n++] = (int32_t)row; /* :380 */
    }
    return n;
}

/* ------------------------------------------------------------------ accumulation */

void ora_bucket_mul(const uint16_t* buckets, int cols, const float* x, long row0,
                    const int32_t* rows, long count, float* out, int nthreads) {
    memset(out, 0, sizeof(float) * 16u * (size_t)cols);
#ifdef _OPENMP
    if (nthreads < 1) nthreads = 1;
#pragma omp parallel for num_threads(nthreads) schedule(static)
#endif
    for (int c = 0; c < cols; ++c) {
        float acc[16];
        for (int s = 0; s < 16; ++s) acc[s] = 0.0f;
        for (long k = 0; k < count; ++k) {
            long row = rows[k];
            float xv = x[(row - row0) / 16];
            uint16_t w = buckets[row * (long)cols + c];
            acc[w & 15u] += xv * ora_half_to_float(w); /* bucketMul.cl:430-434 */
        }
        for (int s = 0; s < 16; ++s) out[c * 16 + s] = acc[s];
    }
    (void)nthreads;
}

long ora_bucketmul_full(const float* x, const uint16_t* stats, int stats_stride,
                        const uint16_t* probes, const uint16_t* buckets, int expert_no,
                        int in_dim, int bucket_cols, long expert_size, float effort, float* out,
                        int32_t* rows_scratch, float* cutoff_out, int nthreads) {
    int P = ora_probes_count(in_dim);
    int target = ora_target_count(effort, P);
    /* probes offset expNo*PROBES_COUNT (bucketMul.cl:103), rows offset expertSize*expNo
     * (bucketMul.cl:363). */
    float cutoff =
        ora_find_cutoff(x, probes + (long)expert_no * ORA_PROBES_COUNT, P, target, NULL);
    long row0 = (long)expert_no * expert_size;
    long n = ora_prepare_dispatch(x, stats, stats_stride, row0, expert_size, in_dim, cutoff,
                                  rows_scratch);
    ora_bucket_mul(buckets, bucket_cols, x, row0, rows_scratch, n, out, nthreads);
    if (cutoff_out) *cutoff_out = cutoff;
    return n;
}

void ora_dense_gemv(const uint16_t* W, int M, int N, const float* x, double* out) {
    for (int j = 0; j < M; ++j) {
        double acc = 0.0;
        for (int i = 0; i < N; ++i) acc += (double)ora_half_to_float(W[(long)j * N + i]) * x[i];
        out[j] = acc;
    }
}

/* ------------------------------------------------------------------ layer glue */

void ora_rmsnorm(const float* x, int n, float eps, const uint16_t* gain, float* out) {
    float sum = 0.0f;
    if (n >= 256 && n % 256 == 0) {
        /* rmsNorm32fast order: 256 threads each sum a contiguous run of n/256, then a
         * halving tree over the 256 partials (aux.cl:165-186). */
        float part[256];
        int e = n / 256;
        for (int t = 0; t < 256; ++t) {
            float s = 0.0f;
            for (int i = t * e; i < t * e + e; ++i) s += x[i] * x[i];
            part[t] = s;
        }
        for (int s = 128; s > 0; s >>= 1)
            for (int t = 0; t < s; ++t) part[t] += part[t + s];
        sum = part[0];
    } else {
        for (int i = 0; i < n; ++i) sum += x[i] * x[i];
    }
    float scale = 1.0f / sqrtf(sum / (float)n + eps); /* aux.cl:190 rsqrt */
    for (int i = 0; i < n; ++i) {
        float v = x[i] * scale;
        out[i] = gain ? ora_half_to_float(gain[i]) * v : v; /* mul16x32, aux.cl:434-440 */
    }
}

void ora_rope_table(int pos, int head_dim, double theta, float* cs) {
    /* attention.hpp:213-220 */
    for (int i = 0; i < head_dim / 2; ++i) {
        double exponent = (2.0 * i) / head_dim;
        float freq = (float)(1.0 / pow(theta, exponent));
        float angle = (float)pos * freq;
        cs[2 * i] = cosf(angle);
        cs[2 * i + 1] = sinf(angle);
    }
}

void ora_rope_apply(const float* in, int n_heads, int head_dim, const float* cs, float* out) {
    int half = head_dim / 2;
    for (int h = 0; h < n_heads; ++h) {
        const float* m = in + (long)h * head_dim;
        float* o = out + (long)h * head_dim;
        for (int d = 0; d < head_dim; ++d) {
            int f = d % half;
            float c = cs[2 * f], s = cs[2 * f + 1];
            if (d < half) {
                float a = m[d] * c, b = m[d + half] * s;
                o[d] = a - b; /* aux.cl:244 */
            } else {
                float a = m[d] * c, b = m[d - half] * s;
                o[d] = a + b; /* aux.cl:246 */
            }
        }
    }
}

void ora_silu_mul(const float* g, const float* u, int n, float* out) {
    for (int i = 0; i < n; ++i) out[i] = u[i] * g[i] / (1.0f + expf(-g[i])); /* matrix.cl:31 */
}

static float ora_tree_dot(const float* q, const uint16_t* k, int hd) {
    /* dotSetScore2 local halving tree over head_dim products (aux.cl:523-534) */
    float lp[1024];
    for (int d = 0; d < hd; ++d) lp[d] = q[d] * ora_half_to_float(k[d]);
    for (int s = hd / 2; s > 0; s >>= 1)
        for (int d = 0; d < s; ++d) lp[d] += lp[d + s];
    return lp[0];
}

void ora_attention(const ora_config* cfg, const float* q, const uint16_t* k_layer,
                   const uint16_t* v_layer, int n_tokens, float* out) {
    int hd = cfg->head_dim, group = cfg->n_heads / cfg->n_kv_heads;
    float* p = (float*)malloc(sizeof(float) * (size_t)n_tokens);
    float inv_scale = sqrtf((float)hd);
    for (int h = 0; h < cfg->n_heads; ++h) {
        int kvh = h / group; /* repeat4x32 GQA mapping, aux.cl:266-275 */
        const uint16_t* kb = k_layer + (long)kvh * cfg->max_ctx * hd;
        const uint16_t* vb = v_layer + (long)kvh * cfg->max_ctx * hd;
        float sum = 0.0f;
        for (int t = 0; t < n_tokens; ++t) {
            float score = ora_tree_dot(q + (long)h * hd, kb + (long)t * hd, hd) / inv_scale;
            p[t] = score;
        }
        for (int t = 0; t < n_tokens; ++t) sum += expf(p[t]); /* aux.cl:204-210 */
        for (int t = 0; t < n_tokens; ++t) p[t] = expf(p[t]) / sum; /* aux.cl:219-225 */
        for (int d = 0; d < hd; ++d) {
            float acc = 0.0f;
            for (int t = 0; t < n_tokens; ++t)
                acc += p[t] * ora_half_to_float(vb[(long)t * hd + d]); /* aux.cl:379-381 */
            out[(long)h * hd + d] = acc;
        }
    }
    free(p);
}

void ora_lm_head(const uint16_t* W, int rows, int cols, const float* x, float* logits,
                 int nthreads) {
#ifdef _OPENMP
    if (nthreads < 1) nthreads = 1;
#pragma omp parallel for num_threads(nthreads) schedule(static)
#endif
    for (int r = 0; r < rows; ++r) {
        float part[256];
        const uint16_t* w = W + (long)r * cols;
        for (int t = 0; t < 256; ++t) {
            float s = 0.0f;
            for (int i = t; i < cols; i += 256) s += ora_half_to_float(w[i]) * x[i];
            part[t] = s;
        }
        for (int s = 128; s > 0; s >>= 1)
            for (int t = 0; t < s; ++t) part[t] += part[t + s];
        logits[r] = part[0];
    }
    (void)nthreads;
}

long ora_model_scratch_floats(const ora_config* c) {
    long d = c->dim, q = (long)c->n_heads * c->head_dim, kv = (long)c->n_kv_heads * c->head_dim;
    long f = c->ffn_dim;
    return 4 * d + 3 * q + 2 * kv + 3 * f + 4 * (c->head_dim / 2 + 1);
}

/* effort < 0: every bucket row selected (the dense path's product, bucketMul.cl:392-497 over
 * the whole bucket matrix) instead of the cutoff search and dispatch. */
static long ora_bm(const ora_bm_weight* w, const float* x, float effort, float* out,
                   int32_t* rows, int nthreads) {
    if (effort < 0.0f) {
        long n = 16L * w->in_dim;
        for (long i = 0; i < n; ++i) rows[i] = (int32_t)i;
        ora_bucket_mul(w->buckets, w->out_dim / 16, x, 0, rows, n, out, nthreads);
        return n;
    }
    return ora_bucketmul_full(x, w->stats, w->stats_stride, w->probes, w->buckets, 0, w->in_dim,
                              w->out_dim / 16, 16L * w->in_dim, effort, out, rows, NULL,
                              nthreads);
}

static int model_forward(const ora_model* m, int token, int pos, float effort, float* logits,
                         long* sel_rows, int nthreads);

int ora_model_forward(const ora_model* m, int token, int pos, float effort, float* logits,
                      long* sel_rows, int nthreads) {
    return model_forward(m, token, pos, effort, logits, sel_rows, nthreads);
}

int ora_model_forward_dense(const ora_model* m, int token, int pos, float* logits, int nthreads) {
    return model_forward(m, token, pos, -1.0f, logits, NULL, nthreads);
}

static int model_forward(const ora_model* m, int token, int pos, float effort, float* logits,
                         long* sel_rows, int nthreads) {
    const ora_config* c = &m->cfg;
    long d = c->dim, qn = (long)c->n_heads * c->head_dim, kvn = (long)c->n_kv_heads * c->head_dim;
    long f = c->ffn_dim, hd = c->head_dim;
    float* buf = (float*)malloc(sizeof(float) * (size_t)ora_model_scratch_floats(c));
    long maxin = f > d ? f : d;
    int32_t* rows = (int32_t*)malloc(sizeof(int32_t) * (size_t)(16 * maxin));
    float *x = buf, *h = x + d, *x1 = h + d, *o = x1 + d;
    float *q = o + d, *qr = q + qn, *att = qr + qn;
    float *k = att + qn, *v = k + kvn;
    float *g = v + kvn, *u = g + f, *a = u + f;
    float* cs = a + f;
    long sel = 0;

    for (long i = 0; i < d; ++i) x[i] = ora_half_to_float(m->embed[(long)token * d + i]);
    ora_rope_table(pos, c->head_dim, c->rope_theta, cs);

    for (int l = 0; l < c->n_layers; ++l) {
        const ora_layer* L = &m->layers[l];
        ora_rmsnorm(x, (int)d, c->norm_eps, L->attn_norm, h);
        sel += ora_bm(&L->wq, h, effort, q, rows, nthreads);
        sel += ora_bm(&L->wk, h, effort, k, rows, nthreads);
        sel += ora_bm(&L->wv, h, effort, v, rows, nthreads);
        ora_rope_apply(q, c->n_heads, c->head_dim, cs, qr);
        ora_rope_apply(k, c->n_kv_heads, c->head_dim, cs, o); /* post-RoPE k, o as temp */
        long layer_off = (long)l * c->n_kv_heads * c->max_ctx * hd;
        for (int kh = 0; kh < c->n_kv_heads; ++kh) {
            long base = layer_off + ((long)kh * c->max_ctx + pos) * hd;
            for (long e = 0; e < hd; ++e) {
                m->k_cache[base + e] = ora_float_to_half(o[kh * hd + e]);
                m->v_cache[base + e] = ora_float_to_half(v[kh * hd + e]);
            }
        }
        ora_attention(c, qr, m->k_cache + layer_off, m->v_cache + layer_off, pos + 1, att);
        sel += ora_bm(&L->wo, att, effort, o, rows, nthreads);
        for (long i = 0; i < d; ++i) x1[i] = x[i] + o[i]; /* add32 */
        ora_rmsnorm(x1, (int)d, c->norm_eps, L->ffn_norm, h);
        sel += ora_bm(&L->w1, h, effort, g, rows, nthreads);
        sel += ora_bm(&L->w3, h, effort, u, rows, nthreads);
        ora_silu_mul(g, u, (int)f, a);
        sel += ora_bm(&L->w2, a, effort, o, rows, nthreads);
        for (long i = 0; i < d; ++i) x[i] = x1[i] + o[i];
    }
    ora_rmsnorm(x, (int)d, c->norm_eps, m->final_norm, h);
    ora_lm_head(m->lm_head, c->vocab, (int)d, h, logits, nthreads);
    int best = 0;
    for (int r = 1; r < c->vocab; ++r)
        if (logits[r] > logits[best]) best = r;
    if (sel_rows) *sel_rows += sel;
    free(rows);
    free(buf);
    return best;
}
