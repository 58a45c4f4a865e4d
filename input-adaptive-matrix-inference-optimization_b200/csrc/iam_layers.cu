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
#include <algorithm>
#include <cfloat>

#include "iam_bucketmul.cuh"
#include "iam_layers.h"
#include "iam_tp_push.cuh"

namespace iam {

// ------------------------------------------------------------------ embedding

// x = float(embed[token]); token from `token_arg` or, when `token_key` is given, from the
// previous step's argmax key.  Also clears `argmax_key` for this step's LM head.
__global__ void embed_kernel(const uint16_t* __restrict__ embed, int dim, int token_arg,
                             const unsigned long long* token_key, const int* token_dev, float* __restrict__ x,
                             unsigned long long* argmax_key, int* token_used) {
    pdl_trigger();
    pdl_wait();
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
__global__ void clear_key_kernel(unsigned long long* key) {
    pdl_trigger();
    pdl_wait();
    *key = 0ull;
}

// ------------------------------------------------------------------ attention

// RoPE of one head (rotate-half, aux.cl:243-247) with separately rounded products.
IAM_DEV float rope_at(const float* m, const float* cs, int d, int half) {
    const int f = d % half;
    const float c = cs[2 * f], s = cs[2 * f + 1];
    if (d < half) return __fsub_rn(__fmul_rn(m[d], c), __fmul_rn(m[d + half], s));
    return __fadd_rn(__fmul_rn(m[d], c), __fmul_rn(m[d - half], s));
}

// Loads VD consecutive fp16 values (VD = head_dim / 32 per lane) as floats.
template <int VD>
IAM_DEV void load_half_vec(const uint16_t* p, float* o) {
    if constexpr (VD == 4) {
        const uint2 v = *reinterpret_cast<const uint2*>(p);
        o[0] = h2f(v.x & 0xffffu);
        o[1] = h2f(v.x >> 16);
        o[2] = h2f(v.y & 0xffffu);
        o[3] = h2f(v.y >> 16);
    } else if constexpr (VD == 2) {
        const uint32_t v = *reinterpret_cast<const uint32_t*>(p);
        o[0] = h2f(v & 0xffffu);
        o[1] = h2f(v >> 16);
    } else {
#pragma unroll
        for (int e = 0; e < VD; ++e) o[e] = h2f(p[e]);
    }
}

// Loads 2*NV halves (16-byte aligned when NV >= 4) as floats.
template <int VD>
IAM_DEV void load_halves(const uint16_t* p, float* o) {
    if constexpr (VD % 8 == 0) {
#pragma unroll
        for (int c = 0; c < VD; c += 8) {
            const uint4 v = *reinterpret_cast<const uint4*>(p + c);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                o[c + 2 * e] = h2f(w[e] & 0xffffu);
                o[c + 2 * e + 1] = h2f(w[e] >> 16);
            }
        }
    } else {
        load_half_vec<VD>(p, o);
    }
}

// 16-byte global -> shared copy that does not wait (cp.async; completed by cp_async_wait_all).
IAM_DEV void cp_async16(void* dst_smem, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst_smem)),
                 "l"(__cvta_generic_to_global(src))
                 : "memory");
}
IAM_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// mma.sync m16n8k16, f16 x f16 -> f32 (fragments as the PTX ISA lays them out: A rows
// g = lane / 4 and g + 8, columns 2 * (lane % 4) + {0, 1} and + 8; B rows 2 * (lane % 4) + {0, 1}
// and + 8, column g; C rows g and g + 8, columns 2 * (lane % 4) + {0, 1}).
IAM_DEV void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
IAM_DEV void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
IAM_DEV void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
IAM_DEV uint32_t pack_h2(float a, float b) {  // a in the low half, both rounded to fp16
    return (uint32_t)__half_as_ushort(__float2half_rn(a)) | ((uint32_t)__half_as_ushort(__float2half_rn(b)) << 16);
}
// x = hi + lo with hi = fp16(x): the low part of a two-term fp16 split (exact in fp32)
IAM_DEV float split_lo(float x) { return __fsub_rn(x, __half2float(__float2half_rn(x))); }

// Long-context layout of one chunk [t0, t1) on the tensor cores (GQ <= 4 query heads per KV
// head, head_dim 64 or 128): warp w takes the 32-token groups t0 + 32w, t0 + 32(w + 8), ...
// For a group, the K rows go to the warp's shared tile (cp.async, 16-byte pieces XOR-swizzled
// by the row's low 3 bits so that ldmatrix reads are conflict-free) and the scores are
// S[32 tokens][8] = K . Q^T with the queries split in two fp16 terms (columns 0..3 the high
// parts, 4..7 the low parts of the GQ heads, summed after the product): the fp16 K values times
// the two-term queries, accumulated in fp32, equal the fp32 dot product to about 2^-22.  The
// group's max and sum per head are warp reductions, the probabilities are split the same way
// (A rows 0..3 high, 4..7 low), the V rows replace the K rows in the tile, and O += P . V on
// the tensor cores, the two halves summed at the end.  The running max, sum and p.V per head
// land in cm/cl/co slot `warp` (slots 0..7).  The new token pos is patched into the tile from
// knew/vnew (its fp16-rounded K/V), never read from the cache row this launch writes.
template <int GQ, int VD>
IAM_DEV void attn_mma_chunk(const float* __restrict__ qr, const float* __restrict__ knew,
                            const float* __restrict__ vnew, const uint16_t* __restrict__ kc,
                            const uint16_t* __restrict__ vc, uint16_t* tiles, int t0, int t1, int pos, float* cm,
                            float* cl, float* co) {
    constexpr int HD = 16 * VD;
    constexpr int KS = HD / 16;  // k-steps of the scores
    constexpr int NT = HD / 8;   // n-tiles of p.V
    constexpr int CPR = HD / 8;  // 16-byte pieces per row
    constexpr int NW = kAttnThreads / 32;
    static_assert(GQ <= 4 && (HD == 64 || HD == 128), "tensor-core attention: GQ <= 4, head_dim 64 or 128");
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, tig = lane & 3;
    char* tile = reinterpret_cast<char*>(tiles + (size_t)warp * 32 * HD);  // 32 rows of HD fp16
    const uint32_t tile_s = (uint32_t)__cvta_generic_to_shared(tile);
    __shared__ __align__(16) float ps_all[kAttnThreads / 32][32 * 4];
    float* ps = ps_all[warp];  // the group's probabilities [token][4 heads]
    auto off = [](int r, int c) { return r * (HD * 2) + ((c ^ (r & 7)) << 4); };
    auto load_rows = [&](const uint16_t* src, int base, int nv) {
#pragma unroll
        for (int i = 0; i < CPR; ++i) {
            const int f = i * 32 + lane, r = f / CPR, c = f % CPR;
            if (r < nv) cp_async16(tile + off(r, c), src + (size_t)(base + r) * HD + c * 8);
            else *reinterpret_cast<uint4*>(tile + off(r, c)) = make_uint4(0u, 0u, 0u, 0u);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        cp_async_wait_all();
        __syncwarp();
    };
    auto patch_row = [&](const float* vals, int r) {  // the new token's row, fp16 pairs
        for (int d = 2 * lane; d < HD; d += 64)
            *reinterpret_cast<uint32_t*>(tile + off(r, d >> 3) + (d & 7) * 2) = pack_h2(vals[d], vals[d + 1]);
        __syncwarp();
    };

    // Q^T fragments: column g is head g & 3, its high part (g < 4) or its low part
    uint32_t bq[KS][2];
    {
        const int j = g & 3;
        const bool lo = g >= 4;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            const int d0 = 16 * ks + 2 * tig;
            float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (j < GQ) {
                v[0] = qr[j * HD + d0];
                v[1] = qr[j * HD + d0 + 1];
                v[2] = qr[j * HD + d0 + 8];
                v[3] = qr[j * HD + d0 + 9];
            }
            if (lo)
#pragma unroll
                for (int e = 0; e < 4; ++e) v[e] = split_lo(v[e]);
            bq[ks][0] = pack_h2(v[0], v[1]);
            bq[ks][1] = pack_h2(v[2], v[3]);
        }
    }
    const float scale_div = sqrtf((float)HD);
    // this lane's two heads in the softmax: hp and hp + 1
    const int hp = 2 * (tig & 1);
    float mrun[2] = {-INFINITY, -INFINITY}, lrun[2] = {0.0f, 0.0f};
    float o[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[nt][e] = 0.0f;

    for (int base = t0 + warp * 32; base < t1; base += NW * 32) {
        const int nv = min(32, t1 - base);
        const bool has_pos = pos >= base && pos < base + nv;
        __syncwarp();  // the previous group's tile and probabilities are consumed
        load_rows(kc, base, nv);
        if (has_pos) patch_row(knew, pos - base);
        float sc[2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) sc[mt][e] = 0.0f;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                uint32_t a[4];
                ldsm_x4(a, tile_s + off(mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, 2 * ks + (lane >> 4)));
                mma_16816(sc[mt], a, bq[ks][0], bq[ks][1]);
            }
        }
        // high + low columns (lanes tig and tig ^ 2), scale, mask: token of sc[mt][e] is
        // 16 mt + g + 8 (e >> 1), head hp + (e & 1)
        float pr[2][4];  // [head][k]: tokens g, g + 8, 16 + g, 24 + g
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float full = sc[mt][e] + __shfl_xor_sync(0xffffffffu, sc[mt][e], 2);
                const int k = 2 * mt + (e >> 1), tok = 16 * mt + g + 8 * (e >> 1);
                pr[e & 1][k] = tok < nv ? __fdiv_rn(full, scale_div) : -INFINITY;
            }
        float rsc[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float mx = fmaxf(fmaxf(pr[h][0], pr[h][1]), fmaxf(pr[h][2], pr[h][3]));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float nm = fmaxf(mrun[h], mx);  // token 0 of the group is in range
            rsc[h] = expf(mrun[h] - nm);
            float sum = 0.0f;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                pr[h][k] = pr[h][k] == -INFINITY ? 0.0f : expf(pr[h][k] - nm);
                sum += pr[h][k];
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 4);
            sum += __shfl_xor_sync(0xffffffffu, sum, 8);
            sum += __shfl_xor_sync(0xffffffffu, sum, 16);
            lrun[h] = fmaf(lrun[h], rsc[h], sum);
            mrun[h] = nm;
        }
        if (tig < 2)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int tok = 16 * (k >> 1) + g + 8 * (k & 1);
                *reinterpret_cast<float2*>(ps + tok * 4 + hp) = make_float2(pr[0][k], pr[1][k]);
            }
        {   // rescale the O rows: row g holds head g & 3 (its high or low part)
            const int src = (g & 3) >> 1;  // a lane that owns head g & 3 in the softmax
            const float r0 = __shfl_sync(0xffffffffu, rsc[0], src), r1 = __shfl_sync(0xffffffffu, rsc[1], src);
            const float rr = (g & 1) ? r1 : r0;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                o[nt][0] *= rr;
                o[nt][1] *= rr;
            }
        }
        load_rows(vc, base, nv);  // the K fragments are consumed: V rows into the same tile
        if (has_pos) patch_row(vnew, pos - base);
        // A = P: row g is head g & 3, high part (g < 4) or low part; rows 8..15 zero
        uint32_t ap[2][4];
        {
            const int j = g & 3;
            const bool lo = g >= 4;
#pragma unroll
            for (int kt = 0; kt < 2; ++kt) {
                const int ta = 16 * kt + 2 * tig, tb = ta + 8;
                float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                if (j < GQ) {
                    v[0] = ps[ta * 4 + j];
                    v[1] = ps[(ta + 1) * 4 + j];
                    v[2] = ps[tb * 4 + j];
                    v[3] = ps[(tb + 1) * 4 + j];
                }
                if (lo)
#pragma unroll
                    for (int e = 0; e < 4; ++e) v[e] = split_lo(v[e]);
                ap[kt][0] = pack_h2(v[0], v[1]);
                ap[kt][1] = 0u;
                ap[kt][2] = pack_h2(v[2], v[3]);
                ap[kt][3] = 0u;
            }
        }
#pragma unroll
        for (int kt = 0; kt < 2; ++kt)
#pragma unroll
            for (int n2 = 0; n2 < NT / 2; ++n2) {
                uint32_t bv[4];
                ldsm_x4_t(bv, tile_s + off(16 * kt + (lane & 7) + ((lane >> 3) & 1) * 8, 2 * n2 + (lane >> 4)));
                mma_16816(o[2 * n2], ap[kt], bv[0], bv[1]);
                mma_16816(o[2 * n2 + 1], ap[kt], bv[2], bv[3]);
            }
    }
    // high + low rows (lanes g and g + 4 = lane ^ 16); lanes g < GQ hold head g
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const float v = o[nt][e] + __shfl_xor_sync(0xffffffffu, o[nt][e], 16);
            if (g < GQ) co[(warp * GQ + g) * HD + 8 * nt + 2 * tig + e] = v;
        }
    if (g == 0 && tig < 2)
#pragma unroll
        for (int h = 0; h < 2; ++h)
            if (hp + h < GQ) {
                cm[warp * GQ + hp + h] = mrun[h];
                cl[warp * GQ + hp + h] = lrun[h];
            }
}

// grid = n_kv_heads * n_split, block = kAttnThreads (16 half-warps).  Single pass over the
// context (flash-decoding): the tokens [0, pos] are cut into `active` chunks of at least
// p.min_chunk tokens (n_split follows from the model's KV heads, so the chunks of a context do
// not depend on the tensor-parallel degree); CTA (kvh, s < active) runs chunk s for the GQ
// query heads of KV head kvh.  Two layouts, chosen from the context length on the device (one
// captured step serves every position):
//   * the tensor-core layout (attn_mma_chunk) for contexts of at most lane_short_max tokens,
//     in one chunk per KV head, and of at least lane_min_ctx tokens;
//   * the half-warp layout in between: each half-warp takes kAttnTU tokens at a time (K and V
//     loads issued together, 16 lanes x VD dimensions), reduces the GQ dot products over its
//     16 lanes, and keeps an online softmax (running max, sum and p.V per head) in registers.
// The warps' or half-warps' states are combined in shared memory in slot order; with more than
// one chunk the last CTA of the KV head combines the chunks in chunk order.  The new token's
// K/V (RoPE'd, rounded through fp16) are appended by the CTA whose chunk holds pos and used
// from shared memory for that token.
template <int GQ, int VD>
__global__ void __launch_bounds__(kAttnThreads, 2) attention_kernel(AttnParams p) {
    extern __shared__ __align__(16) float sm[];
    constexpr int HD = 16 * VD;
    constexpr int NH = kAttnThreads / 16;  // half-warps
    constexpr int TU = kAttnTU;
    const int half = HD / 2;
    pdl_wait();
    const int kvh = blockIdx.x / p.n_split, s = blockIdx.x % p.n_split;
    const int tid = threadIdx.x, hw = tid >> 4, hl = tid & 15;
    int pos = *p.pos_dev;
    if (pos >= p.max_ctx) {  // a step past the cache (the host refuses these): flagged, clamped
        if (p.pos_err && blockIdx.x == 0 && tid == 0) *p.pos_err = 1;
        pos = p.max_ctx - 1;
    }
    const int n_tok = pos + 1;
    // the layout by context length: the tensor-core one for a short context (in one chunk per
    // KV head: no combine across CTAs) and for a long one, the half-warp one in between
    const bool tc_layout = n_tok <= p.lane_short_max || n_tok >= p.lane_min_ctx;
    int chunk = (n_tok + p.n_split - 1) / p.n_split;
    if (chunk < p.min_chunk) chunk = p.min_chunk;
    if (tc_layout && n_tok <= p.lane_short_max) chunk = n_tok;
    const int active = (n_tok + chunk - 1) / chunk;
    if (s >= active) return;  // takes no part in the combine
    const int t0 = s * chunk, t1 = min(t0 + chunk, n_tok);

    float* qr = sm;                 // [GQ][HD] roped queries
    float* knew = qr + GQ * HD;     // [HD] roped k at pos, rounded through fp16
    float* vnew = knew + HD;        // [HD] v at pos, rounded through fp16
    float* cm = vnew + HD;          // [NH][GQ] half-warp running max
    float* cl = cm + NH * GQ;       // [NH][GQ] half-warp running sum
    float* wgt = cl + NH * GQ;      // [GQ][n_split] chunk weights (combine)
    float* co = wgt + ((GQ * p.n_split + 3) & ~3);  // [NH][GQ][HD] half-warp p.V, 16-byte aligned
    // [8 warps][32][HD] fp16 K, then V, rows of the long-context layout; co and vt together
    // are the staging area of the chunk combine
    uint16_t* vt = reinterpret_cast<uint16_t*>(co + NH * GQ * HD);
    const int nslots = tc_layout ? kAttnThreads / 32 : NH;  // filled cm/cl/co slots
    const float* cs = p.rope + (size_t)pos * HD;

    for (int e = tid; e < GQ * HD; e += kAttnThreads) {
        const int j = e / HD, d = e % HD;
        qr[e] = rope_at(p.q + (size_t)(kvh * GQ + j) * HD, cs, d, half);
    }
    for (int d = tid; d < HD; d += kAttnThreads) {
        knew[d] = __half2float(__float2half_rn(rope_at(p.k + (size_t)kvh * HD, cs, d, half)));
        vnew[d] = __half2float(__float2half_rn(p.v[(size_t)kvh * HD + d]));
    }
    uint16_t* kc = p.k_cache + (size_t)kvh * p.max_ctx * HD;
    uint16_t* vc = p.v_cache + (size_t)kvh * p.max_ctx * HD;
    __syncthreads();
    if (pos >= t0 && pos < t1) {  // the CTA whose chunk holds pos appends the new k/v
        for (int d = tid; d < HD; d += kAttnThreads) {
            kc[(size_t)pos * HD + d] = __half_as_ushort(__float2half_rn(knew[d]));
            vc[(size_t)pos * HD + d] = __half_as_ushort(__float2half_rn(vnew[d]));
        }
    }
    if (tc_layout) {  // (the host enables the layout only for the shapes it takes)
        if constexpr (GQ <= 4 && (VD == 4 || VD == 8))
            attn_mma_chunk<GQ, VD>(qr, knew, vnew, kc, vc, vt, t0, t1, pos, cm, cl, co);
    } else {
    float qv[GQ][VD];
#pragma unroll
    for (int j = 0; j < GQ; ++j)
#pragma unroll
        for (int e = 0; e < VD; ++e) qv[j][e] = qr[j * HD + hl * VD + e];
    const float scale_div = sqrtf((float)HD);

    float m[GQ], l[GQ], o[GQ][VD];
#pragma unroll
    for (int j = 0; j < GQ; ++j) {
        m[j] = -INFINITY;
        l[j] = 0.0f;
#pragma unroll
        for (int e = 0; e < VD; ++e) o[j][e] = 0.0f;
    }
    // warp-uniform trip count (the dot-product shuffles use the full warp); each half-warp
    // takes TU tokens of its warp's group of 2*TU, masking those past the chunk.  The K/V of
    // the next group are loaded before the current group is scored (software pipeline).
    const int warp = tid >> 5, hwin = (tid >> 4) & 1;  // (in the half-warp path)
    constexpr int NWT = kAttnThreads / 32;
    // K/V travel as raw fp16 words (VD/2 per token) and are widened at use
    constexpr int VW = VD / 2;
    auto load_group = [&](int wb, uint32_t (&kw)[TU][VW], uint32_t (&vw)[TU][VW]) {
        const int tb = wb + hwin * TU;
#pragma unroll
        for (int u = 0; u < TU; ++u) {
            const int t = tb + u;
            if (t < t1 && t != pos) {
                const uint32_t* kp = reinterpret_cast<const uint32_t*>(kc + (size_t)t * HD + hl * VD);
                const uint32_t* vp = reinterpret_cast<const uint32_t*>(vc + (size_t)t * HD + hl * VD);
                if constexpr (VW % 4 == 0) {
#pragma unroll
                    for (int c = 0; c < VW; c += 4) {
                        const uint4 a = *reinterpret_cast<const uint4*>(kp + c);
                        const uint4 b = *reinterpret_cast<const uint4*>(vp + c);
                        kw[u][c] = a.x; kw[u][c + 1] = a.y; kw[u][c + 2] = a.z; kw[u][c + 3] = a.w;
                        vw[u][c] = b.x; vw[u][c + 1] = b.y; vw[u][c + 2] = b.z; vw[u][c + 3] = b.w;
                    }
                } else {
#pragma unroll
                    for (int c = 0; c < VW; ++c) {
                        kw[u][c] = kp[c];
                        vw[u][c] = vp[c];
                    }
                }
            } else {  // the new token (its fp16-rounded k/v from shared memory) or past the chunk
#pragma unroll
                for (int c = 0; c < VW; ++c) {
                    const int d = hl * VD + 2 * c;
                    kw[u][c] = t < t1 ? (uint32_t)__half_as_ushort(__float2half_rn(knew[d])) |
                                            ((uint32_t)__half_as_ushort(__float2half_rn(knew[d + 1])) << 16)
                                      : 0u;
                    vw[u][c] = t < t1 ? (uint32_t)__half_as_ushort(__float2half_rn(vnew[d])) |
                                            ((uint32_t)__half_as_ushort(__float2half_rn(vnew[d + 1])) << 16)
                                      : 0u;
                }
            }
        }
    };
    auto half_at = [](const uint32_t (&w)[VW], int e) { return h2f((e & 1) ? (w[e >> 1] >> 16) : (w[e >> 1] & 0xffffu)); };
    uint32_t kw[TU][VW], vw[TU][VW];
    int wb = t0 + warp * 2 * TU;
    if (wb < t1) load_group(wb, kw, vw);
    for (; wb < t1; wb += NWT * 2 * TU) {
        const int tb = wb + hwin * TU;
        uint32_t kn[TU][VW], vn[TU][VW];
        if (wb + NWT * 2 * TU < t1) load_group(wb + NWT * 2 * TU, kn, vn);
        float sc[TU][GQ];
#pragma unroll
        for (int u = 0; u < TU; ++u)
#pragma unroll
            for (int j = 0; j < GQ; ++j) {
                float d = 0.0f;
#pragma unroll
                for (int e = 0; e < VD; ++e) d = fmaf(qv[j][e], half_at(kw[u], e), d);
#pragma unroll
                for (int off = 8; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);  // 16-lane groups
                sc[u][j] = (tb + u < t1) ? __fdiv_rn(d, scale_div) : -INFINITY;
            }
#pragma unroll
        for (int j = 0; j < GQ; ++j) {
            float mx = m[j];
#pragma unroll
            for (int u = 0; u < TU; ++u) mx = fmaxf(mx, sc[u][j]);
            if (mx == -INFINITY) continue;  // no token of this group in range yet
            const float r = expf(m[j] - mx);
            l[j] *= r;
#pragma unroll
            for (int e = 0; e < VD; ++e) o[j][e] *= r;
#pragma unroll
            for (int u = 0; u < TU; ++u) {
                const float pu = expf(sc[u][j] - mx);
                l[j] += pu;
#pragma unroll
                for (int e = 0; e < VD; ++e) o[j][e] = fmaf(pu, half_at(vw[u], e), o[j][e]);
            }
            m[j] = mx;
        }
#pragma unroll
        for (int u = 0; u < TU; ++u)
#pragma unroll
            for (int c = 0; c < VW; ++c) {
                kw[u][c] = kn[u][c];
                vw[u][c] = vn[u][c];
            }
    }
#pragma unroll
    for (int j = 0; j < GQ; ++j) {
        if (hl == 0) {
            cm[hw * GQ + j] = m[j];
            cl[hw * GQ + j] = l[j];
        }
#pragma unroll
        for (int e = 0; e < VD; ++e) co[(hw * GQ + j) * HD + hl * VD + e] = o[j][e];
    }
    }
    __syncthreads();
    // this chunk: M = max over the slots, L and O rescaled to M (fixed slot order); the slot
    // weights exp(m_h - M) are computed once per query head and kept in cm
    __shared__ float sM[8], sL[8];
    if (tid < GQ) {
        const int j = tid;
        float M = -INFINITY;
        for (int h = 0; h < nslots; ++h) M = fmaxf(M, cm[h * GQ + j]);
        float L = 0.0f;
        for (int h = 0; h < nslots; ++h) {
            const float mh = cm[h * GQ + j];
            const float w = mh == -INFINITY ? 0.0f : expf(mh - M);
            cm[h * GQ + j] = w;
            L = fmaf(w, cl[h * GQ + j], L);
        }
        sM[j] = M;
        sL[j] = L;
    }
    __syncthreads();
    float* stat = p.part + ((size_t)(kvh * p.n_split + s) * GQ) * (HD + 2);
    const unsigned push_epoch = p.tp_push ? tp_push_epoch(p.tp, kTpPushHeads) : 0u;
    for (int idx = tid; idx < GQ * HD; idx += kAttnThreads) {
        const int j = idx / HD, d = idx % HD;
        const float M = sM[j], L = sL[j];
        float O = 0.0f;
        for (int h = 0; h < nslots; ++h) O = fmaf(cm[h * GQ + j], co[(h * GQ + j) * HD + d], O);
        if (active == 1) {
            const int gi = (kvh * GQ + j) * HD + d;
            p.out[gi] = __fdiv_rn(O, L);
            if (p.tp_push && p.push_begin + gi < p.push_limit)
                tp_push_send(p.tp, kTpPushHeads, (size_t)(p.push_begin + gi), __fdiv_rn(O, L), push_epoch);
        } else {
            if (d == 0) {
                stat[j * (HD + 2)] = M;
                stat[j * (HD + 2) + 1] = L;
            }
            stat[j * (HD + 2) + 2 + d] = O;
        }
    }
    pdl_trigger();
    if (active == 1) return;

    // last active CTA of this KV head combines the chunks in chunk order
    __threadfence();
    __syncthreads();
    __shared__ int last;
    if (tid == 0) last = (atomicAdd(p.ctr + kvh, 1) == active - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    const float* base = p.part + (size_t)kvh * p.n_split * GQ * (HD + 2);
    const int lane = tid & 31, warp = tid >> 5;
    constexpr int NWA = kAttnThreads / 32;
    // every chunk's (M, L, O) into shared memory at once (co and vt are free now), when they fit
    constexpr int PER = GQ * (HD + 2);  // floats per chunk
    const bool staged = (PER % 4 == 0) && ((reinterpret_cast<uintptr_t>(base) & 15u) == 0) &&
                        (size_t)active * PER <= (size_t)NH * GQ * HD + (size_t)(kAttnThreads / 32) * 32 * HD / 2;
    if (staged) {
        for (int f = tid; f < active * PER / 4; f += kAttnThreads) cp_async16(co + 4 * f, base + 4 * f);
        asm volatile("cp.async.commit_group;" ::: "memory");
        cp_async_wait_all();
        __syncthreads();
    }
    // (two copies of the loops, so that the staged one never touches global memory)
    auto combine = [&](auto part_at) {
        for (int j = warp; j < GQ; j += NWA) {
            float M = -INFINITY;
            for (int r = lane; r < active; r += 32) M = fmaxf(M, part_at(r * PER + j * (HD + 2)));
#pragma unroll
            for (int o2 = 16; o2 > 0; o2 >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o2));
            float L = 0.0f;
            for (int r = lane; r < active; r += 32) {
                const float w = expf(part_at(r * PER + j * (HD + 2)) - M);
                wgt[j * p.n_split + r] = w;
                L = fmaf(w, part_at(r * PER + j * (HD + 2) + 1), L);
            }
#pragma unroll
            for (int o2 = 16; o2 > 0; o2 >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o2);
            for (int r = lane; r < active; r += 32) wgt[j * p.n_split + r] = __fdiv_rn(wgt[j * p.n_split + r], L);
        }
        __syncthreads();
        for (int e = tid; e < GQ * HD; e += kAttnThreads) {
            const int j = e / HD, d = e % HD;
            float O = 0.0f;
#pragma unroll 8
            for (int r = 0; r < active; ++r) O = fmaf(wgt[j * p.n_split + r], part_at(r * PER + j * (HD + 2) + 2 + d), O);
            const int gi = (kvh * GQ + j) * HD + d;
            p.out[gi] = O;
            if (p.tp_push && p.push_begin + gi < p.push_limit)
                tp_push_send(p.tp, kTpPushHeads, (size_t)(p.push_begin + gi), O, push_epoch);
        }
    };
    if (staged) combine([&](int i) { return co[i]; });
    else combine([&](int i) { return __ldcg(base + i); });
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
// over the grid, 8 x 16 B of the row per lane in flight; also folds the greedy argmax into
// *argmax_key with atomicMax.
__global__ void __launch_bounds__(kHeadThreads) lm_head_kernel(LMHeadParams p) {
    extern __shared__ __align__(16) float xf[];
    __shared__ float red[256];
    __shared__ unsigned long long wbest[kHeadThreads / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NWH = kHeadThreads / 32;
    constexpr int KB = 8;  // 16-byte loads per lane in flight
    const int first = blockIdx.x * NWH + warp;
    // the first row of this warp starts on its way to L2 before the dependency wait
    if (first < p.rows && (p.dim % 8) == 0 && ((reinterpret_cast<uintptr_t>(p.W) & 15u) == 0) && lane == 0)
        prefetch_l2(p.W + (size_t)first * p.dim, (uint32_t)p.dim * 2u);
    pdl_trigger();
    pdl_wait();
    const float scale = block_rms_scale<kHeadThreads>(p.x, p.dim, p.eps, red);
    for (int i = tid; i < p.dim; i += kHeadThreads) xf[i] = __fmul_rn(__fmul_rn(p.x[i], scale), h2f(p.gain[i]));
    __syncthreads();
    unsigned long long best = 0ull;
    const int vec_ok = (p.dim % 256 == 0) && ((reinterpret_cast<uintptr_t>(p.W) & 15u) == 0);
    for (int r = first; r < p.rows; r += gridDim.x * NWH) {
        const uint16_t* w = p.W + (size_t)r * p.dim;
        float acc0 = 0.0f, acc1 = 0.0f;
        if (vec_ok) {
            for (int cb = 0; cb < p.dim; cb += 256 * KB) {
                uint4 v[KB];
#pragma unroll
                for (int k = 0; k < KB; ++k) {
                    const int c = cb + k * 256 + lane * 8;
                    v[k] = c < p.dim ? __ldcs(reinterpret_cast<const uint4*>(w + c)) : make_uint4(0u, 0u, 0u, 0u);
                }
#pragma unroll
                for (int k = 0; k < KB; ++k) {
                    const int c = cb + k * 256 + lane * 8;
                    if (c < p.dim) {
                        const uint32_t wd[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            acc0 = fmaf(h2f(wd[e] & 0xffffu), xf[c + 2 * e], acc0);
                            acc1 = fmaf(h2f(wd[e] >> 16), xf[c + 2 * e + 1], acc1);
                        }
                    }
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
            const unsigned long long k = argmax_key(v, p.row0 + r);
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

// pos += 1 after a generated step (saturating at max_ctx: "no room left"), and the chosen
// token appended to tokens_out[*count].
__global__ void advance_kernel(int* pos, const unsigned long long* key, int* tokens_out, int* count, int max_ctx) {
    pdl_trigger();
    pdl_wait();
    if (tokens_out) tokens_out[*count] = (int)(0xffffffffu - (unsigned)(*key & 0xffffffffull));
    if (count) *count += 1;
    *pos = min(*pos + 1, max_ctx);
}

// ------------------------------------------------------------------ host launchers

int launch_embed(const uint16_t* embed, int dim, int token, const unsigned long long* token_key,
                 const int* token_dev, float* x, unsigned long long* argmax_key, int* token_used, cudaStream_t s,
                 bool pdl) {
    IAM_CUDA_TRY(launch_ex(embed_kernel, dim3((dim + 1023) / 1024), dim3(1024), 0, s, pdl, embed, dim, token,
                           token_key, token_dev, x, argmax_key, token_used));
    if (argmax_key && token_key == argmax_key)
        IAM_CUDA_TRY(launch_ex(clear_key_kernel, dim3(1), dim3(1), 0, s, pdl, argmax_key));
    return IAM_OK;
}

size_t attention_smem(const AttnParams& p, int gq) {
    const size_t hd = p.head_dim, nh = kAttnThreads / 16;
    return sizeof(float) * ((size_t)gq * hd + 2 * hd + 2 * nh * gq + nh * gq * hd + (((size_t)gq * p.n_split + 3) & ~3)) +
           sizeof(uint16_t) * (kAttnThreads / 32) * 32 * hd;
}

template <int GQ, int VD>
int launch_attention_t(const AttnParams& p, size_t smem, cudaStream_t s, bool pdl) {
    auto kern = attention_kernel<GQ, VD>;
    if (smem > 48 * 1024) IAM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    IAM_CUDA_TRY(launch_ex(kern, dim3((unsigned)(p.n_kv_heads * p.n_split)), dim3(kAttnThreads), smem, s, pdl, p));
    return IAM_OK;
}

template <int GQ>
int launch_attention_g(const AttnParams& p, size_t smem, cudaStream_t s, bool pdl) {
    switch (p.head_dim) {
        case 64: return launch_attention_t<GQ, 4>(p, smem, s, pdl);
        case 128: return launch_attention_t<GQ, 8>(p, smem, s, pdl);
        case 256: return launch_attention_t<GQ, 16>(p, smem, s, pdl);
        default: return fail(IAM_ERR_UNSUPPORTED, "attention: head_dim must be 64, 128 or 256");
    }
}

int launch_attention(const AttnParams& p, int gq, cudaStream_t s, bool pdl) {
    const size_t smem = attention_smem(p, gq);
    switch (gq) {
        case 1: return launch_attention_g<1>(p, smem, s, pdl);
        case 2: return launch_attention_g<2>(p, smem, s, pdl);
        case 4: return launch_attention_g<4>(p, smem, s, pdl);
        case 8: return launch_attention_g<8>(p, smem, s, pdl);
        default: return fail(IAM_ERR_UNSUPPORTED, "attention: n_heads / n_kv_heads must be 1, 2, 4 or 8");
    }
}

int launch_lm_head(const LMHeadParams& p, int grid, cudaStream_t s, bool pdl) {
    const size_t smem = sizeof(float) * (size_t)p.dim;
    if (smem > 48 * 1024)
        IAM_CUDA_TRY(cudaFuncSetAttribute(lm_head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    IAM_CUDA_TRY(launch_ex(lm_head_kernel, dim3(grid), dim3(kHeadThreads), smem, s, pdl, p));
    return IAM_OK;
}

int launch_advance(int* pos, const unsigned long long* key, int* tokens_out, int* count, int max_ctx, cudaStream_t s,
                   bool pdl) {
    IAM_CUDA_TRY(launch_ex(advance_kernel, dim3(1), dim3(1), 0, s, pdl, pos, key, tokens_out, count, max_ctx));
    return IAM_OK;
}

}  // namespace iam
