// iam_dense.cu -- the dense tensor-core path: Y[t][o] = sum_i W[o][i] * X[t][i] on tcgen05.
//
// The reference multiplies densely only in GEMV form (basicMul / basicMul2, matrix.cl:80-127:
// out[row] = sum_i v[i] * m[row][i] with fp16 m and fp32 v; matmul16x32, aux.cl:454-490, the
// LM head).  Over the tokens of a prompt the same products form a GEMM, run here on the 5th
// generation tensor cores:
//
//   * one CTA per (128 tokens) x (256 weight rows) tile [x K slice], 128 threads;
//   * warp 0 lane 0 streams K in 64-element stages with TMA (cp.async.bulk.tensor.2d, 128-byte
//     swizzle) into a ring of three 64 KB shared-memory stages: the activation tiles hi / lo
//     [128][64] (operand A) and the weight tile [256][64] (operand B); "full" mbarriers carry
//     the transaction bytes.  With the tokens as the MMA's M, one activation tile serves 256
//     weight rows: the activations every CTA re-reads from L2 are half the weight bytes (hi
//     and lo together equal them), where 128-row weight tiles made them twice the weight bytes;
//   * warp 1 lane 0 issues tcgen05.mma (kind::f16, M = 128, N = 256, K = 16, both operands
//     K-major from shared memory) into two fp32 accumulators in tensor memory (256 columns
//     each, all 512 columns of the SM): hi x W and lo x W, so the sum carries ~22 bits of every
//     fp32 activation and the small lo products never round against the large hi sum; a
//     tcgen05.commit per stage frees the stage ("empty" mbarrier) once its MMAs have read it;
//   * after the last commit all four warps read the accumulators back (tcgen05.ld 32x32b: warp
//     w owns lanes 32(w%4)..+31 = tokens, 16 output columns per load), add hi + lo (IEEE fp32)
//     and store 16 consecutive outputs of their token (+ residual), or a K-slice partial that a
//     second, ordered pass sums (deterministic split-K).
//
// Every wait on an mbarrier is bounded: after ~2 s the thread sets the error word and moves
// on, so a broken pipeline ends the kernel instead of hanging it.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "iam_common.cuh"
#include "iam_dense.h"

namespace iam {

namespace {

constexpr long long kDenseWaitCycles = 4000000000LL;  // ~2 s at the SM clock

// One pipeline stage: the activation tiles hi / lo [kDenseBT][kDenseBK] (operand A, 16 KB each)
// and the weight tile [kDenseBW][kDenseBK] (operand B, 32 KB), each 1024-byte aligned for the
// 128-byte swizzle.
struct Tile {
    static constexpr int kA = kDenseBT * kDenseBK * 2;  // one activation tile (hi or lo)
    static constexpr int kB = kDenseBW * kDenseBK * 2;  // weight tile
    static constexpr int kStage = 2 * kA + kB;          // 64 KB
    static constexpr int kStages = 3;
    // two fp32 accumulators of kDenseBW columns (outputs) x 128 lanes (tokens): the hi products
    // and the lo products -- the whole tensor memory of the SM
    static constexpr int kTmemCols = 2 * kDenseBW;
    static constexpr size_t kSmem = (size_t)kStages * kStage + 1024;  // + 1024-byte alignment slack
    static_assert(kA % 1024 == 0 && kB % 1024 == 0, "stage tiles must stay 1024-byte aligned");
    static_assert(kSmem <= 227 * 1024, "shared memory per CTA");
    static_assert(kTmemCols == 512, "tensor memory columns");
};

IAM_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

IAM_DEV void mbar_init(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}

IAM_DEV void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}

IAM_DEV bool mbar_try_wait(uint64_t* b, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return done != 0u;
}

// Waits for the phase of `parity` to complete; false (and the error word set) after ~2 s.
IAM_DEV bool mbar_wait(uint64_t* b, uint32_t parity, unsigned* err) {
    if (mbar_try_wait(b, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(b, parity)) {
        if (clock64() - t0 > kDenseWaitCycles) {
            if (err) atomicOr(err, 1u);
            return false;
        }
    }
    return true;
}

// 2-D tiled TMA load of box {kDenseBK, rows} at (inner c0, row c1); completes bytes on bar.
IAM_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

IAM_DEV void tmem_alloc(uint32_t* slot, uint32_t ncols) {  // whole warp
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
}
IAM_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
IAM_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
IAM_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
IAM_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrives once on bar when every tcgen05.mma this thread issued so far has completed.
IAM_DEV void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T; accumulate = 0 overwrites D.
IAM_DEV void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}

// 16 consecutive accumulator columns of this thread's lane; returns after the load completed
// (the registers pass through the wait so no use can be scheduled before it).
IAM_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])::"memory");
}

// Shared-memory matrix descriptor of a K-major tile written by TMA with the 128-byte swizzle:
// rows of 128 bytes, 8-row groups 1024 bytes apart (stride byte offset), leading byte offset
// unused (1), descriptor version 1, layout type 2 = SWIZZLE_128B.  The K step of 16 fp16 inside
// the 128-byte row advances the start address by 32 bytes (+2 in 16-byte units).
IAM_DEV uint64_t sw128_desc(const void* tile) {
    const uint32_t a = smem_u32(tile);
    return (uint64_t)((a & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor of kind::f16: D fp32 (bits 4-5 = 1), A and B fp16 (formats 0),
// both K-major, N >> 3 at bit 17, M >> 4 at bit 24.  M = 128 tokens, N = 256 weight rows.
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kDenseBW >> 3) << 17) | ((uint32_t)(kDenseBT >> 4) << 24);

struct GemmArgs {
    int m, n, kb_total, kb_per_split, has_lo;
    float* y;
    int ldy;
    const float* residual;
    int ldr;
    float* partial;  // split-K: [split][n][m]; null when the tile writes y directly
    unsigned* err;
    uint16_t* silu_hi;  // SiLU epilogue (see DenseProblem); null: plain store
    uint16_t* silu_lo;
    int ld_silu;
};

// 16 consecutive floats of one row: vector stores when all are in range and dst is 16-byte
// aligned, else element by element.
IAM_DEV void store_row16(float* dst, const float (&v)[16], int count) {
    if (count >= 16 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
#pragma unroll
        for (int j = 0; j < 16; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else {
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (j < count) dst[j] = v[j];
    }
}

__global__ void __launch_bounds__(128, 1)
    dense_gemm_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap thi,
                      const __grid_constant__ CUtensorMap tlo, GemmArgs a) {
    extern __shared__ unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[Tile::kStages];
    __shared__ __align__(8) uint64_t empty_bar[Tile::kStages];
    __shared__ __align__(8) uint64_t done_bar;
    __shared__ uint32_t tmem_slot;
    unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * kDenseBT, o0 = blockIdx.y * kDenseBW;
    const int kb0 = blockIdx.z * a.kb_per_split;
    const int nkb = min(a.kb_total - kb0, a.kb_per_split);  // >= 1: the host sizes the grid so
    const uint32_t stage_bytes = (uint32_t)((a.has_lo ? 2 : 1) * Tile::kA + Tile::kB);

    if (threadIdx.x == 0) {
        for (int s = 0; s < Tile::kStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(&done_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        tmem_alloc(&tmem_slot, Tile::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    pdl_wait();  // activations (and the residual) come from earlier kernels of the stream

    if (warp == 0 && lane == 0) {
        // producer: stage i of this slice into ring slot i % kStages once its MMAs are done
        int issued = 0;
        for (int i = 0; i < nkb; ++i) {
            const int s = i % Tile::kStages;
            const uint32_t ph = (uint32_t)(i / Tile::kStages) & 1u;
            if (!mbar_wait(&empty_bar[s], ph ^ 1u, a.err)) break;
            unsigned char* st = smem + (size_t)s * Tile::kStage;
            mbar_expect_tx(&full_bar[s], stage_bytes);
            const int kx = (kb0 + i) * kDenseBK;
            tma_load_2d(st, &thi, kx, t0, &full_bar[s]);
            if (a.has_lo) tma_load_2d(st + Tile::kA, &tlo, kx, t0, &full_bar[s]);
            tma_load_2d(st + 2 * Tile::kA, &tw, kx, o0, &full_bar[s]);
            issued = i + 1;
        }
        // drain: no bulk copy of this CTA may still be writing shared memory when it exits.
        // The last stage issued into each ring slot completes its full barrier when its bytes
        // have landed (at once on the normal path, where the MMA warp consumed every stage;
        // after a failed wait of the MMA warp this is what keeps the exit safe).  Bounded.
        for (int s = 0; s < Tile::kStages && s < issued; ++s) {
            const int last = s + Tile::kStages * ((issued - 1 - s) / Tile::kStages);
            mbar_wait(&full_bar[s], (uint32_t)(last / Tile::kStages) & 1u, a.err);
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer: 4 K-steps of 16 per stage; hi products into columns [0, 256), lo into [256, 512)
        for (int i = 0; i < nkb; ++i) {
            const int s = i % Tile::kStages;
            const uint32_t ph = (uint32_t)(i / Tile::kStages) & 1u;
            if (!mbar_wait(&full_bar[s], ph, a.err)) break;
            tc_fence_after();
            const unsigned char* st = smem + (size_t)s * Tile::kStage;
            const uint64_t dh = sw128_desc(st), dl = sw128_desc(st + Tile::kA), dw = sw128_desc(st + 2 * Tile::kA);
#pragma unroll
            for (int kk = 0; kk < kDenseBK / 16; ++kk) {
                const uint32_t acc = (i | kk) != 0 ? 1u : 0u;
                tc_mma(tmem, dh + 2u * kk, dw + 2u * kk, kIdesc, acc);
                if (a.has_lo) tc_mma(tmem + (uint32_t)kDenseBW, dl + 2u * kk, dw + 2u * kk, kIdesc, acc);
            }
            tc_commit(&empty_bar[s]);
        }
        tc_commit(&done_bar);  // also after a failed wait: nobody waits on done_bar forever
    }
    __syncwarp();

    // epilogue: accumulator lanes = tokens, columns = weight rows; a thread stores 16
    // consecutive outputs of its token per load
    mbar_wait(&done_bar, 0u, a.err);
    tc_fence_after();
    const int q = warp & 3;
    const int t = t0 + q * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
    if (a.silu_hi != nullptr && t0 + q * 32 < a.n) {
        // columns [0, 128) hold the gate rows, [128, 256) the up rows of the same FFN columns
        const int f0 = blockIdx.y * (kDenseBW / 2);
        for (int c = 0; c < kDenseBW / 2; c += 16) {
            uint32_t gh[16], gl[16], uh[16], ul[16];
            tmem_ld16(trow + (uint32_t)c, gh);
            tmem_ld16(trow + (uint32_t)(kDenseBW / 2 + c), uh);
            if (a.has_lo) {
                tmem_ld16(trow + (uint32_t)(kDenseBW + c), gl);
                tmem_ld16(trow + (uint32_t)(kDenseBW + kDenseBW / 2 + c), ul);
            }
            if (t < a.n) {
                uint32_t hw[8], lw[8];
#pragma unroll
                for (int j = 0; j < 16; j += 2) {
                    float av[2];
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const float g = __uint_as_float(gh[j + u]) + (a.has_lo ? __uint_as_float(gl[j + u]) : 0.0f);
                        const float up = __uint_as_float(uh[j + u]) + (a.has_lo ? __uint_as_float(ul[j + u]) : 0.0f);
                        av[u] = __fdiv_rn(__fmul_rn(up, g), __fadd_rn(1.0f, expf(-g)));  // matrix.cl:31
                    }
                    const __half h0 = __float2half_rn(av[0]), h1 = __float2half_rn(av[1]);
                    hw[j / 2] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
                    lw[j / 2] = (uint32_t)__half_as_ushort(__float2half_rn(__fsub_rn(av[0], __half2float(h0)))) |
                                ((uint32_t)__half_as_ushort(__float2half_rn(__fsub_rn(av[1], __half2float(h1)))) << 16);
                }
                const size_t o = (size_t)t * a.ld_silu + f0 + c;  // 32-byte aligned: ld_silu % 16 == 0
                uint4* dh = reinterpret_cast<uint4*>(a.silu_hi + o);
                uint4* dl = reinterpret_cast<uint4*>(a.silu_lo + o);
                dh[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                dh[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
                dl[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                dl[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
            }
        }
    } else if (t0 + q * 32 < a.n) {  // warp-uniform: this warp's 32 tokens hold at least one real one
        for (int c = 0; c < kDenseBW; c += 16) {
            const int o = o0 + c;
            if (o >= a.m) break;  // warp-uniform
            uint32_t rh[16], rl[16];
            tmem_ld16(trow + (uint32_t)c, rh);
            if (a.has_lo) tmem_ld16(trow + (uint32_t)(kDenseBW + c), rl);
            if (t < a.n) {
                const int cnt = min(16, a.m - o);
                float v[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(rh[j]) + (a.has_lo ? __uint_as_float(rl[j]) : 0.0f);
                if (a.partial != nullptr) {
                    store_row16(a.partial + ((size_t)blockIdx.z * a.n + t) * a.m + o, v, cnt);
                } else {
                    if (a.residual) {
                        const float* r = a.residual + (size_t)t * a.ldr + o;
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (j < cnt) v[j] = r[j] + v[j];
                    }
                    store_row16(a.y + (size_t)t * a.ldy + o, v, cnt);
                }
            }
        }
    }
    pdl_trigger();
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, Tile::kTmemCols);
    }
}

// y[t][o] = residual[t][o] + sum over slices z (in order) of partial[z][t][o].  Grid: (column
// blocks of 4 x 256 outputs, tokens); `vec` = rows 16-byte aligned (float4 path).
__global__ void __launch_bounds__(256) dense_reduce_kernel(const float* __restrict__ partial, int split, int n, int m,
                                                            float* y, int ldy, const float* residual, int ldr,
                                                            int vec) {
    pdl_wait();
    const int t = blockIdx.y;
    const int o = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (o < m) {
        const size_t plane = (size_t)n * m;
        const float* p = partial + (size_t)t * m + o;
        float* dst = y + (size_t)t * ldy + o;
        const float* r = residual ? residual + (size_t)t * ldr + o : nullptr;
        if (vec && o + 4 <= m) {
            float4 acc = *reinterpret_cast<const float4*>(p);
            for (int z = 1; z < split; ++z) {
                const float4 v = *reinterpret_cast<const float4*>(p + (size_t)z * plane);
                acc.x += v.x;
                acc.y += v.y;
                acc.z += v.z;
                acc.w += v.w;
            }
            if (r) {
                const float4 rv = *reinterpret_cast<const float4*>(r);
                acc.x = rv.x + acc.x;
                acc.y = rv.y + acc.y;
                acc.z = rv.z + acc.z;
                acc.w = rv.w + acc.w;
            }
            *reinterpret_cast<float4*>(dst) = acc;
        } else {
            for (int j = 0; j < 4 && o + j < m; ++j) {
                float acc = p[j];
                for (int z = 1; z < split; ++z) acc += p[(size_t)z * plane + j];
                dst[j] = (r ? r[j] : 0.0f) + acc;
            }
        }
    }
    pdl_trigger();
}

// Grid: (column blocks of 4 x 256, tokens).  k % 4 == 0, x rows 16-byte aligned.
__global__ void __launch_bounds__(256) dense_split_kernel(const float* __restrict__ x, int k, int ldx,
                                                           uint16_t* __restrict__ hi, uint16_t* __restrict__ lo) {
    pdl_wait();
    const int t = blockIdx.y;
    const int i = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (i < k) {
        const float4 v = *reinterpret_cast<const float4*>(x + (size_t)t * ldx + i);
        const __half h0 = __float2half_rn(v.x), h1 = __float2half_rn(v.y), h2 = __float2half_rn(v.z),
                     h3 = __float2half_rn(v.w);
        const size_t o = (size_t)t * k + i;
        uint2 hv;
        hv.x = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
        hv.y = (uint32_t)__half_as_ushort(h2) | ((uint32_t)__half_as_ushort(h3) << 16);
        *reinterpret_cast<uint2*>(hi + o) = hv;
        if (lo != nullptr) {
            const __half l0 = __float2half_rn(v.x - __half2float(h0)), l1 = __float2half_rn(v.y - __half2float(h1)),
                         l2 = __float2half_rn(v.z - __half2float(h2)), l3 = __float2half_rn(v.w - __half2float(h3));
            uint2 lv;
            lv.x = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
            lv.y = (uint32_t)__half_as_ushort(l2) | ((uint32_t)__half_as_ushort(l3) << 16);
            *reinterpret_cast<uint2*>(lo + o) = lv;
        }
    }
    pdl_trigger();
}

// Block: 16 inputs x 32 bucket columns.  The 16 ranks of bucket (i, c) carry the slots 0..15
// once each; every packed word goes to W'[16 c + slot][i] through a shared-memory transpose so
// both the bucket rows and the dense rows are accessed contiguously.
constexpr int kUnpackI = 16, kUnpackC = 32;

__global__ void __launch_bounds__(256) dense_unpack_kernel(const uint16_t* __restrict__ buckets, int in_dim, int cols,
                                                           uint16_t* __restrict__ w, int ldw, int rpb, int pitch,
                                                           int tag_rank) {
    __shared__ __align__(16) uint16_t s_out[kUnpackC * 16][kUnpackI];  // [dense row in tile][input]
    const int i0 = blockIdx.x * kUnpackI, c0 = blockIdx.y * kUnpackC;
    for (int e = threadIdx.x; e < kUnpackC * 16 * kUnpackI; e += blockDim.x) (&s_out[0][0])[e] = 0;
    __syncthreads();
    for (int e = threadIdx.x; e < kUnpackI * 16 * kUnpackC; e += blockDim.x) {
        const int row = e / kUnpackC, c = e % kUnpackC;  // row = il * 16 + rank
        const int il = row >> 4;
        if (i0 + il < in_dim && c0 + c < cols) {
            const uint16_t word = buckets[(size_t)(i0 * 16 + row) * cols + c0 + c];
            // the packed word, or its value bits with its bucket row (rank) in place of the slot
            s_out[c * 16 + (word & 15)][il] = tag_rank ? (uint16_t)((word & 0xFFF0u) | (unsigned)(row & 15)) : word;
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < kUnpackC * 16 * 2; e += blockDim.x) {
        const int orow = e >> 1, half = e & 1;
        const int o = c0 * 16 + orow;
        if (c0 + (orow >> 4) >= cols) continue;
        const int ib = i0 + half * 8;
        const size_t drow = rpb > 0 ? (size_t)(o / rpb) * pitch + o % rpb : (size_t)o;
        uint16_t* dst = w + drow * ldw + ib;
        if (ib + 8 <= in_dim) {
            *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(&s_out[orow][half * 8]);
        } else {
            for (int j = 0; ib + j < in_dim; ++j) dst[j] = s_out[orow][half * 8 + j];
        }
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// Tensor map of an fp16 matrix [rows][inner] (row stride ld elements), box {kDenseBK, box_rows},
// 128-byte swizzle; reads outside the matrix return zeros.
int make_map(CUtensorMap* map, const void* base, int inner, int rows, int ld, int box_rows) {
    auto fn = encoder();
    if (fn == nullptr) return fail(IAM_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 2u};
    const cuuint32_t box[2] = {(cuuint32_t)kDenseBK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1u, 1u};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(IAM_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return IAM_OK;
}

int launch_gemm(const DenseProblem& p, int split, int kb_total, int kb_per, cudaStream_t s, bool pdl) {
    static std::atomic<unsigned long long> attrs_set{0};
    IAM_CUDA_TRY(once_per_device(attrs_set, [] {
        return cudaFuncSetAttribute(dense_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Tile::kSmem);
    }));
    CUtensorMap tw, thi, tlo;
    int rc = make_map(&tw, p.w, p.k, p.m, p.ldw, kDenseBW);
    if (rc == IAM_OK) rc = make_map(&thi, p.x_hi, p.k, p.n, p.k, kDenseBT);
    if (rc == IAM_OK) rc = make_map(&tlo, p.x_lo ? p.x_lo : p.x_hi, p.k, p.n, p.k, kDenseBT);
    if (rc != IAM_OK) return rc;
    GemmArgs a;
    a.m = p.m;
    a.n = p.n;
    a.kb_total = kb_total;
    a.kb_per_split = kb_per;
    a.has_lo = p.x_lo != nullptr;
    a.y = p.y;
    a.ldy = p.ldy;
    a.residual = p.residual;
    a.ldr = p.ldr;
    a.partial = split > 1 ? p.partial : nullptr;
    a.err = p.err;
    a.silu_hi = p.silu_out_hi;
    a.silu_lo = p.silu_out_lo;
    a.ld_silu = p.ld_silu;
    const dim3 grid((p.n + kDenseBT - 1) / kDenseBT, (p.m + kDenseBW - 1) / kDenseBW, split);
    IAM_CUDA_TRY(launch_ex(dense_gemm_kernel, grid, dim3(128), Tile::kSmem, s, pdl, tw, thi, tlo, a));
    return IAM_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int dense_split(const float* x, int n, int k, int ldx, uint16_t* hi, uint16_t* lo, cudaStream_t s, bool pdl) {
    if (x == nullptr || hi == nullptr || n <= 0 || k <= 0 || n > kDenseMaxTokens)
        return fail(IAM_ERR_ARG, "dense_split: bad arguments");
    if (k % 4 != 0 || ldx % 4 != 0 || !aligned16(x) || (reinterpret_cast<uintptr_t>(hi) & 7u) ||
        (lo && (reinterpret_cast<uintptr_t>(lo) & 7u)))
        return fail(IAM_ERR_ARG, "dense_split: k and the row stride must be multiples of 4, x 16-byte aligned");
    IAM_CUDA_TRY(launch_ex(dense_split_kernel, dim3((k / 4 + 255) / 256, n), dim3(256), 0, s, pdl, x, k, ldx, hi, lo));
    return IAM_OK;
}

int dense_auto_split(int m, int k, int n, int sms) {
    const long tiles = (long)((m + kDenseBW - 1) / kDenseBW) * ((n + kDenseBT - 1) / kDenseBT);
    const int kb = (k + kDenseBK - 1) / kDenseBK;
    if (tiles >= sms) return 1;
    int split = (int)std::max(1L, (long)sms / tiles);
    split = std::min(split, kDenseMaxSplit);
    split = std::min(split, std::max(1, kb / 4));  // every slice at least 4 stages
    return split;
}

int dense_gemm(const DenseProblem& p, cudaStream_t s, bool pdl) {
    if (p.w == nullptr || p.x_hi == nullptr || p.y == nullptr || p.m <= 0 || p.k <= 0 || p.n <= 0 ||
        p.n > kDenseMaxTokens)
        return fail(IAM_ERR_ARG, "dense_gemm: bad arguments");
    if (p.k % 8 != 0 || p.ldw % 8 != 0 || p.ldw < p.k || !aligned16(p.w) || !aligned16(p.x_hi) ||
        (p.x_lo && !aligned16(p.x_lo)))
        return fail(IAM_ERR_ARG, "dense_gemm: k and the weight row stride must be multiples of 8 and the "
                                 "operands 16-byte aligned (TMA)");
    if (p.ldy < p.m || (p.residual && p.ldr < p.m)) return fail(IAM_ERR_ARG, "dense_gemm: output stride < m");
    const int kb_total = (p.k + kDenseBK - 1) / kDenseBK;
    int split = std::max(1, std::min(p.split, kDenseMaxSplit));
    int kb_per = (kb_total + split - 1) / split;
    split = (kb_total + kb_per - 1) / kb_per;  // every slice non-empty
    if (split > 1 && p.partial == nullptr) return fail(IAM_ERR_ARG, "dense_gemm: split-K needs a partial buffer");
    if (p.silu_out_hi != nullptr) {
        if (split != 1 || p.m % kDenseBW != 0 || p.silu_out_lo == nullptr || p.ld_silu % 16 != 0 ||
            p.ld_silu < p.m / 2 || !aligned16(p.silu_out_hi) || !aligned16(p.silu_out_lo))
            return fail(IAM_ERR_ARG, "dense_gemm: the SiLU epilogue needs m % 256 == 0, no K split, ld % 16 == 0");
    }
    const int rc = launch_gemm(p, split, kb_total, kb_per, s, pdl);
    if (rc != IAM_OK || split == 1) return rc;
    const int vec = p.m % 4 == 0 && p.ldy % 4 == 0 && aligned16(p.y) && (!p.residual || (p.ldr % 4 == 0 && aligned16(p.residual)));
    IAM_CUDA_TRY(launch_ex(dense_reduce_kernel, dim3((p.m + 1023) / 1024, p.n), dim3(256), 0, s, pdl,
                           (const float*)p.partial, split, p.n, p.m, p.y, p.ldy, p.residual, p.ldr, vec));
    return IAM_OK;
}

int dense_unpack(const uint16_t* buckets, int in_dim, int cols, uint16_t* w, int ldw, cudaStream_t s,
                 int rows_per_block, int block_pitch, bool tag_rank) {
    if (buckets == nullptr || w == nullptr || in_dim <= 0 || cols <= 0 || ldw < in_dim)
        return fail(IAM_ERR_ARG, "dense_unpack: bad arguments");
    if (ldw % 8 != 0 || !aligned16(w)) return fail(IAM_ERR_ARG, "dense_unpack: ldw % 8 and 16-byte alignment");
    if (rows_per_block < 0 || (rows_per_block > 0 && block_pitch < rows_per_block))
        return fail(IAM_ERR_ARG, "dense_unpack: row blocks");
    const dim3 grid((in_dim + kUnpackI - 1) / kUnpackI, (cols + kUnpackC - 1) / kUnpackC);
    dense_unpack_kernel<<<grid, 256, 0, s>>>(buckets, in_dim, cols, w, ldw, rows_per_block, block_pitch, tag_rank ? 1 : 0);
    IAM_CUDA_TRY(cudaGetLastError());
    return IAM_OK;
}

}  // namespace iam

using namespace iam;

// Handle of the C entry points: activation halves and split-K partials for the largest
// problem the caller announced.
struct iam_dense_s {
    int device = 0, sms = 148;
    int max_tokens = 0, max_in = 0, max_out = 0;
    uint16_t* hi = nullptr;
    uint16_t* lo = nullptr;
    float* partial = nullptr;
    size_t partial_cap = 0;  // floats
    unsigned* err = nullptr;
};

extern "C" {

int iam_dense_destroy(iam_dense_t h) {
    if (!h) return IAM_OK;
    cudaFree(h->hi);
    cudaFree(h->lo);
    cudaFree(h->partial);
    cudaFree(h->err);
    delete h;
    return IAM_OK;
}

int iam_dense_create(int max_tokens, int max_in_dim, int max_out_dim, int device, iam_dense_t* out) {
    if (!out) return fail(IAM_ERR_ARG, "iam_dense_create: null out");
    *out = nullptr;
    if (max_tokens <= 0 || max_tokens > kDenseMaxTokens || max_in_dim <= 0 || max_out_dim <= 0 || max_in_dim % 8 != 0)
        return fail(IAM_ERR_ARG, "iam_dense_create: sizes must be positive, max_tokens <= 65535, max_in_dim % 8 == 0");
    int rc = iam_device_info(device, nullptr, nullptr, nullptr);
    if (rc) return rc;
    IAM_CUDA_TRY(cudaSetDevice(device));
    iam_dense_s* h = new iam_dense_s();
    h->device = device;
    h->max_tokens = max_tokens;
    h->max_in = max_in_dim;
    h->max_out = max_out_dim;
    cudaDeviceGetAttribute(&h->sms, cudaDevAttrMultiProcessorCount, device);
    // the automatic split keeps tiles x split <= SMs, so its partials fit in SMs x one tile
    const size_t act = (size_t)max_tokens * max_in_dim;
    h->partial_cap = dense_partial_floats(h->sms);
    cudaError_t e = cudaMalloc(&h->hi, act * sizeof(uint16_t));
    if (e == cudaSuccess) e = cudaMalloc(&h->lo, act * sizeof(uint16_t));
    if (e == cudaSuccess) e = cudaMalloc(&h->partial, h->partial_cap * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&h->err, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(h->err, 0, sizeof(unsigned));
    if (e != cudaSuccess) {
        iam_dense_destroy(h);
        return cuda_fail(e, "iam_dense_create: cudaMalloc");
    }
    *out = h;
    return IAM_OK;
}

int iam_dense_gemm(iam_dense_t h, const uint16_t* w_dev, int out_dim, int in_dim, const float* x_dev, int n_tokens,
                   const float* residual_dev, float* y_dev, int precision, int split_k, void* stream) {
    if (!h || !w_dev || !x_dev || !y_dev) return fail(IAM_ERR_ARG, "iam_dense_gemm: null argument");
    if (n_tokens <= 0 || out_dim <= 0 || in_dim <= 0 || n_tokens > h->max_tokens || in_dim > h->max_in ||
        out_dim > h->max_out)
        return fail(IAM_ERR_ARG, "iam_dense_gemm: sizes outside the handle's limits");
    if (precision != 0 && precision != 1) return fail(IAM_ERR_ARG, "iam_dense_gemm: precision must be 0 or 1");
    if (split_k < 0) return fail(IAM_ERR_ARG, "iam_dense_gemm: split_k < 0");
    const cudaStream_t s = (cudaStream_t)stream;
    int rc = dense_split(x_dev, n_tokens, in_dim, in_dim, h->hi, precision == 0 ? h->lo : nullptr, s);
    if (rc) return rc;
    DenseProblem p{};
    p.w = w_dev;
    p.m = out_dim;
    p.k = in_dim;
    p.ldw = in_dim;
    p.x_hi = h->hi;
    p.x_lo = precision == 0 ? h->lo : nullptr;
    p.n = n_tokens;
    p.y = y_dev;
    p.ldy = out_dim;
    p.residual = residual_dev;
    p.ldr = out_dim;
    p.split = split_k == 0 ? dense_auto_split(out_dim, in_dim, n_tokens, h->sms) : split_k;
    if (p.split > 1 && (size_t)std::min(p.split, kDenseMaxSplit) * n_tokens * out_dim > h->partial_cap)
        return fail(IAM_ERR_ARG, "iam_dense_gemm: split_k x n_tokens x out_dim exceeds the split-K scratch");
    p.partial = h->partial;
    p.err = h->err;
    return dense_gemm(p, s);
}

int iam_dense_status(iam_dense_t h) {
    if (!h) return fail(IAM_ERR_ARG, "iam_dense_status: null handle");
    IAM_CUDA_TRY(cudaSetDevice(h->device));
    IAM_CUDA_TRY(cudaDeviceSynchronize());
    unsigned v = 0;
    IAM_CUDA_TRY(cudaMemcpy(&v, h->err, sizeof(v), cudaMemcpyDeviceToHost));
    if (v == 0) return IAM_OK;
    IAM_CUDA_TRY(cudaMemset(h->err, 0, sizeof(unsigned)));
    return fail(IAM_ERR_TIMEOUT, "iam_dense: a pipeline wait gave up");
}

int iam_dense_unpack(const uint16_t* buckets_dev, int in_dim, int bucket_cols, uint16_t* w_out_dev, void* stream) {
    return dense_unpack(buckets_dev, in_dim, bucket_cols, w_out_dev, in_dim, (cudaStream_t)stream);
}

}  // extern "C"
