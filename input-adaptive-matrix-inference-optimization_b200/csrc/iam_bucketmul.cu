// iam_bucketmul.cu -- fused bucketMul kernel (sm_100a) and its launch planning.
//
// Reference operator: BucketMul (bucket_mul.hpp:99-268) over bucketMul.cl:68-497.
//
// One launch runs up to kMaxProblems bucketMuls.  Grid = clusters of G CTAs; a cluster owns
// one column tile of one problem and one of n_split input ranges.  Per CTA (rank g):
//   0. weights-only prologue (the probes and this CTA's stats segment towards L2), then the
//      programmatic-dependent-launch wait for the previous kernel of the stream;
//   1. cutoff: block_find_cutoff over x[0:P] by 4 warps (every CTA, identical result) while
//      the other warps compute the row importances of the CTA's inputs;
//   2. selection masks for its share of the cluster's inputs (block_masks_pre), then its
//      selected rows as 16-bit offsets in its own shared memory; one cluster barrier; a
//      prefix over the G counts read through DSMEM numbers the cluster's rows 0..S-1;
//   3. the CTA takes rows [S*g/G, S*(g+1)/G) of that numbering, wherever they live: it
//      stages {row*C, x(row)} for 2048 rows at a time (row offsets read from the owner's
//      shared memory through DSMEM, next chunk fetched during the current one); each lane
//      keeps a ring of kD rows of VEC-wide weight slices in registers and adds x*w into
//      lane-private per-slot accumulators in shared memory, addressed with one shift and
//      one LOP3 per weight (accumulate_sh);
//   4. lane accumulators -> a partial tile per CTA -> fixed-order DSMEM sum across the
//      cluster; with n_split > 1 the partial tiles go to global scratch and the last cluster
//      to arrive at each slice adds them in split order -> out (+ residual).
// No float atomics anywhere: results are bitwise deterministic.
#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>

#include "iam_bucketmul.cuh"
#include "iam_bucketmul_launch.h"

namespace iam {

constexpr int kCH = 2048;  // rows per staged chunk
#ifndef IAM_BM_RING
#define IAM_BM_RING 8
#endif
constexpr int kD = IAM_BM_RING;  // rows per lane in flight (register ring; 8 fits 128 registers)
constexpr int kSumBatch = 16;  // split partials loaded at once by the last cluster

// Threads per CTA for a vector width: the lane accumulators (16 slots x VEC floats per
// lane) fill 128 KB of shared memory either way; narrower loads buy more warps.
template <int VEC>
struct Threads {
    static constexpr int value = VEC == 4 ? 512 : 256;
};

template <int NT>
struct FusedHeader {
    CutoffShared<NT> cut;
    ScanShared<NT> scan;
    float red[256];
    int my_count;
    int my_row_base;
    int last_flag;
    int pre[kMaxCluster + 1];
    int row_base[kMaxCluster];
};

constexpr size_t align16(size_t n) { return (n + 15) / 16 * 16; }

template <int VEC>
constexpr size_t fixed_smem_bytes() {
    constexpr int NT = Threads<VEC>::value;
    return align16(sizeof(FusedHeader<NT>)) + 2 * kCH * sizeof(uint2)  // header, staging
           + sizeof(float) * 16 * VEC * 32                             // partial tile
           + (16u << SlotShift<VEC>::value)                            // alignment of the accumulators
           + sizeof(float) * NT * VEC * 16;                            // lane accumulators
}

size_t bm_smem_bytes(int vec, int seg_inputs) {
    const size_t lists = align16((size_t)seg_inputs * sizeof(uint16_t))         // masks
                         + align16((size_t)seg_inputs * 16 * sizeof(uint16_t));  // local rows
    if (vec == 8) return fixed_smem_bytes<8>() + lists;
    if (vec == 4) return fixed_smem_bytes<4>() + lists;
    return fixed_smem_bytes<1>() + lists;
}

IAM_DEV void stamp(long long* dbg, int k) { debug_stamp(dbg, k); }

template <int XM, int NT>
struct Provider;
template <int NT>
struct Provider<kXPlain, NT> {
    using T = XPlain;
    static IAM_DEV T make(const BMProblem& p, float*) { return XPlain{p.x}; }
};
template <int NT>
struct Provider<kXRms, NT> {
    using T = XRms;
    static IAM_DEV T make(const BMProblem& p, float* red) {
        return XRms{p.x, p.gain, block_rms_scale<NT>(p.x, p.norm_n, p.norm_eps, red)};
    }
};
template <int NT>
struct Provider<kXSilu, NT> {
    using T = XSilu;
    static IAM_DEV T make(const BMProblem& p, float*) { return XSilu{p.x, p.x2}; }
};

template <int VEC, int XM>
__global__ void __launch_bounds__(Threads<VEC>::value, 1) bm_fused_kernel(const __grid_constant__ BMBatch batch) {
    constexpr int NT = Threads<VEC>::value, NW = NT / 32;
    using VL = VecLoad<VEC>;
    using VT = typename VL::T;
    cg::cluster_group cluster = cg::this_cluster();
    const int G = (int)cluster.num_blocks();
    const int g = (int)cluster.block_rank();
    const int ci = (int)(blockIdx.x / G);
    int pi = 0;
    while (pi + 1 < batch.nprob && ci >= batch.p[pi + 1].cluster_begin) ++pi;
    const BMProblem& pr = batch.p[pi];
    const int local = ci - pr.cluster_begin;
    const int tile = local % pr.n_tiles, split = local / pr.n_tiles;
    const int K = pr.n_split;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    long long* dbg = (ci == 0 && g == 0 && tid == 0) ? pr.dbg : nullptr;
    long long* tr = (pr.trace && tid == 0 && (int)blockIdx.x < pr.trace_cap) ? pr.trace + 8 * blockIdx.x : nullptr;
    stamp(dbg, 0);
    stamp(tr, 0);

    extern __shared__ __align__(16) unsigned char smem_raw[];
    FusedHeader<NT>& hdr = *reinterpret_cast<FusedHeader<NT>*>(smem_raw);
    uint2* stage = reinterpret_cast<uint2*>(smem_raw + align16(sizeof(FusedHeader<NT>)));
    float* part = reinterpret_cast<float*>(stage + 2 * kCH);
    // lane accumulators: one region of 16 << SS bytes per warp, aligned to its size in the
    // shared window so that slot bits can be OR-ed into the lane's address
    constexpr uint32_t kRegion = 16u << SlotShift<VEC>::value;
    const uint32_t acc_sh0 = (uint32_t)__cvta_generic_to_shared(part + 16 * VEC * 32);
    const uint32_t acc_sh = (acc_sh0 + kRegion - 1) & ~(kRegion - 1);
    float* acc = part + 16 * VEC * 32 + (acc_sh - acc_sh0) / sizeof(float);
    uint16_t* masks = reinterpret_cast<uint16_t*>(acc + NT * VEC * 16);
    uint16_t* rows16 = masks + align16((size_t)pr.seg_inputs * sizeof(uint16_t)) / sizeof(uint16_t);

    const long long row0 = pr.row0;
    const bool from_list = batch.mode == kModeMulOnly;
    const int span = (pr.n_inputs - pr.in_begin + K - 1) / K;
    const int klo = min(pr.in_begin + split * span, pr.n_inputs);
    const int khi = min(klo + span, pr.n_inputs);
    const int i0 = min(klo + g * pr.seg_inputs, khi);
    const int i1 = min(i0 + pr.seg_inputs, khi);

    // ---- prologue on weights only (nothing an earlier kernel of the stream writes): the
    // cutoff's probes and this CTA's stats segment start on their way to L2
    if (!from_list) {
        if (tid == 0 && ((reinterpret_cast<uintptr_t>(pr.probes) & 15u) == 0) && (pr.P % 8) == 0)
            prefetch_l2(pr.probes, (uint32_t)pr.P * 2u);
        const uint16_t* s0 = pr.stats + (row0 + 16LL * i0) * pr.stats_stride;
        const long long sbytes = 32LL * (i1 - i0) * pr.stats_stride;
        if (((reinterpret_cast<uintptr_t>(s0) & 15u) == 0)) {
            for (long long off = (long long)tid * 16384; off < sbytes; off += (long long)NT * 16384)
                prefetch_l2(reinterpret_cast<const unsigned char*>(s0) + off, (uint32_t)min(16384LL, sbytes - off));
        }
    }
    pdl_wait();  // from here on: x, residuals and scratch written by earlier kernels

    const auto xp = Provider<XM, NT>::make(pr, hdr.red);

    // ---- phases 1-2: cutoff, selection masks, cluster-local row numbering
    int S, list_lo = 0;
    if (!from_list) {
        int iters = 0;
        // the warps outside the cutoff search compute the row importances of the first
        // NT - 128 inputs of this CTA's segment meanwhile; only the comparisons wait
        constexpr int kSearch = 128, kPre = NT - kSearch;
        float pimp[16];
        int pin = -1;
        auto side = [&]() {
            const int i = i0 + (tid - kSearch);
            if (i < i1) {
                input_importances(xp, pr.stats, pr.stats_stride, row0, pr.n_rows_valid, i, pimp);
                pin = i;
            }
        };
        const float cutoff = block_find_cutoff<NT, 4>(xp, pr.probes, pr.P, pr.target, hdr.cut, &iters,
                                                      dbg ? dbg + 8 : nullptr, side);
        stamp(dbg, 1);
        stamp(tr, 1);
        const int n = block_masks_pre<NT>(xp, pr.stats, pr.stats_stride, row0, pr.n_rows_valid, i0, i1, kPre, cutoff,
                                          pin, pimp, masks, hdr.scan);
        block_write_rows_local<NT>(masks, i0, i1, rows16, hdr.scan);
        if (tid == 0) {
            hdr.my_count = n;
            hdr.my_row_base = (int)(row0 + 16LL * i0);
        }
        stamp(dbg, 2);
        stamp(tr, 2);
        cluster.sync();  // counts and local row lists visible cluster-wide
        if (warp == 0) {  // all G peer counts read in parallel, then a warp scan
            const int c = lane < G ? *cluster.map_shared_rank(&hdr.my_count, lane) : 0;
            if (lane < G) hdr.row_base[lane] = *cluster.map_shared_rank(&hdr.my_row_base, lane);
            int inc = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += t;
            }
            if (lane <= G) hdr.pre[lane] = inc - c;
        }
        __syncthreads();
        S = hdr.pre[G];
        if (batch.mode == kModeSelectOnly) {  // one cluster per problem: publish the compact list
            const int base = hdr.pre[g];
            for (int j = tid; j < n; j += NT) pr.list[base + j] = hdr.my_row_base + (int)rows16[j];
            if (g == 0 && tid == 0) {
                if (pr.cutoff_out) *pr.cutoff_out = cutoff;
                if (pr.iters_out) *pr.iters_out = iters;
                if (pr.count_out) *pr.count_out = S;
                if (pr.sel_total) *pr.sel_total = S;
            }
            cluster.sync();  // peers are done reading my counts
            return;
        }
        if (tile == 0 && g == 0 && tid == 0) {
            if (split == 0 && pr.cutoff_out) *pr.cutoff_out = cutoff;
            if (split == 0 && pr.iters_out) *pr.iters_out = iters;
            if (K == 1 && pr.count_out) *pr.count_out = S;
            if (K > 1) pr.split_sel[split] = S;
        }
        stamp(dbg, 3);
        stamp(tr, 3);
    } else {
        const int total = __ldcg(pr.sel_total);
        list_lo = (int)(((long long)total * split) / K);
        S = (int)(((long long)total * (split + 1)) / K) - list_lo;
    }

    // ---- phase 3: accumulate rows [a, b) of the cluster's numbering
    const int a = (int)(((long long)S * g) / G);
    const int b = (int)(((long long)S * (g + 1)) / G);
    if (tr) tr[7] = b - a;
    const int log2L = pr.log2L;
    const int L = 1 << log2L, P = 32 >> log2L;
    const int rg = lane >> log2L, q = lane & (L - 1);
    const int TW = VEC * L;
    const int c0 = tile * TW + q * VEC;
    const bool col_ok = c0 < pr.cols;
    const uint16_t* __restrict__ wbase = pr.buckets + (col_ok ? c0 : 0);
    const int cols = pr.cols;
    const int32_t bucket_row0 = (int32_t)pr.bucket_row0;

    float* my_acc = acc + (size_t)warp * 16 * VEC * 32 + lane;
    const uint32_t acc_lane = acc_sh + (uint32_t)warp * kRegion + (uint32_t)lane * 4u;
#pragma unroll 4
    for (int j = 0; j < 16 * VEC; ++j) my_acc[j * 32] = 0.0f;

    constexpr int SPT = kCH / NT;  // staged rows per thread per chunk
    auto stage_fetch = [&](int p0, int n, int32_t* rr, float* xx) {
#pragma unroll
        for (int k = 0; k < SPT; ++k) {
            const int j = tid + k * NT;
            if (j < n) {
                const int p = p0 + j;
                int32_t row;
                if (from_list) {
                    row = __ldcg(pr.list + list_lo + p);
                } else {
                    int gs = 0;
                    while (gs + 1 < G && p >= hdr.pre[gs + 1]) ++gs;
                    row = hdr.row_base[gs] + (int32_t)cluster.map_shared_rank(rows16, gs)[p - hdr.pre[gs]];
                }
                rr[k] = row;
                xx[k] = xp((int)((row - row0) >> 4));
            }
        }
    };
    auto stage_store = [&](uint2* st, int n, const int32_t* rr, const float* xx) {
#pragma unroll
        for (int k = 0; k < SPT; ++k) {
            const int j = tid + k * NT;
            if (j < n) st[j] = make_uint2((uint32_t)(rr[k] - bucket_row0) * (uint32_t)cols, __float_as_uint(xx[k]));
        }
    };

    int32_t rr[SPT];
    float xx[SPT];
    {
        const int n0 = min(kCH, b - a);
        stage_fetch(a, n0, rr, xx);
        stage_store(stage, n0, rr, xx);
    }
    __syncthreads();

    int buf = 0;
    for (int cstart = a; cstart < b; cstart += kCH, buf ^= 1) {
        const int n = min(kCH, b - cstart);
        const int nn = min(kCH, b - (cstart + kCH));
        stage_fetch(cstart + kCH, nn, rr, xx);  // next chunk, overlapped with this one

        const uint2* st = stage + buf * kCH;
        // rows j = rg + P*(warp + NW*m), m = 0..mw-1; a ring of kD rows per lane: row m is
        // accumulated, then row m + kD is loaded into its registers (kD - 1 rows in flight).
        // Past the end a lane re-reads the last row with x = 0 (adds exact zeros), so the
        // loop carries no branches; lanes of a partial tile read column 0 into accumulators
        // that are never written out.
        const int first = P * warp;
        const int mw = n > first ? (n - first + P * NW - 1) / (P * NW) : 0;
        if (mw > 0) {
            const int j0 = rg + first, jstep = P * NW, jlast = n - 1;
            VT w[kD];
            float xs[kD];
            auto load_row = [&](int m, VT& wr, float& xr) {
                const int j = j0 + m * jstep;
                const bool ok = j < n;
                const uint2 e = st[ok ? j : jlast];
                wr = VL::load(wbase + e.x);
                xr = ok ? __uint_as_float(e.y) : 0.0f;
            };
#pragma unroll
            for (int d = 0; d < kD; ++d) load_row(d, w[d], xs[d]);
            for (int base = 0; base < mw; base += kD) {
#pragma unroll
                for (int d = 0; d < kD; ++d) {
                    accumulate_sh<VEC>(acc_lane, w[d], xs[d]);
                    load_row(base + d + kD, w[d], xs[d]);
                }
            }
        }

        stage_store(stage + (buf ^ 1) * kCH, nn, rr, xx);
        __syncthreads();
    }
    stamp(dbg, 4);
    stamp(tr, 4);
    pdl_trigger();  // the successor may start its weights-only prologue on SMs this launch frees

    // ---- phase 4: lane accumulators -> CTA partial tile -> cluster sum -> splits
    for (int sk = warp; sk < 16 * VEC; sk += NW) {
        float v = 0.0f;
#pragma unroll
        for (int w2 = 0; w2 < NW; ++w2) v += acc[((size_t)w2 * 16 * VEC + sk) * 32 + lane];
        for (int o = 16; o >= L; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane < L) {
            const int slot = sk / VEC, k = sk % VEC;
            part[(lane * VEC + k) * 16 + slot] = v;
        }
    }
    cluster.sync();
    stamp(dbg, 5);
    stamp(tr, 5);
    const int nout = 16 * TW;
    const int per = (nout + G - 1) / G;
    const int o0 = min(nout, g * per), o1 = min(nout, o0 + per);
    const int n_own = o1 - o0;
    float* gathered = acc;  // [n_own][G]; the accumulators are dead, peers only read `part`
    for (int k = tid; k < n_own * G; k += NT) {  // all remote loads in flight at once
        const int oo = k / G, r = k - oo * G;
        gathered[k] = cluster.map_shared_rank(part, r)[o0 + oo];
    }
    __syncthreads();
    const size_t tile_out = (size_t)tile * TW * 16;
    const size_t split_stride = (size_t)16 * cols;
    for (int oo = tid; oo < n_own; oo += NT) {
        float s = 0.0f;
        for (int r = 0; r < G; ++r) s += gathered[oo * G + r];  // fixed order: deterministic
        const int o = o0 + oo;
        if (tile * TW + o / 16 < cols) {
            const size_t j = tile_out + o;  // = col*16 + slot
            if (K == 1) {
                if (pr.residual) s = pr.residual[j] + s;  // add32 (bucketMul.cl:517-520)
                pr.out[j] = s;
            } else {
                pr.partials[(size_t)split * split_stride + j] = s;
            }
        }
    }
    if (K > 1) {  // last cluster to finish this slice adds the splits in order
        __threadfence();
        __syncthreads();
        if (tid == 0) hdr.last_flag = (atomicAdd(pr.slice_ctr + tile * G + g, 1) == K - 1);
        __syncthreads();
        if (hdr.last_flag) {
            __threadfence();
            for (int oo = tid; oo < n_own; oo += NT) {
                const int o = o0 + oo;
                if (tile * TW + o / 16 < cols) {
                    const size_t j = tile_out + o;
                    const float res = pr.residual ? pr.residual[j] : 0.0f;  // in flight with the partials
                    float s = 0.0f;
                    for (int kb = 0; kb < K; kb += kSumBatch) {  // kSumBatch loads in flight, added in split order
                        float v[kSumBatch];
#pragma unroll
                        for (int u = 0; u < kSumBatch; ++u)
                            v[u] = kb + u < K ? __ldcg(pr.partials + (size_t)(kb + u) * split_stride + j) : 0.0f;
#pragma unroll
                        for (int u = 0; u < kSumBatch; ++u)
                            if (kb + u < K) s += v[u];
                    }
                    if (pr.residual) s = res + s;
                    pr.out[j] = s;
                }
            }
            if (tid == 0) pr.slice_ctr[tile * G + g] = 0;  // ready for the next launch
            if (warp == NW - 1 && tile == 0 && g == 0 && pr.count_out) {  // one warp, all loads at once
                int t = 0;
                for (int k = lane; k < K; k += 32) t += __ldcg(pr.split_sel + k);
                t = __reduce_add_sync(0xffffffffu, t);
                if (lane == 0) *pr.count_out = t;
            }
        }
    }
    cluster.sync();  // peers are done reading `part` and my row list
    stamp(dbg, 6);
    stamp(tr, 6);
}

// ------------------------------------------------------------------ standalone kernels

template <int NT>
__global__ void __launch_bounds__(NT) bm_cutoff_kernel(const float* x, const uint16_t* probes, int P,
                                                       int target, float* out, int* iters) {
    __shared__ CutoffShared<NT> sm;
    int it = 0;
    const float c = block_find_cutoff<NT>(XPlain{x}, probes, P, target, sm, &it);
    if (threadIdx.x == 0) {
        out[0] = c;
        if (iters) iters[0] = it;
    }
}

__global__ void stats_pack_kernel(const uint16_t* s4, long long rows, uint16_t* s1) {
    for (long long r = blockIdx.x * (long long)blockDim.x + threadIdx.x; r < rows;
         r += (long long)gridDim.x * blockDim.x)
        s1[r] = s4[r * 4 + 3];
}

// ------------------------------------------------------------------ host launch helpers

namespace {

int env_int(const char* name, int dflt) {
    const char* v = getenv(name);
    return (v && *v) ? atoi(v) : dflt;
}

template <int VEC, int XM>
cudaError_t set_attrs() {
    static std::atomic<unsigned long long> done{0};
    return once_per_device(done, [] {
        auto kern = bm_fused_kernel<VEC, XM>;
        cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (err == cudaSuccess) err = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        return err;
    });
}

template <int VEC, int XM>
int launch_one(const BMBatch& b, int G, int n_clusters, size_t smem, cudaStream_t s) {
    auto kern = bm_fused_kernel<VEC, XM>;
    cudaError_t e = set_attrs<VEC, XM>();
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(bm_fused)");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(n_clusters * G));
    cfg.blockDim = dim3(Threads<VEC>::value);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)G;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = b.pdl ? 2 : 1;
    IAM_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, b));
    return IAM_OK;
}

template <int VEC>
int launch_vec(const BMBatch& b, int G, int n, size_t smem, cudaStream_t s) {
    switch (b.xmode) {
        case kXRms: return launch_one<VEC, kXRms>(b, G, n, smem, s);
        case kXSilu: return launch_one<VEC, kXSilu>(b, G, n, smem, s);
        default: return launch_one<VEC, kXPlain>(b, G, n, smem, s);
    }
}

template <int VEC>
int occupancy_clusters(int G, size_t smem) {
    auto kern = bm_fused_kernel<VEC, kXPlain>;
    if (set_attrs<VEC, kXPlain>() != cudaSuccess) return 1;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)G;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.blockDim = dim3(Threads<VEC>::value);
    cfg.gridDim = dim3((unsigned)(G * 64));
    cfg.dynamicSmemBytes = smem;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = 1;
    }
    return n;
}

int seg_inputs_max(const BMBatch& b) {
    int m = 1;
    for (int i = 0; i < b.nprob; ++i) m = std::max(m, b.p[i].seg_inputs);
    return m;
}

}  // namespace

int bm_max_active_clusters(int vec, int G) {
    // occupancy with the fixed part of shared memory plus lists for 256 inputs per CTA
    static std::mutex mu;
    static std::map<std::pair<int, int>, int> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    const auto key = std::make_pair(vec * 64 + G, dev);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    const size_t smem = bm_smem_bytes(vec, 256);
    const int n = vec == 8 ? occupancy_clusters<8>(G, smem) : vec == 4 ? occupancy_clusters<4>(G, smem)
                                                                       : occupancy_clusters<1>(G, smem);
    cache[key] = n;
    return n;
}

int bm_default_cluster() {
    const int g = env_int("IAM_BM_CLUSTER", 4);
    return (g == 1 || g == 2 || g == 4 || g == 8 || g == 16) ? g : 4;
}

// Launch plan: every problem gets the widest column tiles its row width allows (32 lanes x
// VEC columns, i.e. 256 or 512 B of each row per tile), then as many input splits as its
// share of the resident clusters (by selected-row work) allows, so the batch is one full
// wave; splits are raised further if a CTA's input segment would not fit shared memory.
void bm_plan(BMBatch& b, int vec, int G, int max_clusters, int max_splits) {
    const int forced_l2 = env_int("IAM_BM_LOG2L", -1);
    const int forced_k = env_int("IAM_BM_SPLIT", -1);
    double work_total = 0.0;
    for (int i = 0; i < b.nprob; ++i) work_total += (double)b.p[i].cols * b.p[i].n_rows_valid;
    int begin = 0;
    for (int i = 0; i < b.nprob; ++i) {
        BMProblem& p = b.p[i];
        int l2 = 0;
        while (l2 < 5 && (vec << l2) < p.cols) ++l2;
        if (forced_l2 >= 0 && forced_l2 <= 5) l2 = forced_l2;
        p.log2L = l2;
        p.n_tiles = (p.cols + (vec << l2) - 1) / (vec << l2);
        const int inputs = std::max(1, p.n_inputs - p.in_begin);
        int K = 1;
        if (b.mode != kModeSelectOnly) {
            const double share = work_total > 0 ? max_clusters * ((double)p.cols * p.n_rows_valid) / work_total
                                                : (double)max_clusters;
            K = std::max(1, (int)(share / p.n_tiles));
            if (forced_k > 0) K = forced_k;
            K = std::min(K, std::max(1, inputs / G));  // at least one input per CTA
            K = std::min(K, std::min(max_splits, kMaxSplits));
        }
        int seg;
        for (;;) {
            const int span = (inputs + K - 1) / K;
            seg = (span + G - 1) / G;
            if ((seg <= kMaxSegInputs && bm_smem_bytes(vec, seg) <= 227 * 1024) || K >= std::min(max_splits, kMaxSplits))
                break;
            ++K;
        }
        p.n_split = K;
        p.seg_inputs = std::max(1, seg);
        p.cluster_begin = begin;
        begin += p.n_tiles * K;
    }
}

int bm_total_clusters(const BMBatch& b) {
    int n = 0;
    for (int i = 0; i < b.nprob; ++i) n += b.p[i].n_tiles * b.p[i].n_split;
    return n;
}

int bm_launch(const BMBatch& b, int vec, int G, cudaStream_t s) {
    const int n = b.mode == kModeSelectOnly ? b.nprob : bm_total_clusters(b);
    if (seg_inputs_max(b) > kMaxSegInputs)
        return fail(IAM_ERR_UNSUPPORTED, "bucketmul: more than 4096 inputs per CTA segment");
    const size_t smem = bm_smem_bytes(vec, seg_inputs_max(b));
    if (smem > 227 * 1024) return fail(IAM_ERR_UNSUPPORTED, "bucketmul: segment too large for shared memory");
    if (vec == 8) return launch_vec<8>(b, G, n, smem, s);
    if (vec == 4) return launch_vec<4>(b, G, n, smem, s);
    return launch_vec<1>(b, G, n, smem, s);
}

int bm_launch_cutoff(const float* x, const uint16_t* probes, int P, int target, float* out, int* iters,
                     cudaStream_t s) {
    bm_cutoff_kernel<256><<<1, 256, 0, s>>>(x, probes, P, target, out, iters);
    IAM_CUDA_TRY(cudaGetLastError());
    return IAM_OK;
}

int bm_launch_stats_pack(const uint16_t* s4, long long rows, uint16_t* s1, cudaStream_t s) {
    const int blocks = (int)std::min<long long>((rows + 255) / 256, 4096);
    stats_pack_kernel<<<blocks > 0 ? blocks : 1, 256, 0, s>>>(s4, rows, s1);
    IAM_CUDA_TRY(cudaGetLastError());
    return IAM_OK;
}

}  // namespace iam
