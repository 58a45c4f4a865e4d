// iam_bucketmul.cu -- fused bucketMul kernels and the bucketMul C ABI.
//
// Reference operator: BucketMul (bucket_mul.hpp:99-268) over bucketMul.cl:68-497.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "iam_bucketmul.cuh"
#include "iam_bucketmul_launch.h"

namespace iam {

// ------------------------------------------------------------------ fused kernel

template <int NT>
struct FusedHeader {
    CutoffShared<NT> cut;
    ScanShared<NT> scan;
    int my_count;
    int pre[kMaxCluster + 1];
};

template <int VEC, int NT>
constexpr size_t fused_smem_bytes() {
    return ((sizeof(FusedHeader<NT>) + 15) / 16) * 16     // header
           + sizeof(float) * 16 * VEC * 32                // part: one column tile, 16 slots
           + sizeof(float) * (NT / 32) * 32 * VEC * 16;   // per-warp lane-private accumulators
}

// One launch = up to kMaxProblems independent bucketMuls (e.g. q/k/v sharing x).
// Cluster ci belongs to problem p and covers column tile (ci - p.cluster_begin).
template <int VEC, int NT, int U>
__global__ void __launch_bounds__(NT, 1) bm_fused_kernel(const __grid_constant__ BMBatch batch) {
    constexpr int NW = NT / 32;
    cg::cluster_group cluster = cg::this_cluster();
    const int G = (int)cluster.num_blocks();
    const int g = (int)cluster.block_rank();
    const int ci = (int)(blockIdx.x / G);
    int pi = 0;
    while (pi + 1 < batch.nprob && ci >= batch.p[pi + 1].cluster_begin) ++pi;
    const BMProblem& pr = batch.p[pi];
    const int tile = ci - pr.cluster_begin;

    extern __shared__ __align__(16) unsigned char smem_raw[];
    FusedHeader<NT>& hdr = *reinterpret_cast<FusedHeader<NT>*>(smem_raw);
    float* part = reinterpret_cast<float*>(smem_raw + ((sizeof(FusedHeader<NT>) + 15) / 16) * 16);
    float* acc = part + 16 * VEC * 32;

    const int seg_cap = pr.seg_inputs * 16;
    const int i0 = min(g * pr.seg_inputs, pr.n_inputs);
    const int i1 = min(i0 + pr.seg_inputs, pr.n_inputs);

    // ---- phase 1+2: cutoff and selection of this CTA's input segment
    if (batch.mode != kModeMulOnly) {
        int iters = 0;
        const float cutoff = block_find_cutoff<NT>(pr.x, pr.probes, pr.P, pr.target, hdr.cut, &iters);
        const int n = block_select<NT>(pr.x, pr.stats, pr.stats_stride, pr.row0, pr.n_rows_valid,
                                       i0, i1, cutoff, pr.list + (size_t)g * seg_cap, hdr.scan);
        if (threadIdx.x == 0) {
            hdr.my_count = n;
            if (batch.mode == kModeSelectOnly) pr.seg_counts[g] = n;
            if (tile == 0 && g == 0) {
                if (pr.cutoff_out) *pr.cutoff_out = cutoff;
                if (pr.iters_out) *pr.iters_out = iters;
            }
        }
    } else if (threadIdx.x == 0) {
        hdr.my_count = __ldcg(pr.seg_counts + g);
    }
    cluster.sync();  // segment lists (global) and counts (smem) visible cluster-wide

    if (threadIdx.x == 0) {
        int s = 0;
        for (int r = 0; r < G; ++r) {
            hdr.pre[r] = s;
            s += *cluster.map_shared_rank(&hdr.my_count, r);
        }
        hdr.pre[G] = s;
        if (batch.mode != kModeMulOnly && tile == 0 && g == 0 && pr.count_out) *pr.count_out = s;
    }
    __syncthreads();
    if (batch.mode == kModeSelectOnly) {
        cluster.sync();  // peers may still read my_count
        return;
    }

    // ---- phase 3: accumulate this CTA's balanced share of the cluster's selected rows
    const int S = hdr.pre[G];
    const int a = (int)(((long long)S * g) / G);
    const int b = (int)(((long long)S * (g + 1)) / G);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int log2L = pr.log2L;
    const int L = 1 << log2L, P = 32 >> log2L;
    const int rg = lane >> log2L, q = lane & (L - 1);
    const int TW = VEC * L;
    const int c0 = tile * TW + q * VEC;
    const bool col_ok = c0 < pr.cols;

    float* my_acc = acc + (size_t)warp * 16 * VEC * 32 + lane;
#pragma unroll 4
    for (int j = 0; j < 16 * VEC; ++j) my_acc[j * 32] = 0.0f;

    const int32_t* list = pr.list;
    auto row_at = [&](int p) -> int32_t {
        int gs = 0;
        while (gs + 1 < G && p >= hdr.pre[gs + 1]) ++gs;
        return __ldcg(list + (size_t)gs * seg_cap + (p - hdr.pre[gs]));
    };

    const int stride_u = NW * P;
    const int step = stride_u * U;
    const uint16_t* __restrict__ wb = pr.buckets + c0;
    const float* __restrict__ xv_base = pr.x;
    const long long row0 = pr.row0;
    const size_t cols = (size_t)pr.cols;

    int rows[U];
    const int first = a + warp * P;
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int p = first + u * stride_u + rg;
        rows[u] = (p < b) ? row_at(p) : -1;
    }
    for (int s0 = first; s0 < b; s0 += step) {
        typename VecLoad<VEC>::T w[U];
        float xv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (rows[u] >= 0 && col_ok) {
                w[u] = VecLoad<VEC>::load(wb + (size_t)rows[u] * cols);
                xv[u] = __ldg(xv_base + ((rows[u] - row0) >> 4));
            }
        }
        int next[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int p = s0 + step + u * stride_u + rg;
            next[u] = (p < b) ? row_at(p) : -1;
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (rows[u] >= 0 && col_ok) accumulate<VEC>(my_acc, w[u], xv[u]);
#pragma unroll
        for (int u = 0; u < U; ++u) rows[u] = next[u];
    }
    __syncthreads();

    // ---- reduce the lane-private accumulators into this CTA's tile partial
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

    // ---- cluster reduction of the G partial tiles, fixed order (deterministic)
    const int nout = 16 * TW;
    const int per = (nout + G - 1) / G;
    const int o0 = g * per, o1 = min(nout, o0 + per);
    for (int o = o0 + (int)threadIdx.x; o < o1; o += NT) {
        float s = 0.0f;
        for (int r = 0; r < G; ++r) s += cluster.map_shared_rank(part, r)[o];
        const int col = tile * TW + o / 16;
        if (col < pr.cols) {
            const size_t j = (size_t)tile * TW * 16 + o;  // = col*16 + slot
            if (pr.residual) s = pr.residual[j] + s;      // add32 fused (bucketMul.cl:517-520)
            pr.out[j] = s;
        }
    }
    cluster.sync();  // keep `part` alive until every peer has read it
}

// ------------------------------------------------------------------ standalone cutoff

template <int NT>
__global__ void __launch_bounds__(NT) bm_cutoff_kernel(const float* x, const uint16_t* probes, int P,
                                                       int target, float* out, int* iters) {
    __shared__ CutoffShared<NT> sm;
    int it = 0;
    const float c = block_find_cutoff<NT>(x, probes, P, target, sm, &it);
    if (threadIdx.x == 0) {
        out[0] = c;
        if (iters) iters[0] = it;
    }
}

// Concatenates the G segments of a dispatch list (ascending rows).
__global__ void bm_gather_dispatch_kernel(const int32_t* list, const int* seg_counts, int G,
                                          int seg_cap, int32_t* rows_out, int* count_out) {
    __shared__ int pre[kMaxCluster + 1];
    if (threadIdx.x == 0) {
        int s = 0;
        for (int r = 0; r < G; ++r) {
            pre[r] = s;
            s += seg_counts[r];
        }
        pre[G] = s;
        if (count_out) *count_out = s;
    }
    __syncthreads();
    if (!rows_out) return;
    for (int r = 0; r < G; ++r) {
        const int n = pre[r + 1] - pre[r];
        for (int k = threadIdx.x; k < n; k += blockDim.x)
            rows_out[pre[r] + k] = list[(size_t)r * seg_cap + k];
    }
}

__global__ void stats_pack_kernel(const uint16_t* s4, long long rows, uint16_t* s1) {
    for (long long r = blockIdx.x * (long long)blockDim.x + threadIdx.x; r < rows;
         r += (long long)gridDim.x * blockDim.x)
        s1[r] = s4[r * 4 + 3];
}

// ------------------------------------------------------------------ host launch helpers

namespace {

constexpr int kNT = 256;
constexpr int kU = 8;

template <int VEC>
int launch_fused(const BMBatch& b, int G, int n_clusters, cudaStream_t s) {
    auto kern = bm_fused_kernel<VEC, kNT, kU>;
    const size_t smem = fused_smem_bytes<VEC, kNT>();
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(once, [&] {
        attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (attr_err == cudaSuccess)
            attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    });
    if (attr_err != cudaSuccess) return cuda_fail(attr_err, "cudaFuncSetAttribute(bm_fused)");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(n_clusters * G));
    cfg.blockDim = dim3(kNT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)G;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    IAM_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, b));
    return IAM_OK;
}

int env_int(const char* name, int dflt) {
    const char* v = getenv(name);
    return (v && *v) ? atoi(v) : dflt;
}

}  // namespace

int bm_max_active_clusters(int vec, int G) {
    static std::mutex mu;
    static int cache[2][kMaxCluster + 1] = {};
    std::lock_guard<std::mutex> lk(mu);
    const int vi = vec == 8 ? 0 : 1;
    if (cache[vi][G]) return cache[vi][G];
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)G;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.blockDim = dim3(kNT);
    cfg.gridDim = dim3((unsigned)(G * 64));
    int n = 0;
    cudaError_t e;
    if (vec == 8) {
        auto kern = bm_fused_kernel<8, kNT, kU>;
        cfg.dynamicSmemBytes = fused_smem_bytes<8, kNT>();
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cfg.dynamicSmemBytes);
        cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    } else {
        auto kern = bm_fused_kernel<1, kNT, kU>;
        cfg.dynamicSmemBytes = fused_smem_bytes<1, kNT>();
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cfg.dynamicSmemBytes);
        cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    }
    if (e != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = 1;
    }
    cache[vi][G] = n;
    return n;
}

int bm_default_cluster() {
    const int g = env_int("IAM_BM_CLUSTER", 8);
    return (g == 2 || g == 4 || g == 8 || g == 16) ? g : 8;
}

// Fills the tiling of each problem (log2L, n_tiles, cluster_begin) so the whole batch is
// about one wave of resident clusters, giving wider tiles to problems with more work.
void bm_plan_tiles(BMBatch& b, int vec, int G, int max_clusters) {
    double work_total = 0.0;
    for (int i = 0; i < b.nprob; ++i) work_total += (double)b.p[i].cols * b.p[i].n_rows_valid;
    const int forced = env_int("IAM_BM_LOG2L", -1);
    int begin = 0;
    for (int i = 0; i < b.nprob; ++i) {
        BMProblem& p = b.p[i];
        const double share = work_total > 0 ? max_clusters * ((double)p.cols * p.n_rows_valid) / work_total : 1.0;
        int best = 5;
        if (forced >= 0 && forced <= 5) {
            best = forced;
        } else {
            for (int l2 = 5; l2 >= 0; --l2) {
                const int tw = vec << l2;
                const int tiles = (p.cols + tw - 1) / tw;
                best = l2;
                if (tiles >= share) break;  // first (widest) tiling that fills its share
            }
            // never narrower than needed to cover >1 lane group per row when cols is tiny
        }
        const int tw = vec << best;
        p.log2L = best;
        p.n_tiles = (p.cols + tw - 1) / tw;
        p.cluster_begin = begin;
        begin += p.n_tiles;
    }
}

int bm_total_clusters(const BMBatch& b) {
    int n = 0;
    for (int i = 0; i < b.nprob; ++i) n += b.p[i].n_tiles;
    return n;
}

int bm_launch(const BMBatch& b, int vec, int G, cudaStream_t s) {
    const int n = b.mode == kModeSelectOnly ? b.nprob : bm_total_clusters(b);
    if (vec == 8) return launch_fused<8>(b, G, n, s);
    return launch_fused<1>(b, G, n, s);
}

int bm_launch_cutoff(const float* x, const uint16_t* probes, int P, int target, float* out, int* iters,
                     cudaStream_t s) {
    bm_cutoff_kernel<256><<<1, 256, 0, s>>>(x, probes, P, target, out, iters);
    IAM_CUDA_TRY(cudaGetLastError());
    return IAM_OK;
}

int bm_launch_gather(const int32_t* list, const int* seg_counts, int G, int seg_cap, int32_t* rows_out,
                     int* count_out, cudaStream_t s) {
    bm_gather_dispatch_kernel<<<1, 256, 0, s>>>(list, seg_counts, G, seg_cap, rows_out, count_out);
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
