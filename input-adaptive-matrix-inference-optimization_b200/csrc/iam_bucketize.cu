// iam_bucketize.cu -- GPU restatement of the reference's weight preprocessing
// (preprocess_layer_fixed_gpu.py:110-242, bucketize_fp16_packed), so a synthetic model of
// Mistral-7B size can be laid out on the device in seconds.  Output is bit-identical to
// the reference function: ties in |w| are ordered by lower original slot (what the
// reference's torch.argsort produced on the recorded tie fixture), stats use numpy's
// pairwise float32 summation (np.mean over the contiguous axis) and probes numpy's
// sequential float32 summation (np.mean over the strided axis of the transposed view).
#include "iam_bucketmul_launch.h"
#include "iam_common.cuh"

namespace iam {

// One thread per bucket (input i, column c): sort the 16 outputs c*16..c*16+15 of input i
// by |w| descending (composite key -> ties keep slot order) and write the 16 rank rows.
__global__ void bucketize_sort_kernel(const uint16_t* __restrict__ W, int M, int N,
                                      uint16_t* __restrict__ buckets) {
    const int C = M / 16;
    const long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (t >= (long long)C * N) return;
    const int c = (int)(t % C), i = (int)(t / C);
    uint32_t key[16];
#pragma unroll
    for (int s = 0; s < 16; ++s) {
        const uint32_t h = W[(size_t)(c * 16 + s) * N + i];
        key[s] = ((0x7fffu - (h & 0x7fffu)) << 4) | (uint32_t)s;
    }
#pragma unroll
    for (int k = 2; k <= 16; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
#pragma unroll
            for (int a = 0; a < 16; ++a) {
                const int bidx = a ^ j;
                if (bidx > a) {
                    const bool up = (a & k) == 0;
                    const uint32_t ka = key[a], kb = key[bidx];
                    if ((ka > kb) == up) {
                        key[a] = kb;
                        key[bidx] = ka;
                    }
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) {
        const uint32_t s = key[r] & 15u;
        const uint32_t h = W[(size_t)(c * 16 + s) * N + i];
        buckets[((size_t)i * 16 + r) * C + c] = (uint16_t)((h & 0xfff0u) | s);  // :196
    }
}

// |value| of bucket row `row`, column c, as the fp32 the reference averaged (:212).
struct RowAbs {
    const uint16_t* W;
    const uint16_t* brow;
    int N, i;
    IAM_DEV float operator()(int c) const {
        const uint32_t s = brow[c] & 15u;
        return fabsf(h2f(W[(size_t)(c * 16 + s) * N + i]));
    }
};

// numpy's float32 pairwise summation of f(off .. off+n-1) (blocks of 8 partial sums
// below 128 elements, halving split rounded to a multiple of 8 above).
template <class F>
__device__ float np_pairwise_sum(const F& f, int off, int n) {
    if (n < 8) {
        float r = 0.0f;
        for (int k = 0; k < n; ++k) r = __fadd_rn(r, f(off + k));
        return r;
    }
    if (n <= 128) {
        float r[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) r[j] = f(off + j);
        int k = 8;
        for (; k < n - (n % 8); k += 8) {
#pragma unroll
            for (int j = 0; j < 8; ++j) r[j] = __fadd_rn(r[j], f(off + k + j));
        }
        float res = __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[1]), __fadd_rn(r[2], r[3])),
                              __fadd_rn(__fadd_rn(r[4], r[5]), __fadd_rn(r[6], r[7])));
        for (; k < n; ++k) res = __fadd_rn(res, f(off + k));
        return res;
    }
    int n2 = n / 2;
    n2 -= n2 % 8;
    return __fadd_rn(np_pairwise_sum(f, off, n2), np_pairwise_sum(f, off + n2, n - n2));
}

__global__ void bucketize_stats_kernel(const uint16_t* __restrict__ W, int M, int N,
                                       const uint16_t* __restrict__ buckets, uint16_t* stats4,
                                       uint16_t* stats1) {
    const int C = M / 16;
    const long long row = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (row >= 16LL * N) return;
    RowAbs f{W, buckets + row * C, N, (int)(row / 16)};
    const float mean = __fdiv_rn(np_pairwise_sum(f, 0, C), (float)C);
    const uint16_t h = __half_as_ushort(__float2half_rn(mean));
    if (stats4) {
        uint2 v;
        v.x = (uint32_t)h | ((uint32_t)h << 16);
        v.y = v.x;
        *reinterpret_cast<uint2*>(stats4 + row * 4) = v;  // all 4 channels (:217-221)
    }
    if (stats1) stats1[row] = h;
}

__global__ void bucketize_probes_kernel(const uint16_t* __restrict__ W, int M, int N,
                                        uint16_t* __restrict__ probes) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= N) return;
    float s = 0.0f;
    for (int j = 0; j < M; ++j) s = __fadd_rn(s, fabsf(h2f(W[(size_t)j * N + i])));
    probes[i] = __half_as_ushort(__float2half_rn(__fdiv_rn(s, (float)M)));  // :154
}

int bucketize_launch(const uint16_t* w, int out_dim, int in_dim, uint16_t* buckets, uint16_t* stats4,
                     uint16_t* stats1, uint16_t* probes, cudaStream_t s) {
    const long long nb = (long long)(out_dim / 16) * in_dim;
    bucketize_sort_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, s>>>(w, out_dim, in_dim, buckets);
    IAM_CUDA_TRY(cudaGetLastError());
    if (stats4 || stats1) {
        const long long rows = 16LL * in_dim;
        bucketize_stats_kernel<<<(unsigned)((rows + 127) / 128), 128, 0, s>>>(w, out_dim, in_dim, buckets,
                                                                             stats4, stats1);
        IAM_CUDA_TRY(cudaGetLastError());
    }
    if (probes) {
        bucketize_probes_kernel<<<(in_dim + 127) / 128, 128, 0, s>>>(w, out_dim, in_dim, probes);
        IAM_CUDA_TRY(cudaGetLastError());
    }
    return IAM_OK;
}

}  // namespace iam
