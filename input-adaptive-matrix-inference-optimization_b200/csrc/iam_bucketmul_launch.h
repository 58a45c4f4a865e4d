// iam_bucketmul_launch.h -- host-side description of a fused bucketMul launch.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace iam {

constexpr int kMaxProblems = 4;
constexpr int kMaxCluster = 16;

enum BMMode { kModeFused = 0, kModeSelectOnly = 1, kModeMulOnly = 2 };

// One bucketMul (one weight matrix times one input vector).
struct BMProblem {
    const uint16_t* buckets;  // [R_total][cols] (full tensor; rows are absolute)
    const uint16_t* stats;    // [R_total][stats_stride]
    const uint16_t* probes;   // already offset by expert_no * 4096
    const float* x;           // [in_dim]
    float* out;               // [16 * cols]
    const float* residual;    // optional: out = residual + result
    int32_t* list;            // dispatch list scratch: G segments of seg_inputs*16 rows
    int* seg_counts;          // [G] segment counts (select-only writes, mul-only reads)
    float* cutoff_out;        // optional
    int* count_out;           // optional
    int* iters_out;           // optional
    long long row0;           // expert row offset (expertSize * expertNo)
    int n_rows_valid;         // rows considered: min(expert_size, 16*in_dim)
    int n_inputs;             // ceil(n_rows_valid / 16)
    int cols;                 // bucket columns C
    int stats_stride;         // 4 (file layout) or 1 (packed channel 3)
    int P;                    // probes used by the cutoff: min(in_dim, 4096)
    int target;               // P - quantile
    int seg_inputs;           // inputs per cluster segment
    int log2L;                // lanes per row segment = 1 << log2L
    int n_tiles;              // column tiles (clusters) of this problem
    int cluster_begin;        // index of its first cluster in the launch
};

struct BMBatch {
    BMProblem p[kMaxProblems];
    int nprob;
    int mode;
};

int bm_default_cluster();
int bm_max_active_clusters(int vec, int G);
void bm_plan_tiles(BMBatch& b, int vec, int G, int max_clusters);
int bm_total_clusters(const BMBatch& b);
int bm_launch(const BMBatch& b, int vec, int G, cudaStream_t s);
int bm_launch_cutoff(const float* x, const uint16_t* probes, int P, int target, float* out, int* iters,
                     cudaStream_t s);
int bm_launch_gather(const int32_t* list, const int* seg_counts, int G, int seg_cap, int32_t* rows_out,
                     int* count_out, cudaStream_t s);
int bm_launch_stats_pack(const uint16_t* s4, long long rows, uint16_t* s1, cudaStream_t s);
int bucketize_launch(const uint16_t* w, int out_dim, int in_dim, uint16_t* buckets, uint16_t* stats4,
                     uint16_t* stats1, uint16_t* probes, cudaStream_t s);

// Target count of the cutoff search: P - int((P-1)*(1-effort)) (bucket_mul.hpp:164).
inline int bm_target(float effort, int P) {
    const int quantile = (int)((double)(P - 1) * (1.0 - (double)effort));
    return P - quantile;
}

}  // namespace iam
