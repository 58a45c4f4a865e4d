// iam_bucketmul_launch.h -- host-side description of a fused bucketMul launch.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace iam {

constexpr int kMaxProblems = 4;
constexpr int kMaxCluster = 16;
constexpr int kMaxSplits = 64;
constexpr int kMaxSegInputs = 4096;  // 16-bit local row offsets

enum BMMode { kModeFused = 0, kModeSelectOnly = 1, kModeMulOnly = 2 };

// How the bucketMul input x is produced (all CTAs derive bit-identical x).
enum BMXMode {
    kXPlain = 0,  // x = x[i]
    kXRms = 1,    // x = rmsNorm32fast(x)[i] * gain[i]        (aux.cl:156-196, :434-440)
    kXSilu = 2    // x = up[i] * x[i] / (1 + exp(-x[i])), x = gate  (matrix.cl:27-32)
};

// One bucketMul (one weight matrix times one input vector).
//
// Grid layout of a problem: n_tiles column tiles x n_split row splits clusters of G CTAs.
// Fused mode splits the inputs [in_begin, n_inputs) into n_split ranges; mul-only mode
// splits the positions of the compact dispatch list.  With n_split > 1 every cluster
// writes its partial tile to `partials` and the last cluster to finish a slice of the tile
// (slice_ctr) adds the n_split partials in split order, so results stay deterministic.
struct BMProblem {
    const uint16_t* buckets;  // [R_total][cols]; rows are absolute indices minus bucket_row0
    const uint16_t* stats;    // [R_total][stats_stride]
    const uint16_t* probes;   // already offset by expert_no * 4096
    const float* x;           // input (plain), RMS source (kXRms) or gate (kXSilu)
    const float* x2;          // up (kXSilu)
    const uint16_t* gain;     // RMS gain (kXRms)
    float norm_eps;           // kXRms
    int norm_n;               // kXRms: length of the normalised vector
    float* out;               // [16 * cols]
    const float* residual;    // optional: out = residual + result (add32, bucketMul.cl:517-520)
    int32_t* list;            // compact dispatch list (select-only writes, mul-only reads)
    int* sel_total;           // selected-row total (select-only writes, mul-only reads)
    float* partials;          // [n_split][16 * cols] when n_split > 1
    int* slice_ctr;           // [n_tiles * G] zero-initialised arrival counters (self-resetting)
    int* split_sel;           // [n_split] selected rows per split (count_out when n_split > 1)
    float* cutoff_out;        // optional
    int* count_out;           // optional
    int* iters_out;           // optional
    long long* dbg;           // optional per-phase globaltimer stamps (cluster 0, CTA 0)
    long long* trace;         // optional: 8 stamps per CTA (blockIdx.x < trace_cap), see iam_bucketmul_trace
    int trace_cap;
    long long row0;           // expert row offset (expertSize * expertNo)
    long long bucket_row0;    // absolute row held by buckets[0] (0, or the first row of a shard)
    int in_begin;             // first input of this shard (row-parallel tensor parallelism)
    int n_rows_valid;         // rows of the expert considered: min(expert_size, 16*in_dim)
    int n_inputs;             // inputs end: ceil(n_rows_valid / 16)
    int cols;                 // bucket columns C of the buckets tensor
    int stats_stride;         // 4 (file layout) or 1 (packed channel 3)
    int P;                    // probes used by the cutoff: min(in_dim, 4096)
    int target;               // P - quantile
    int seg_inputs;           // inputs per CTA (fused: per CTA of a split)
    int log2L;                // lanes per row segment = 1 << log2L
    int n_tiles;              // column tiles of this problem
    int n_split;              // row splits (clusters per tile)
    int cluster_begin;        // index of its first cluster in the launch
};

struct BMBatch {
    BMProblem p[kMaxProblems];
    int nprob;
    int mode;
    int xmode;
    int pdl;  // launched with programmatic stream serialization (waits on its predecessor in-kernel)
    int cluster;  // cluster size the plan was made for (0: the caller's)
};

// Scratch a problem needs beyond its inputs and outputs (device memory the caller owns).
struct BMScratch {
    int32_t* list;     // >= n_rows_valid rows (select-only / mul-only modes)
    int* sel_total;    // 1 int
    float* partials;   // >= kMaxSplits * 16 * cols floats
    int* slice_ctr;    // >= n_tiles * G ints, zero-initialised once
    int* split_sel;    // >= kMaxSplits ints
};

int bm_default_cluster();
int bm_max_active_clusters(int vec, int G);
size_t bm_smem_bytes(int vec, int seg_inputs);
void bm_plan(BMBatch& b, int vec, int G, int max_clusters, int max_splits = kMaxSplits);
int bm_total_clusters(const BMBatch& b);
int bm_launch(const BMBatch& b, int vec, int G, cudaStream_t s);
int bm_launch_cutoff(const float* x, const uint16_t* probes, int P, int target, float* out, int* iters,
                     cudaStream_t s);
int bm_launch_stats_pack(const uint16_t* s4, long long rows, uint16_t* s1, cudaStream_t s);
int bucketize_launch(const uint16_t* w, int out_dim, int in_dim, uint16_t* buckets, uint16_t* stats4,
                     uint16_t* stats1, uint16_t* probes, cudaStream_t s);

// Target count of the cutoff search: P - int((P-1)*(1-effort)) (bucket_mul.hpp:164).
inline int bm_target(float effort, int P) {
    const int quantile = (int)((double)(P - 1) * (1.0 - (double)effort));
    return P - quantile;
}

}  // namespace iam
