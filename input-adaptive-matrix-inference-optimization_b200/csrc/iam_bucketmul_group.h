// iam_bucketmul_group.h -- host-side description of a launch of the range bucketMul kernel.
//
// The fused bucketMul (bucketMul.cl:68-497: cutoff, row selection, accumulation, integrate)
// as ONE launch of at most one CTA per SM: CTA (tile, range) owns a tile of bucket columns
// and a contiguous range of inputs.  It finds the cutoff (every CTA, identical bits), selects
// its range's bucket rows (for monotone row statistics a per-input prefix), accumulates them
// for its columns and writes a partial; after a grid-wide barrier the CTAs add the partials
// in range order (deterministic; see iam_bucketmul_group.cu).
#pragma once

#include <cuda_runtime.h>

#include "iam_tp.h"
#include <stdint.h>

namespace iam {

constexpr int kGMaxProblems = 3;
// Diagnostics: int64 slots per CTA of a traced launch: globaltimer stamps (ns) [0] start,
// [1] cutoff inputs loaded, [8] values binned, [9] bins scanned, [10] values sorted by bin,
// [2] cutoff done, [3] selection done, [4] accumulation done, [5] partial written, [11]
// barrier passed, [6] end; counts [7] rows of the range, [12] largest bin, [13] bisection
// steps, [14] stats copy state (0 landed or not staged, -1 late).
constexpr int kTraceSlots = 16;

struct BGProblem {
    const uint16_t* buckets;  // [rows held][cols]
    const uint16_t* stats;    // [rows][stats_stride] (all rows of the expert, every rank)
    int stats_stride;         // 4 (file layout) or 1 (packed channel 3)
    const uint16_t* probes;   // already offset by expert_no * 4096
    const float* x;           // input (plain), RMS source (kXRms) or gate (kXSilu)
    const float* x2;          // up (kXSilu)
    const uint16_t* gain;     // RMS gain (kXRms)
    float norm_eps;           // kXRms
    int norm_n;               // kXRms: length of the normalised vector
    float* out;               // [16 * cols]
    const float* residual;    // optional: out = residual + sum (add32, bucketMul.cl:517-520)
    float* cutoff_out;        // optional
    int* count_out;           // optional: selected rows of the inputs held
    int* iters_out;           // optional: bisection steps
    float* partials;          // scratch [n_ranges][16 * cols] + n_ranges ints (bg_scratch_floats)
    float* x_capture;         // optional diagnostics: receives x[in_begin, in_begin + n_in) as used
    long long row0;           // expert row offset (expertSize * expertNo)
    long long bucket_row0;    // absolute row held by buckets[0] (row0 + 16 * in_begin)
    int n_rows_valid;         // rows of the expert considered: min(expert_size, 16 * in_dim)
    int in_begin;             // first input held (row-parallel shards), else 0
    int n_in;                 // inputs held
    int cols;                 // bucket columns held
    const uint16_t* dense;    // dense launches: [16 * cols][n_in] the weights at their output
                              // positions, low 4 bits = the weight's bucket row (rank) r
    int dense_rows;           // dense launches: output rows per tile (a multiple of 16)
    int full_in;              // inputs of the whole matrix over all ranks (0: n_in)
    int full_cols;            // bucket columns of the whole matrix over all ranks (0: cols)
    int fixed_ranges;         // > 0: input ranges of the whole matrix, fixed (must divide full_in)
    int P;                    // probes used by the cutoff: min(in_dim, 4096)
    int target;               // P - quantile
    int vec;                  // columns per lane (1, 2 or 4; bg_choose_shape)
    int n_ranges;             // input ranges (bg_choose_shape)
    int range_max;            // most inputs in one range (bg_plan)
    int n_tiles;              // column tiles (bg_plan)
    int cta_begin;            // first CTA of this problem in the launch (bg_plan)
    int out_begin;            // global index of out[0] (column-parallel shards; tp_push)
};

struct BGBatch {
    BGProblem p[kGMaxProblems];
    int nprob;
    int xmode;                // BMXMode (iam_bucketmul_launch.h)
    int rowl;                 // row lanes per warp: 1 or 2
    int stage_stats;          // bulk-copy each range's packed stats into shared memory first
    int pdl;                  // launched with programmatic stream serialization
    int dense;                // stream the dense copies (every weight, selected by rank) instead
                              // of the selected bucket rows: same selection, register accumulators
    int tp_fused;             // tensor-parallel row-parallel launch (o, down): every range partial
                              // also goes to each peer's mailbox (tp.fused_off), and the range
                              // reduction adds the ranges of every rank in range order
    TpWindow tp;              // tp_fused / tp_push / tp_wait: the peers' windows
    int tp_push;              // 1 + kind: outputs at global index out_begin + o below push_limit
    int push_limit;           // also go to every peer's mailbox of that kind (iam_tp_push.cuh),
                              // problem i at offset i * tp.pmb_ffn; 0: none
    int tp_wait;              // 1 + kind: x outside this rank's inputs [in_begin, in_begin + n_in)
                              // is read from this rank's mailbox of that kind (x2 at + pmb_ffn)
    int partials_only;        // write each range's partial (and its row count) and stop: the
                              // ranges are summed by the tensor-parallel exchange (tp_gather_reduce)
    unsigned* barrier;        // scratch: 4 words {arrivals, generation, error, -}, zeroed once
    long long* trace;         // optional: kTraceSlots int64 per CTA (blockIdx.x < trace_cap)
    int trace_cap;
};

// Floats of partial scratch a problem needs for n_ranges ranges of cols bucket columns.
inline size_t bg_scratch_floats(int n_ranges, int cols) {
    return (size_t)n_ranges * 16 * (size_t)cols + (size_t)n_ranges + 16;
}
// Most input ranges any plan uses (partial scratch can be sized with it).
constexpr int kMaxRanges = 64;

// Row lanes, columns per lane, input ranges and stats staging of a batch.  Each output's sum
// order depends only on the row lanes and the input ranges, and both follow from the whole
// matrices (full_cols, full_in), so every tensor-parallel shard adds its outputs in the order
// one GPU does: 1 row lane per warp for matrices of 512 or more bucket columns, else 2; input
// ranges fixed_ranges, or as many per problem (in proportion to its work) as one wave of one
// CTA per SM holds on one GPU.  The shard then takes its share of those ranges (row-parallel
// shards hold whole ranges) and the widest tiles (up to 4 columns per lane) that still fill
// the SMs.
void bg_choose_shape(BGBatch& b);
// Input ranges of a dense launch over a whole matrix of full_in inputs (0: no dense shape).
int bg_dense_ranges(int full_in, bool row_parallel);
// Fills n_tiles, range_max and cta_begin of every problem; returns the CTAs of the launch.
int bg_plan(BGBatch& b);
size_t bg_smem_bytes(const BGBatch& b);
int bg_launch(const BGBatch& b, cudaStream_t s);

}  // namespace iam
