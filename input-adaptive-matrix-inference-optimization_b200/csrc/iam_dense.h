// iam_dense.h -- the dense tensor-core path (tcgen05): batched products with fp16 weights.
//
// Y[t][o] = sum_i W[o][i] * X[t][i] for tokens t < n: the reference's dense GEMV kernels
// (basicMul / basicMul2, matrix.cl:80-127) batched over the tokens of a prompt.  W is a
// dense fp16 matrix [out][in] (row stride = in); X arrives as fp32 and is split into two fp16
// halves (hi = fp16(x), lo = fp16(x - hi)) so that the tensor cores, whose f16 kind needs both
// operands in fp16, still see ~22 bits of every activation.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace iam {

constexpr int kDenseBT = 128;      // tokens per tile: the MMA's M (operand A = activations)
constexpr int kDenseBW = 256;      // weight rows (outputs) per tile: the MMA's N (operand B = W)
constexpr int kDenseBK = 64;       // K per pipeline stage: one 128-byte swizzle row of fp16
constexpr int kDenseMaxSplit = 8;  // K slices of one tile at most (deterministic second pass)
constexpr int kDenseMaxTokens = 65535;  // tokens per call (the element-wise passes grid them in y)

// Split-K scratch (floats) that covers every split dense_auto_split picks on `sms` SMs.
inline size_t dense_partial_floats(int sms) { return (size_t)sms * kDenseBT * kDenseBW; }

struct DenseProblem {
    const uint16_t* w;      // [m][ldw] fp16, K contiguous (ldw >= k, ldw % 8 == 0, 16-byte aligned base)
    int m, k, ldw;
    const uint16_t* x_hi;   // [n][k] fp16 (row stride k)
    const uint16_t* x_lo;   // [n][k] fp16; null: activations are fp16 already (hi only)
    int n;
    float* y;               // [n][ldy]: columns [0, m) written
    int ldy;
    const float* residual;  // [n][ldr] added to the product (may alias y); null: none
    int ldr;
    float* partial;         // split-K scratch: split * n * m floats (needed when split > 1)
    int split;              // K slices (1 = none); clamped to the K blocks
    unsigned* err;          // device word set when a pipeline wait gave up (may be null)
    // SiLU epilogue (silu_out_hi != null): W's rows come in blocks of 256 = 128 gate rows then
    // the 128 up rows of the same FFN columns; instead of y the tile writes
    // a = up * gate / (1 + exp(-gate)) of its 128 FFN columns as fp16 hi / lo [n][ld_silu].
    // Needs m % 256 == 0 and no K split.
    uint16_t* silu_out_hi;
    uint16_t* silu_out_lo;
    int ld_silu;
};

// Splits fp32 X [n][k] (row stride ldx) into fp16 hi / lo [n][k].
int dense_split(const float* x, int n, int k, int ldx, uint16_t* hi, uint16_t* lo, cudaStream_t s,
                bool pdl = false);
// The split the launcher would pick for this problem on an SM count (tiles x split ~ SMs).
int dense_auto_split(int m, int k, int n, int sms);
int dense_gemm(const DenseProblem& p, cudaStream_t s, bool pdl = false);
// Dense fp16 matrix W'[16*c + slot][i] from the bucket layout buckets[16*in][cols]: the
// packed word (value with its slot in the low 4 bits) lands at its original position, which
// is the multiplicand bucketMul uses when every bucket row is selected.
// rows_per_block > 0 places dense row o at (o / rows_per_block) * block_pitch + o % rows_per_block
// (used to interleave the gate and up matrices for the SiLU epilogue).  tag_rank: each weight's
// low 4 bits hold its bucket row (rank within its group of 16) instead of its slot, which the
// position already gives (the decode's dense stream selects weights by rank).
int dense_unpack(const uint16_t* buckets, int in_dim, int cols, uint16_t* w, int ldw, cudaStream_t s,
                 int rows_per_block = 0, int block_pitch = 0, bool tag_rank = false);

}  // namespace iam
