// iam_common.cuh -- shared device helpers and host error plumbing for libiamb200.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/iam_b200.h"

#define IAM_DEV __device__ __forceinline__

namespace iam {

constexpr int kProbes = IAM_PROBES_COUNT;  // bucketMul.cl:18
constexpr float kCutoffScale = 100000.0f;  // bucketMul.cl:17
constexpr int kMaxIters = 20;              // bucketMul.cl:148

// Exact fp16 -> fp32 of raw bits (the 4 slot bits stay part of the value, as in
// bucketMul.cl:430-431 where the unmasked packed weight is the multiplicand).
IAM_DEV float h2f(uint32_t bits) { return __half2float(__ushort_as_half((unsigned short)bits)); }

// 1e5 * |x * s| with both multiplies rounded separately (bucketMul.cl:110, :378).
IAM_DEV float importance(float x, float s) {
    return __fmul_rn(kCutoffScale, fabsf(__fmul_rn(x, s)));
}

// Host-side: per-thread last error message.
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

}  // namespace iam

#define IAM_CUDA_TRY(expr)                                          \
    do {                                                            \
        cudaError_t _e = (expr);                                    \
        if (_e != cudaSuccess) return ::iam::cuda_fail(_e, #expr);  \
    } while (0)
