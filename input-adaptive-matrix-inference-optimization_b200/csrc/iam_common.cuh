// iam_common.cuh -- shared device helpers and host error plumbing for libiamb200.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>

#include "../../include/iam_b200.h"

#define IAM_DEV __device__ __forceinline__

namespace iam {

constexpr int kProbes = IAM_PROBES_COUNT;  // bucketMul.cl:18
constexpr float kCutoffScale = 100000.0f;  // bucketMul.cl:17
constexpr int kMaxIters = 20;              // bucketMul.cl:148

// Asks the L2 to fetch [p, p + bytes) (cp.async.bulk.prefetch.L2; p 16-byte aligned, bytes a
// multiple of 16).  No registers, no shared memory, no completion to wait for.
IAM_DEV void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(__cvta_generic_to_global(p)), "r"(bytes)
                 : "memory");
}

// Programmatic dependent launch: a kernel launched with programmatic stream serialization
// may start while its predecessor still runs; pdl_wait() returns once the predecessor grid
// has completed and its writes are visible (immediately when launched without the
// attribute).  pdl_trigger() lets the successor launch early.
IAM_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
IAM_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Exact fp16 -> fp32 of raw bits (the 4 slot bits stay part of the value, as in
// bucketMul.cl:430-431 where the unmasked packed weight is the multiplicand).
IAM_DEV float h2f(uint32_t bits) { return __half2float(__ushort_as_half((unsigned short)bits)); }

// 1e5 * |x * s| with both multiplies rounded separately (bucketMul.cl:110, :378).
IAM_DEV float importance(float x, float s) {
    return __fmul_rn(kCutoffScale, fabsf(__fmul_rn(x, s)));
}

// Host-side: runs `set` (e.g. cudaFuncSetAttribute calls) once for the current device; CUDA
// function attributes belong to a device's context, so a process that drives several devices
// sets them on each.  Concurrent first calls may both run `set` (idempotent).
template <class F>
cudaError_t once_per_device(std::atomic<unsigned long long>& done, F&& set) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = 1ull << (dev & 63);
    if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
    e = set();
    if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

// Host-side: per-thread last error message.
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

}  // namespace iam

// cudaLaunchKernelEx with programmatic stream serialization when `pdl` is set (the kernel
// must call pdl_wait() before it touches what earlier kernels of the stream write).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                             Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

#define IAM_CUDA_TRY(expr)                                          \
    do {                                                            \
        cudaError_t _e = (expr);                                    \
        if (_e != cudaSuccess) return ::iam::cuda_fail(_e, #expr);  \
    } while (0)
