// iam_capi.cu -- C ABI entry points of libiamb200.so for the bucketMul operator.
// Declarations and the reference interface each one replaces: include/iam_b200.h.
#include <cmath>
#include <cstdlib>
#include <mutex>
#include <cstring>
#include <string>

#include "iam_bucketmul_group.h"
#include "iam_bucketmul_launch.h"
#include "iam_common.cuh"

namespace iam {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
    return e == cudaErrorMemoryAllocation ? IAM_ERR_NOMEM : IAM_ERR_CUDA;
}

}  // namespace iam

using namespace iam;

struct iam_bucketmul_s {
    int device = 0;
    int32_t* list = nullptr;  // compact dispatch list scratch
    size_t list_cap = 0;      // capacity in rows
    float* partials = nullptr;  // split partial tiles
    size_t partials_cap = 0;    // capacity in floats
    int* ctr = nullptr;         // slice arrival counters (zeroed once, self-resetting)
    float* cutoff = nullptr;    // device scalar
    int* ints = nullptr;        // device scalars: [0] count, [1] iters, [2] selected total, [8..] split counts
    float* gpartials = nullptr;  // range-kernel partials (iam_bucketmul_full)
    size_t gpartials_cap = 0;    // capacity in floats
    unsigned* bar = nullptr;     // range-kernel grid barrier words (zeroed once)
    // dispatch recorded by iam_bucketmul_calc_dispatch (consumed by iam_bucketmul_mul)
    bool have_dispatch = false;
    BMProblem disp{};
    int disp_G = 8;
    int disp_bucket_cols = 0;
    long long* dbg = nullptr;  // optional phase stamps
    long long* trace = nullptr;  // optional per-CTA stamps
    int trace_cap = 0;
};

namespace {

int ensure_list(iam_bucketmul_s* h, size_t rows) {
    if (rows <= h->list_cap) return IAM_OK;
    if (h->list) {
        IAM_CUDA_TRY(cudaFree(h->list));
        h->list = nullptr;
        h->list_cap = 0;
    }
    IAM_CUDA_TRY(cudaMalloc(&h->list, rows * sizeof(int32_t)));
    h->list_cap = rows;
    return IAM_OK;
}

bool effort_ok(float e) { return std::isfinite(e) && e > 0.0f && e <= 1.0f; }

// Fills the selection part of a problem (shared by calc_dispatch and full).
int fill_problem(iam_bucketmul_s* h, BMProblem& p, int G, const float* x, const uint16_t* stats,
                 int stats_stride, const uint16_t* probes, int expert_no, int in_dim, int bucket_cols,
                 int expert_size, float effort) {
    if (!x || !stats || !probes) return fail(IAM_ERR_ARG, "bucketmul: null input/stats/probes pointer");
    if (in_dim <= 0 || bucket_cols <= 0 || expert_size <= 0 || expert_no < 0)
        return fail(IAM_ERR_ARG, "bucketmul: in_dim, bucket_cols, expert_size must be > 0, expert_no >= 0");
    if (stats_stride != 1 && stats_stride != 4)
        return fail(IAM_ERR_ARG, "bucketmul: stats_stride must be 1 (packed) or 4 (file layout)");
    if (!effort_ok(effort)) return fail(IAM_ERR_ARG, "bucketmul: effort must be in (0, 1]");
    memset(&p, 0, sizeof(p));
    p.x = x;
    p.stats = stats;
    p.stats_stride = stats_stride;
    p.probes = probes + (size_t)expert_no * IAM_PROBES_COUNT;  // bucketMul.cl:103
    p.row0 = (long long)expert_size * expert_no;               // bucketMul.cl:363
    p.n_rows_valid = expert_size < 16 * in_dim ? expert_size : 16 * in_dim;
    p.n_inputs = (p.n_rows_valid + 15) / 16;
    p.cols = bucket_cols;
    p.P = in_dim < IAM_PROBES_COUNT ? in_dim : IAM_PROBES_COUNT;
    p.target = bm_target(effort, p.P);
    p.seg_inputs = (p.n_inputs + G - 1) / G;
    if ((p.row0 + p.n_rows_valid) * (long long)bucket_cols >= (1LL << 31))
        return fail(IAM_ERR_UNSUPPORTED, "bucketmul: rows * bucket_cols must stay below 2^31 elements");
    int rc = ensure_list(h, (size_t)p.n_rows_valid);
    if (rc) return rc;
    p.list = h->list;
    p.sel_total = h->ints + 2;
    p.split_sel = h->ints + 8;
    p.slice_ctr = h->ctr;
    p.dbg = h->dbg;
    p.trace = h->trace;
    p.trace_cap = h->trace_cap;
    const size_t need = (size_t)kMaxSplits * 16 * (size_t)bucket_cols;
    if (need > h->partials_cap) {
        if (h->partials) IAM_CUDA_TRY(cudaFree(h->partials));
        h->partials = nullptr;
        h->partials_cap = 0;
        IAM_CUDA_TRY(cudaMalloc(&h->partials, need * sizeof(float)));
        h->partials_cap = need;
    }
    p.partials = h->partials;
    return IAM_OK;
}

constexpr int kCtrSlots = 4096;

// The slice counters must cover n_tiles * G of the problem.
bool plan_fits(const BMBatch& b, int G) {
    for (int i = 0; i < b.nprob; ++i)
        if (b.p[i].n_tiles * G > kCtrSlots) return false;
    return true;
}

// Vector width: 4 columns per lane (IAM_BM_VEC may pick 8 or 1), lowered to what every
// problem's column count and alignment allow.
int pick_vec(const BMBatch& b) {
    int vec = 4;
    const char* env = getenv("IAM_BM_VEC");
    if (env && (atoi(env) == 8 || atoi(env) == 4 || atoi(env) == 1)) vec = atoi(env);
    for (int i = 0; i < b.nprob; ++i) {
        const BMProblem& p = b.p[i];
        const uintptr_t a = reinterpret_cast<uintptr_t>(p.buckets);
        while (vec > 1 && (p.cols % vec != 0 || (a & (uintptr_t)(2 * vec - 1)) != 0)) vec = vec == 8 ? 4 : 1;
    }
    return vec;
}

}  // namespace

extern "C" {

const char* iam_version(void) { return "iam-b200 0.1 (sm_100a)"; }

const char* iam_last_error(void) { return g_last_error.c_str(); }

int iam_device_info(int device, int* sm_count, int* cc_major, int* cc_minor) {
    cudaDeviceProp prop;
    IAM_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    if (sm_count) *sm_count = prop.multiProcessorCount;
    if (cc_major) *cc_major = prop.major;
    if (cc_minor) *cc_minor = prop.minor;
    if (prop.major != 10) return fail(IAM_ERR_UNSUPPORTED, "libiamb200 is built for sm_100a only");
    return IAM_OK;
}

int iam_bucketmul_plan_info(int vec, int cluster_size, int bucket_cols, int in_dim, int* max_active_clusters,
                            int* log2_lanes, int* n_tiles, int* n_splits) {
    if ((vec != 8 && vec != 4 && vec != 1) || cluster_size < 1 || cluster_size > kMaxCluster || bucket_cols <= 0 || in_dim <= 0)
        return fail(IAM_ERR_ARG, "iam_bucketmul_plan_info: bad arguments");
    const int mac = bm_max_active_clusters(vec, cluster_size);
    BMBatch b;
    memset(&b, 0, sizeof(b));
    b.nprob = 1;
    b.p[0].cols = bucket_cols;
    b.p[0].n_rows_valid = 16 * in_dim;
    b.p[0].n_inputs = in_dim;
    b.mode = kModeFused;
    bm_plan(b, vec, cluster_size, mac);
    if (max_active_clusters) *max_active_clusters = mac;
    if (log2_lanes) *log2_lanes = b.p[0].log2L;
    if (n_tiles) *n_tiles = b.p[0].n_tiles;
    if (n_splits) *n_splits = b.p[0].n_split;
    return IAM_OK;
}

int iam_bucketmul_create(iam_bucketmul_t* out, int device) {
    if (!out) return fail(IAM_ERR_ARG, "iam_bucketmul_create: null out");
    *out = nullptr;
    int rc = iam_device_info(device, nullptr, nullptr, nullptr);
    if (rc) return rc;
    IAM_CUDA_TRY(cudaSetDevice(device));
    iam_bucketmul_s* h = new iam_bucketmul_s();
    h->device = device;
    cudaError_t e = cudaMalloc(&h->cutoff, sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&h->ints, sizeof(int) * (8 + kMaxSplits));
    if (e == cudaSuccess) e = cudaMalloc(&h->ctr, sizeof(int) * kCtrSlots);
    if (e == cudaSuccess) e = cudaMemset(h->ctr, 0, sizeof(int) * kCtrSlots);
    if (e == cudaSuccess) e = cudaMalloc(&h->bar, 4 * sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(h->bar, 0, 4 * sizeof(unsigned));
    if (e != cudaSuccess) {
        iam_bucketmul_destroy(h);
        return cuda_fail(e, "iam_bucketmul_create: cudaMalloc");
    }
    *out = h;
    return IAM_OK;
}

int iam_bucketmul_destroy(iam_bucketmul_t h) {
    if (!h) return IAM_OK;
    cudaFree(h->list);
    cudaFree(h->partials);
    cudaFree(h->ctr);
    cudaFree(h->cutoff);
    cudaFree(h->ints);
    cudaFree(h->gpartials);
    cudaFree(h->bar);
    delete h;
    return IAM_OK;
}

int iam_bucketmul_cutoff(iam_bucketmul_t h, const float* x_dev, const uint16_t* probes_dev, int expert_no,
                         int in_dim, float effort, float* cutoff_dev, int* iters_dev, void* stream) {
    if (!h || !x_dev || !probes_dev || !cutoff_dev) return fail(IAM_ERR_ARG, "iam_bucketmul_cutoff: null pointer");
    if (in_dim <= 0 || expert_no < 0) return fail(IAM_ERR_ARG, "iam_bucketmul_cutoff: bad in_dim/expert_no");
    if (!effort_ok(effort)) return fail(IAM_ERR_ARG, "iam_bucketmul_cutoff: effort must be in (0, 1]");
    const int P = in_dim < IAM_PROBES_COUNT ? in_dim : IAM_PROBES_COUNT;
    return bm_launch_cutoff(x_dev, probes_dev + (size_t)expert_no * IAM_PROBES_COUNT, P, bm_target(effort, P),
                            cutoff_dev, iters_dev, (cudaStream_t)stream);
}

int iam_bucketmul_calc_dispatch(iam_bucketmul_t h, const float* x_dev, const uint16_t* stats_dev, int stats_stride,
                                const uint16_t* probes_dev, int expert_no, int in_dim, int bucket_cols,
                                int expert_size, float effort, void* stream) {
    if (!h) return fail(IAM_ERR_ARG, "iam_bucketmul_calc_dispatch: null handle");
    h->have_dispatch = false;
    const int G = bm_default_cluster();
    BMBatch b;
    memset(&b, 0, sizeof(b));
    int rc = fill_problem(h, b.p[0], G, x_dev, stats_dev, stats_stride, probes_dev, expert_no, in_dim,
                          bucket_cols, expert_size, effort);
    if (rc) return rc;
    b.p[0].cutoff_out = h->cutoff;
    b.p[0].count_out = h->ints;
    b.p[0].iters_out = h->ints + 1;
    b.nprob = 1;
    b.mode = kModeSelectOnly;
    bm_plan(b, 1, G, 1);
    rc = bm_launch(b, 1, G, (cudaStream_t)stream);
    if (rc) return rc;
    h->disp = b.p[0];
    h->disp_G = G;
    h->disp_bucket_cols = bucket_cols;
    h->have_dispatch = true;
    return IAM_OK;
}

int iam_bucketmul_read_dispatch(iam_bucketmul_t h, int32_t* rows_dev, int* count_dev, float* cutoff_dev,
                                void* stream) {
    if (!h || !h->have_dispatch) return fail(IAM_ERR_ARG, "iam_bucketmul_read_dispatch: no dispatch recorded");
    cudaStream_t s = (cudaStream_t)stream;
    if (rows_dev)
        IAM_CUDA_TRY(cudaMemcpyAsync(rows_dev, h->list, sizeof(int32_t) * (size_t)h->disp.n_rows_valid,
                                     cudaMemcpyDeviceToDevice, s));
    if (count_dev) IAM_CUDA_TRY(cudaMemcpyAsync(count_dev, h->ints, sizeof(int), cudaMemcpyDeviceToDevice, s));
    if (cutoff_dev) IAM_CUDA_TRY(cudaMemcpyAsync(cutoff_dev, h->cutoff, sizeof(float), cudaMemcpyDeviceToDevice, s));
    return IAM_OK;
}

int iam_bucketmul_mul(iam_bucketmul_t h, const uint16_t* buckets_dev, int bucket_rows, int bucket_cols,
                      float* out_dev, void* stream) {
    if (!h || !h->have_dispatch) return fail(IAM_ERR_ARG, "iam_bucketmul_mul: call iam_bucketmul_calc_dispatch first");
    if (!buckets_dev || !out_dev) return fail(IAM_ERR_ARG, "iam_bucketmul_mul: null buckets/out");
    if (bucket_cols != h->disp_bucket_cols)
        return fail(IAM_ERR_ARG, "iam_bucketmul_mul: bucket_cols differs from the dispatch's bucketCols");
    if ((long long)bucket_rows < h->disp.row0 + h->disp.n_rows_valid)
        return fail(IAM_ERR_ARG, "iam_bucketmul_mul: buckets tensor has fewer rows than the dispatch covers");
    BMBatch b;
    memset(&b, 0, sizeof(b));
    b.p[0] = h->disp;
    b.p[0].buckets = buckets_dev;
    b.p[0].out = out_dev;
    b.p[0].cutoff_out = nullptr;
    b.p[0].count_out = nullptr;
    b.p[0].iters_out = nullptr;
    b.nprob = 1;
    b.mode = kModeMulOnly;
    const int G = h->disp_G;
    const int vec = pick_vec(b);
    bm_plan(b, vec, G, bm_max_active_clusters(vec, G));
    if (!plan_fits(b, G)) return fail(IAM_ERR_UNSUPPORTED, "iam_bucketmul_mul: plan exceeds scratch");
    return bm_launch(b, vec, G, (cudaStream_t)stream);
}

int iam_bucketmul_full(iam_bucketmul_t h, const float* x_dev, const uint16_t* stats_dev, int stats_stride,
                       const uint16_t* probes_dev, const uint16_t* buckets_dev, int expert_no, int in_dim,
                       int bucket_cols, int expert_size, float effort, float* out_dev, int* count_dev,
                       float* cutoff_dev, void* stream) {
    if (!h) return fail(IAM_ERR_ARG, "iam_bucketmul_full: null handle");
    if (!buckets_dev || !out_dev) return fail(IAM_ERR_ARG, "iam_bucketmul_full: null buckets/out");
    if (!x_dev || !stats_dev || !probes_dev) return fail(IAM_ERR_ARG, "bucketmul: null input/stats/probes pointer");
    if (in_dim <= 0 || bucket_cols <= 0 || expert_size <= 0 || expert_no < 0)
        return fail(IAM_ERR_ARG, "bucketmul: in_dim, bucket_cols, expert_size must be > 0, expert_no >= 0");
    if (stats_stride != 1 && stats_stride != 4)
        return fail(IAM_ERR_ARG, "bucketmul: stats_stride must be 1 (packed) or 4 (file layout)");
    if (!effort_ok(effort)) return fail(IAM_ERR_ARG, "bucketmul: effort must be in (0, 1]");
    // one launch of the range kernel (iam_bucketmul_group.cu); its partials and barrier words
    // live in the handle
    const size_t need = bg_scratch_floats(kMaxRanges, bucket_cols);
    if (need > h->gpartials_cap) {
        if (h->gpartials) IAM_CUDA_TRY(cudaFree(h->gpartials));
        h->gpartials = nullptr;
        h->gpartials_cap = 0;
        IAM_CUDA_TRY(cudaMalloc(&h->gpartials, need * sizeof(float)));
        h->gpartials_cap = need;
    }
    BGBatch b;
    memset(&b, 0, sizeof(b));
    BGProblem& p = b.p[0];
    p.x = x_dev;
    p.stats = stats_dev;
    p.stats_stride = stats_stride;
    p.probes = probes_dev + (size_t)expert_no * IAM_PROBES_COUNT;  // bucketMul.cl:103
    p.buckets = buckets_dev;
    p.row0 = (long long)expert_size * expert_no;                    // bucketMul.cl:363
    p.bucket_row0 = 0;
    p.n_rows_valid = expert_size < 16 * in_dim ? expert_size : 16 * in_dim;
    p.in_begin = 0;
    p.n_in = (p.n_rows_valid + 15) / 16;
    p.cols = bucket_cols;
    p.P = in_dim < IAM_PROBES_COUNT ? in_dim : IAM_PROBES_COUNT;
    p.target = bm_target(effort, p.P);
    p.out = out_dev;
    p.count_out = count_dev;
    p.cutoff_out = cutoff_dev;
    p.partials = h->gpartials;
    if ((p.row0 + p.n_rows_valid) * (long long)bucket_cols >= (1LL << 31))
        return fail(IAM_ERR_UNSUPPORTED, "bucketmul: rows * bucket_cols must stay below 2^31 elements");
    b.nprob = 1;
    b.xmode = kXPlain;
    b.barrier = h->bar;
    b.trace = h->trace ? h->trace : h->dbg;
    b.trace_cap = h->trace ? h->trace_cap : (h->dbg ? 1 : 0);
    bg_choose_shape(b);
    return bg_launch(b, (cudaStream_t)stream);
}

int iam_bucketmul_status(iam_bucketmul_t h) {
    if (!h) return fail(IAM_ERR_ARG, "iam_bucketmul_status: null handle");
    IAM_CUDA_TRY(cudaSetDevice(h->device));
    IAM_CUDA_TRY(cudaDeviceSynchronize());
    unsigned bar[4] = {0, 0, 0, 0};
    IAM_CUDA_TRY(cudaMemcpy(bar, h->bar, sizeof(bar), cudaMemcpyDeviceToHost));
    if (bar[2]) return fail(IAM_ERR_TIMEOUT, "iam_bucketmul_full: a launch gave up waiting at its grid barrier");
    return IAM_OK;
}

int iam_bucketmul_phase_times(iam_bucketmul_t h, long long* times_dev) {
    if (!h) return fail(IAM_ERR_ARG, "iam_bucketmul_phase_times: null handle");
    h->dbg = times_dev;
    return IAM_OK;
}

int iam_bucketmul_trace(iam_bucketmul_t h, long long* trace_dev, int capacity) {
    if (!h || capacity < 0) return fail(IAM_ERR_ARG, "iam_bucketmul_trace: bad arguments");
    h->trace = trace_dev;
    h->trace_cap = trace_dev ? capacity : 0;
    return IAM_OK;
}

int iam_stats_pack(const uint16_t* stats4_dev, long long rows, uint16_t* stats1_dev, void* stream) {
    if (!stats4_dev || !stats1_dev || rows < 0) return fail(IAM_ERR_ARG, "iam_stats_pack: bad arguments");
    if (rows == 0) return IAM_OK;
    return bm_launch_stats_pack(stats4_dev, rows, stats1_dev, (cudaStream_t)stream);
}

int iam_bucketize(const uint16_t* w_dev, int out_dim, int in_dim, uint16_t* buckets_dev, uint16_t* stats4_dev,
                  uint16_t* stats1_dev, uint16_t* probes_dev, void* stream) {
    if (!w_dev || !buckets_dev) return fail(IAM_ERR_ARG, "iam_bucketize: null W/buckets");
    if (out_dim <= 0 || in_dim <= 0 || out_dim % 16 != 0)
        return fail(IAM_ERR_ARG, "iam_bucketize: out_dim must be a positive multiple of 16");
    return bucketize_launch(w_dev, out_dim, in_dim, buckets_dev, stats4_dev, stats1_dev, probes_dev,
                            (cudaStream_t)stream);
}

}  // extern "C"

// ------------------------------------------------------------------ no-allocation variant
//
// Some callers of a bucketMul cannot allocate device memory at all: code that runs inside a
// host-side allocator or memory-pool callback, a plug-in whose host framework owns every
// device allocation and forbids its plug-ins from calling cudaMalloc, or a context where an
// allocation would synchronise the device at the wrong moment.  For them the fused
// bucketMul's scratch (the partial tiles of the input splits, the arrival counters and the
// per-split selected counts) lives in one file-scope __device__ array instead of a handle.
// The array is part of the module: every GPU that loads the library holds its ~1 MiB until
// the process exits.

namespace {

constexpr int kNoAllocMaxCols = 1024;  // bucket columns, i.e. out_dim <= 16384
constexpr int kNoAllocMaxSplits = 16;  // input splits the plan may use
constexpr int kNoAllocCtrSlots = 1024; // column tiles x cluster size
constexpr size_t kNoAllocPartials = (size_t)kNoAllocMaxSplits * 16 * kNoAllocMaxCols;  // floats
constexpr size_t kNoAllocFloats = kNoAllocPartials + kNoAllocCtrSlots + kNoAllocMaxSplits;

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocFloats];

// Device address of g_noalloc_scratch on the current device (the host-side name is only a
// stand-in for the symbol and must never reach a kernel).  Every call made outside a stream
// capture looks the address up again (cudaGetSymbolAddress, no allocation) and remembers it
// for the device, so a context torn down and re-created (cudaDeviceReset) gets the new
// module's address; a call made while `stream` is being captured uses the remembered one,
// which an earlier call outside capture on the same device must have set.
int noalloc_scratch(cudaStream_t stream, float** out) {
    static std::mutex mu;
    static float* addr[256] = {};
    int dev = 0;
    IAM_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 256) return fail(IAM_ERR_UNSUPPORTED, "iam_bucketmul_full_noalloc: device index >= 256");
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    IAM_CUDA_TRY(cudaStreamIsCapturing(stream, &cap));
    std::lock_guard<std::mutex> lk(mu);
    if (cap == cudaStreamCaptureStatusNone) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "iam_bucketmul_full_noalloc: cudaGetSymbolAddress");
        addr[dev] = static_cast<float*>(p);
    } else if (!addr[dev]) {
        return fail(IAM_ERR_ARG,
                    "iam_bucketmul_full_noalloc: the first call on a device must come before any stream capture");
    }
    *out = addr[dev];
    return IAM_OK;
}

}  // namespace

extern "C" int iam_bucketmul_full_noalloc(const float* x_dev, const uint16_t* stats_dev, int stats_stride,
                                          const uint16_t* probes_dev, const uint16_t* buckets_dev, int expert_no,
                                          int in_dim, int bucket_cols, int expert_size, float effort, float* out_dev,
                                          int* count_dev, float* cutoff_dev, void* stream) {
    if (!x_dev || !stats_dev || !probes_dev || !buckets_dev || !out_dev)
        return fail(IAM_ERR_ARG, "iam_bucketmul_full_noalloc: null input, stats, probes, buckets or output");
    if (in_dim <= 0 || bucket_cols <= 0 || expert_size <= 0 || expert_no < 0)
        return fail(IAM_ERR_ARG, "iam_bucketmul_full_noalloc: in_dim, bucket_cols, expert_size must be > 0");
    if (bucket_cols > kNoAllocMaxCols)
        return fail(IAM_ERR_ARG,
                    "iam_bucketmul_full_noalloc: bucket_cols exceeds the built-in scratch (at most 1024 bucket "
                    "columns, i.e. out_dim <= 16384); use iam_bucketmul_full");
    if (stats_stride != 1 && stats_stride != 4)
        return fail(IAM_ERR_ARG, "iam_bucketmul_full_noalloc: stats_stride must be 1 or 4");
    if (!effort_ok(effort)) return fail(IAM_ERR_ARG, "iam_bucketmul_full_noalloc: effort must be in (0, 1]");
    float* scratch = nullptr;
    int rc = noalloc_scratch((cudaStream_t)stream, &scratch);
    if (rc) return rc;
    const int G = bm_default_cluster();
    BMBatch b;
    memset(&b, 0, sizeof(b));
    BMProblem& p = b.p[0];
    p.x = x_dev;
    p.stats = stats_dev;
    p.stats_stride = stats_stride;
    p.probes = probes_dev + (size_t)expert_no * IAM_PROBES_COUNT;
    p.buckets = buckets_dev;
    p.row0 = (long long)expert_size * expert_no;
    p.n_rows_valid = expert_size < 16 * in_dim ? expert_size : 16 * in_dim;
    p.n_inputs = (p.n_rows_valid + 15) / 16;
    p.cols = bucket_cols;
    p.P = in_dim < IAM_PROBES_COUNT ? in_dim : IAM_PROBES_COUNT;
    p.target = bm_target(effort, p.P);
    p.out = out_dev;
    p.count_out = count_dev;
    p.cutoff_out = cutoff_dev;
    p.partials = scratch;
    p.slice_ctr = reinterpret_cast<int*>(scratch + kNoAllocPartials);
    p.split_sel = reinterpret_cast<int*>(scratch + kNoAllocPartials + kNoAllocCtrSlots);
    if ((p.row0 + p.n_rows_valid) * (long long)bucket_cols >= (1LL << 31))
        return fail(IAM_ERR_UNSUPPORTED, "iam_bucketmul_full_noalloc: rows * bucket_cols must stay below 2^31");
    b.nprob = 1;
    b.mode = kModeFused;
    const int vec = pick_vec(b);
    bm_plan(b, vec, G, bm_max_active_clusters(vec, G), kNoAllocMaxSplits);
    if (p.n_tiles * G > kNoAllocCtrSlots)
        return fail(IAM_ERR_UNSUPPORTED, "iam_bucketmul_full_noalloc: too many column tiles for the scratch");
    // the arrival counters must start at zero (a launch leaves them at zero, but a call that
    // failed before its kernel ran, or a kernel error, would not)
    IAM_CUDA_TRY(cudaMemsetAsync(p.slice_ctr, 0, sizeof(int) * kNoAllocCtrSlots, (cudaStream_t)stream));
    return bm_launch(b, vec, G, (cudaStream_t)stream);
}
