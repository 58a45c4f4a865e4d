// iam_tp.cu -- one-shot NVLink collectives for the tensor-parallel decode step (see iam_tp.h).
//
// Low-latency protocol: every element travels as one 8-byte store {value bits, epoch} into
// the receiver's mailbox (an aligned 8-byte store is seen whole, so no fence or separate flag
// is needed); the receiver polls each of its elements (bounded) until the epoch word matches.
// Every launch has kTpCtas CTAs and each advances its own copy of the epoch, so all copies
// hold the number of collective calls so far: an epoch names one call on every element, and
// every rank makes the same sequence of calls.  The mailbox is double-buffered by epoch parity: a sender can only reach
// epoch e + 2 after every peer finished the launch of epoch e that read the same half.
#include "iam_common.cuh"
#include "iam_tp.h"

namespace iam {

namespace {

IAM_DEV void st_ll(uint2* p, uint32_t bits, uint32_t epoch) {
    asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(bits), "r"(epoch) : "memory");
}

IAM_DEV uint2 ld_ll(const uint2* p) {
    uint2 v;
    asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
    return v;
}

IAM_DEV uint2* mbox_of(const TpWindow& w, int owner, uint32_t epoch, int src) {
    return reinterpret_cast<uint2*>(w.base[owner] + w.mbox_off) +
           ((size_t)(epoch & 1u) * w.world + src) * (size_t)w.mbox_floats;
}

// Epoch of this launch for slice c (read by the whole CTA).
IAM_DEV uint32_t begin_epoch(const TpWindow& w, int c, uint32_t* s_epoch) {
    if (threadIdx.x == 0) *s_epoch = reinterpret_cast<uint32_t*>(w.base[w.rank] + w.epoch_off)[c] + 1u;
    __syncthreads();
    return *s_epoch;
}

IAM_DEV void end_epoch(const TpWindow& w, int c, uint32_t epoch) {
    __syncthreads();
    if (threadIdx.x == 0) reinterpret_cast<uint32_t*>(w.base[w.rank] + w.epoch_off)[c] = epoch;
}

// Sends element i of this rank to every peer's mailbox slot (this rank, i).
IAM_DEV void send(const TpWindow& w, uint32_t epoch, int i, float v) {
    for (int p = 0; p < w.world; ++p)
        if (p != w.rank) st_ll(mbox_of(w, p, epoch, w.rank) + i, __float_as_uint(v), epoch);
}

// Element i from rank r (bounded wait); on a timeout the error word is set and 0 returned.
// Once this rank has given up on any wait, later exchanges do not wait at all (their outputs
// are invalid anyway; the host learns of it from iam_model_status).
IAM_DEV float recv(const TpWindow& w, uint32_t epoch, int r, int i) {
    volatile uint32_t* err = reinterpret_cast<volatile uint32_t*>(w.base[w.rank] + w.err_off);
    const uint2* q = mbox_of(w, w.rank, epoch, r) + i;
    long long n = 0;
    for (;;) {
        const uint2 v = ld_ll(q);
        if (v.y == epoch) return __uint_as_float(v.x);
        if (++n > w.spin_limit || *err != 0u) {
            *err = 1u;
            return 0.0f;
        }
        if (n > 64) __nanosleep(32);
    }
}

__global__ void __launch_bounds__(kTpThreads) tp_allgather_kernel(TpWindow w, size_t off_a, size_t off_b, int chunk) {
    pdl_wait();
    __shared__ uint32_t s_epoch;
    const int c = blockIdx.x;
    const uint32_t epoch = begin_epoch(w, c, &s_epoch);
    const int nb = off_b == (size_t)-1 ? 1 : 2;
    const int n = nb * chunk;  // element e: buffer e / chunk, index e % chunk
    const int per = (n + kTpCtas - 1) / kTpCtas;
    const int e0 = min(n, c * per), e1 = min(n, e0 + per);
    const size_t mine = (size_t)w.rank * chunk;
    for (int e = e0 + threadIdx.x; e < e1; e += kTpThreads) {
        const size_t off = e < chunk ? off_a : off_b;
        send(w, epoch, e, reinterpret_cast<const float*>(w.base[w.rank] + off)[mine + e % chunk]);
    }
    for (int e = e0 + threadIdx.x; e < e1; e += kTpThreads) {
        float* dst = reinterpret_cast<float*>(w.base[w.rank] + (e < chunk ? off_a : off_b));
        for (int r = 0; r < w.world; ++r)
            if (r != w.rank) dst[(size_t)r * chunk + e % chunk] = recv(w, epoch, r, e);
    }
    pdl_trigger();
    end_epoch(w, c, epoch);
}

__global__ void __launch_bounds__(kTpThreads) tp_allreduce_kernel(TpWindow w, size_t off, int n) {
    pdl_wait();
    __shared__ uint32_t s_epoch;
    const int c = blockIdx.x;
    const uint32_t epoch = begin_epoch(w, c, &s_epoch);
    const int per = (n + kTpCtas - 1) / kTpCtas;
    const int i0 = min(n, c * per), i1 = min(n, i0 + per);
    float* buf = reinterpret_cast<float*>(w.base[w.rank] + off);
    for (int i = i0 + threadIdx.x; i < i1; i += kTpThreads) send(w, epoch, i, buf[i]);
    for (int i = i0 + threadIdx.x; i < i1; i += kTpThreads) {
        float acc = 0.0f;
        for (int r = 0; r < w.world; ++r) {
            const float v = r == w.rank ? buf[i] : recv(w, epoch, r, i);
            acc = r == 0 ? v : acc + v;  // rank order: the same bits on every rank
        }
        buf[i] = acc;
    }
    pdl_trigger();
    end_epoch(w, c, epoch);
}

// Each rank holds the partials of r_local consecutive input ranges (ranges rank * r_local ..,
// [r_local][M] floats, then r_local row counts); every rank receives all of them and adds the
// R = world * r_local <= kTpMaxRanges partials of each output in range order, then the residual
// -- the order in which one GPU's bucketMul kernel adds its R ranges -- so the sum is identical
// on every rank and to the single-GPU one.  A thread takes one output and issues the loads of
// its R partials together (its own from memory, the peers' from the mailbox), then polls again
// only for those whose epoch has not arrived (bounded).  The rank's own row count goes to
// *count_out.
constexpr int kTpMaxRanges = 32;

__global__ void __launch_bounds__(kTpThreads) tp_gather_reduce_kernel(TpWindow w, const float* part, int M,
                                                                      int r_local, const float* residual,
                                                                      float* out, int* count_out) {
    pdl_wait();
    __shared__ uint32_t s_epoch;
    const int c = blockIdx.x;
    const uint32_t epoch = begin_epoch(w, c, &s_epoch);
    const int n = r_local * M;  // payload elements (the row counts stay local)
    const int gt = c * kTpThreads + threadIdx.x, nt = kTpCtas * kTpThreads;
    for (int e = gt; e < n; e += nt) send(w, epoch, e, part[e]);
    const int R = r_local * w.world;
    volatile uint32_t* err = reinterpret_cast<volatile uint32_t*>(w.base[w.rank] + w.err_off);
    for (int i = gt; i < M; i += nt) {
        float v[kTpMaxRanges];
        uint32_t pend = 0u;
#pragma unroll
        for (int g = 0; g < kTpMaxRanges; ++g) {
            v[g] = 0.0f;
            if (g < R) {
                const int owner = g / r_local, e = (g - owner * r_local) * M + i;
                if (owner == w.rank) {
                    v[g] = part[e];
                } else {
                    const uint2 x = ld_ll(mbox_of(w, w.rank, epoch, owner) + e);
                    if (x.y == epoch) v[g] = __uint_as_float(x.x);
                    else pend |= 1u << g;
                }
            }
        }
        for (long long polls = 0; pend;) {
            if (++polls > w.spin_limit || *err != 0u) {  // a peer never sent: flag it, give up
                *err = 1u;
                break;
            }
            if (polls > 64) __nanosleep(32);
#pragma unroll
            for (int g = 0; g < kTpMaxRanges; ++g)
                if ((pend >> g) & 1u) {
                    const int owner = g / r_local, e = (g - owner * r_local) * M + i;
                    const uint2 x = ld_ll(mbox_of(w, w.rank, epoch, owner) + e);
                    if (x.y == epoch) {
                        v[g] = __uint_as_float(x.x);
                        pend &= ~(1u << g);
                    }
                }
        }
        float acc = 0.0f;
#pragma unroll
        for (int g = 0; g < kTpMaxRanges; ++g)
            if (g < R) acc += v[g];
        out[i] = residual ? residual[i] + acc : acc;  // add32 (bucketMul.cl:517-520)
    }
    if (c == 0 && threadIdx.x == 0 && count_out) {
        const int* rows = reinterpret_cast<const int*>(part + n);
        int t = 0;
        for (int r = 0; r < r_local; ++r) t += rows[r];
        *count_out = t;
    }
    pdl_trigger();
    end_epoch(w, c, epoch);
}

// The packed argmax key (64 bits) travels as two elements: high and low words.
__global__ void __launch_bounds__(kTpThreads) tp_keymax_kernel(TpWindow w, unsigned long long* key) {
    pdl_wait();
    __shared__ uint32_t s_epoch;
    const int c = blockIdx.x;  // every CTA advances its epoch; CTA 0 does the work
    const uint32_t epoch = begin_epoch(w, c, &s_epoch);
    if (c == 0 && threadIdx.x == 0) {
        const unsigned long long k = *key;
        send(w, epoch, 0, __uint_as_float((uint32_t)(k >> 32)));
        send(w, epoch, 1, __uint_as_float((uint32_t)k));
        unsigned long long m = k;
        for (int r = 0; r < w.world; ++r) {
            if (r == w.rank) continue;
            const unsigned long long hi = __float_as_uint(recv(w, epoch, r, 0));
            const unsigned long long lo = __float_as_uint(recv(w, epoch, r, 1));
            const unsigned long long kr = (hi << 32) | lo;
            m = kr > m ? kr : m;
        }
        *key = m;
    }
    pdl_trigger();
    end_epoch(w, c, epoch);
}

}  // namespace

int tp_allgather(const TpWindow& w, size_t off_a, size_t off_b, int chunk, cudaStream_t s, bool pdl) {
    if ((off_b == (size_t)-1 ? 1 : 2) * chunk > w.mbox_floats) return fail(IAM_ERR_UNSUPPORTED, "tp all-gather larger than the mailbox");
    IAM_CUDA_TRY(launch_ex(tp_allgather_kernel, dim3(kTpCtas), dim3(kTpThreads), 0, s, pdl, w, off_a, off_b, chunk));
    return IAM_OK;
}

int tp_allreduce_sum(const TpWindow& w, size_t off, int n, cudaStream_t s, bool pdl) {
    if (n > w.mbox_floats) return fail(IAM_ERR_UNSUPPORTED, "tp all-reduce larger than the mailbox");
    IAM_CUDA_TRY(launch_ex(tp_allreduce_kernel, dim3(kTpCtas), dim3(kTpThreads), 0, s, pdl, w, off, n));
    return IAM_OK;
}

int tp_gather_reduce(const TpWindow& w, const float* partials, int M, int r_local, const float* residual, float* out,
                     int* count_out, cudaStream_t s, bool pdl) {
    if ((long long)r_local * M > w.mbox_floats) return fail(IAM_ERR_UNSUPPORTED, "tp gather-reduce larger than the mailbox");
    if (r_local < 1 || r_local * w.world > kTpMaxRanges) return fail(IAM_ERR_UNSUPPORTED, "tp gather-reduce: too many ranges");
    IAM_CUDA_TRY(launch_ex(tp_gather_reduce_kernel, dim3(kTpCtas), dim3(kTpThreads), 0, s, pdl, w, partials, M, r_local,
                           residual, out, count_out));
    return IAM_OK;
}

int tp_keymax(const TpWindow& w, unsigned long long* key, cudaStream_t s, bool pdl) {
    IAM_CUDA_TRY(launch_ex(tp_keymax_kernel, dim3(kTpCtas), dim3(kTpThreads), 0, s, pdl, w, key));
    return IAM_OK;
}

}  // namespace iam

// ------------------------------------------------------------------ bounded-wait self-test

using namespace iam;

extern "C" int iam_tp_wait_selftest(int device, int n, long long spin_limit, unsigned* err_out, float* first_ms,
                                    float* second_ms) {
    if (n <= 0 || n > (1 << 20) || spin_limit <= 0) return fail(IAM_ERR_ARG, "iam_tp_wait_selftest: bad n or spin_limit");
    IAM_CUDA_TRY(cudaSetDevice(device));
    // two windows on this GPU: rank 0's own and a stand-in for rank 1 that no kernel ever
    // writes into rank 0's mailbox, so every wait of rank 0 runs to its poll bound
    TpWindow w{};
    w.rank = 0;
    w.world = 2;
    w.mbox_floats = n;
    w.spin_limit = spin_limit;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += (bytes + 255) / 256 * 256;
        return o;
    };
    const size_t o_buf = take((size_t)n * 4);
    w.epoch_off = take(4 * kTpCtas);
    w.err_off = take(4);
    w.mbox_off = take((size_t)2 * w.world * w.mbox_floats * 8);
    char* mem[2] = {nullptr, nullptr};
    cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
    cudaStream_t s = nullptr;
    int rc = IAM_OK;
    cudaError_t e = cudaMalloc(&mem[0], off);
    if (e == cudaSuccess) e = cudaMalloc(&mem[1], off);
    if (e == cudaSuccess) e = cudaMemset(mem[0], 0, off);
    if (e == cudaSuccess) e = cudaMemset(mem[1], 0, off);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    for (int i = 0; i < 3 && e == cudaSuccess; ++i) e = cudaEventCreate(&ev[i]);
    if (e != cudaSuccess) rc = cuda_fail(e, "iam_tp_wait_selftest: setup");
    w.base[0] = mem[0];
    w.base[1] = mem[1];
    if (!rc && (e = cudaEventRecord(ev[0], s)) != cudaSuccess) rc = cuda_fail(e, "iam_tp_wait_selftest: event");
    if (!rc) rc = tp_allreduce_sum(w, o_buf, n, s, false);
    if (!rc && (e = cudaEventRecord(ev[1], s)) != cudaSuccess) rc = cuda_fail(e, "iam_tp_wait_selftest: event");
    if (!rc) rc = tp_allreduce_sum(w, o_buf, n, s, false);  // the error word is set: no waiting
    if (!rc && (e = cudaEventRecord(ev[2], s)) != cudaSuccess) rc = cuda_fail(e, "iam_tp_wait_selftest: event");
    if (!rc && (e = cudaStreamSynchronize(s)) != cudaSuccess) rc = cuda_fail(e, "iam_tp_wait_selftest: run");
    unsigned err = 0;
    if (!rc && (e = cudaMemcpy(&err, mem[0] + w.err_off, sizeof(err), cudaMemcpyDeviceToHost)) != cudaSuccess)
        rc = cuda_fail(e, "iam_tp_wait_selftest: read error word");
    float t1 = 0.0f, t2 = 0.0f;
    if (!rc) {
        cudaEventElapsedTime(&t1, ev[0], ev[1]);
        cudaEventElapsedTime(&t2, ev[1], ev[2]);
    }
    for (cudaEvent_t x : ev)
        if (x) cudaEventDestroy(x);
    if (s) cudaStreamDestroy(s);
    cudaFree(mem[0]);
    cudaFree(mem[1]);
    if (rc) return rc;
    if (err_out) *err_out = err;
    if (first_ms) *first_ms = t1;
    if (second_ms) *second_ms = t2;
    if (err) return fail(IAM_ERR_TIMEOUT, "iam_tp_wait_selftest: the exchange gave up waiting for the missing peer");
    return IAM_OK;
}
