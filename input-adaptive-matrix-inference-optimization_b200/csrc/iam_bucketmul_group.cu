// iam_bucketmul_group.cu -- the range bucketMul kernel (sm_100a): the fused BucketMul::fullMul
// (bucket_mul.hpp:254-267 over bucketMul.cl:68-497) as one launch of at most one CTA per SM.
//
// Work split.  CTA (tile, range) owns a tile of TW bucket columns and a contiguous range of
// inputs of one matrix (a launch holds up to 3 matrices that share x).  512 threads per CTA.
//   0. before the dependency wait (weights only): the range's packed stats rows are
//      bulk-copied (cp.async.bulk, no multicast) into shared memory, probes toward L2;
//   1. the cutoff over x[0:P] (findCutoffBinarySearch, bucketMul.cl:68-214), bit for bit,
//      as a counting sort plus an exact bisection: every importance gets a bin
//      floor((v - min) * 1024 / (max - min)), a monotone function of v, so for any tested
//      mid the values in bins above mid's bin are above it and those below are below; one
//      histogram, one scan and one scatter sort the values by bin, and each bisection step
//      (one warp) then compares mid with the values of its own bin only;
//   2. the selection (prepareDispatch, bucketMul.cl:351-386) of the range's bucket rows: a
//      16-bit mask per input, a prefix over the inputs, and a list of {row offset, x} in
//      shared memory in ascending row order (chunks).  With the reference layout the stats of
//      an input fall with the rank, so its selected rows are a prefix of its 16 and one
//      contiguous run of the buckets; the mask handles any stats;
//   3. the accumulation (bucketMul.cl:392-447): list position j goes to set j % NSETS =
//      (warp, row lane); each lane streams its rows' slices of `vec` columns (a register ring
//      of loads in flight) and adds x*w into lane-private per-slot accumulators in shared
//      memory, in list order;
//   4. the integrate (bucketMul.cl:453-497): the NSETS accumulators of every output are added
//      in set order into the CTA's partial (global scratch), a grid-wide barrier (all CTAs of
//      a launch are resident: one wave of at most one CTA per SM), then every CTA adds the
//      partials of a slice of outputs in range order and the residual.
// No float atomics: results are bitwise deterministic for a given device.  Every wait is
// bounded (the barrier sets an error word after ~2 s; the stats copy falls back to global
// loads and is drained before exit).
#include <algorithm>
#include <atomic>
#include <mutex>

#include "iam_bucketmul.cuh"
#include "iam_bucketmul_group.h"
#include "iam_bucketmul_launch.h"
#include "iam_tp_push.cuh"

namespace iam {

namespace {

constexpr int kGT = 512;             // threads per CTA
constexpr int kGW = kGT / 32;        // warps per CTA
constexpr int kVPT = kProbes / kGT;  // cutoff values per thread (8)
constexpr int kNB = 1024;            // bins of the counting sort
constexpr int kVMax = 4;             // columns per lane at most
constexpr int kSS = 9;               // log2(kVMax * 128): slot stride of the accumulators
constexpr uint32_t kRegion = 32u * 16u * 4u * kVMax;  // one warp's accumulators (bytes)
constexpr int kChunk = 2048;         // list rows per chunk
constexpr long long kBulkWaitPolls = 1LL << 22;  // bound of the stats copy wait
constexpr long long kBarrierPolls = 1LL << 22;   // bound of the grid barrier wait (~2 s)
constexpr int kRedFloats = 8192;     // final-reduce staging (inside the accumulators)
constexpr int kWinMax = 1024;        // most values ranked around the target (else the bin bisection)

struct GHeader {
    unsigned long long bar;  // mbarrier of the stats copy
    float wmin[kGW], wmax[kGW];
    int wsum[kGW];
    float red[256];  // block_rms_scale
    float result;
    int it, total, staged, maxbin;
    int blo, bhi, wn;  // bins holding the order statistics around the target, values gathered
    unsigned fepoch;   // tp_fused: the epoch of this launch's mailbox elements
};

constexpr size_t a16(size_t n) { return (n + 15) / 16 * 16; }

// Byte offsets of the dynamic shared memory (host and device agree).
struct GOffsets {
    size_t xall, xr, mask, pre, sts, list, acc, total;
};

__host__ __device__ inline GOffsets g_offsets(int range_max, bool stage) {
    GOffsets o{};
    size_t off = a16(sizeof(GHeader));
    o.xall = off;  off = a16(off + sizeof(float) * kProbes);
    o.xr = off;    off = a16(off + sizeof(float) * (size_t)range_max);
    o.mask = off;  off = a16(off + sizeof(uint16_t) * (size_t)range_max);
    o.pre = off;   off = a16(off + sizeof(int) * ((size_t)range_max + 1));
    o.sts = off;   off = a16(off + (stage ? 32 * (size_t)range_max : 0));
    o.list = off;  off = a16(off + sizeof(uint2) * (size_t)kChunk);
    o.acc = off;
    off += (size_t)(kGW + 1) * kRegion;  // + one region of alignment slack
    o.total = off;
    return o;
}

// The inputs other ranks made, when they are pushed (tp_wait): read from this rank's mailbox of
// that kind, polled until they carry the launch's epoch.  w == nullptr: every input is local.
struct PullIn {
    const TpWindow* w;
    int kind, lo, hi;  // this rank's inputs [lo, hi)
    unsigned epoch;
    IAM_DEV bool remote(int i) const { return w && (i < lo || i >= hi); }
    IAM_DEV bool local8(int i) const { return !w || (i >= lo && i + 8 <= hi); }
    IAM_DEV float get(size_t idx) const { return tp_push_recv(*w, kind, idx, epoch); }
    // elements idx .. idx + 7 (idx even): all eight loads in flight, then a poll of any late one
    IAM_DEV void get8(size_t idx, float* o) const {
        const uint4* q = reinterpret_cast<const uint4*>(tp_push_mbox(*w, w->rank, kind) + idx);
        uint4 v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
            asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(v[k].x), "=r"(v[k].y), "=r"(v[k].z), "=r"(v[k].w)
                         : "l"(q + k)
                         : "memory");
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            o[2 * k] = v[k].y == epoch ? __uint_as_float(v[k].x) : get(idx + 2 * k);
            o[2 * k + 1] = v[k].w == epoch ? __uint_as_float(v[k].z) : get(idx + 2 * k + 1);
        }
    }
};

// Tensor-parallel x: the local inputs through L2 (__ldcg), not the read-only path -- a peer
// stores this GPU's pushed inputs while the launch runs, so x is not read-only for the
// kernel's life -- and the others from the mailbox.
IAM_DEV void ldcg8(const float* p, float* o) {
    const float4 a = __ldcg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldcg(reinterpret_cast<const float4*>(p + 4));
    o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
    o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}

struct GXPlain {
    static constexpr bool kVectorizable = true;
    const float* x;
    PullIn in;
    IAM_DEV float operator()(int i) const { return in.remote(i) ? in.get((size_t)i) : __ldcg(x + i); }
    IAM_DEV bool aligned16() const { return (reinterpret_cast<uintptr_t>(x) & 15u) == 0; }
    IAM_DEV void load8(int i, float* o) const {
        if (in.local8(i)) ldcg8(x + i, o);
        else if (!in.remote(i) || !in.remote(i + 7)) {  // straddles this rank's inputs
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = (*this)(i + e);
        } else {
            in.get8((size_t)i, o);
        }
    }
};

struct GXSilu {
    static constexpr bool kVectorizable = true;
    const float* gate;
    const float* up;
    PullIn in;
    IAM_DEV float operator()(int i) const {
        return in.remote(i) ? XSilu::f(in.get((size_t)i), in.get((size_t)in.w->pmb_ffn + i))
                            : XSilu::f(__ldcg(gate + i), __ldcg(up + i));
    }
    IAM_DEV bool aligned16() const {
        return ((reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(up)) & 15u) == 0;
    }
    IAM_DEV void load8(int i, float* o) const {
        float g[8], u[8];
        if (in.local8(i)) {
            ldcg8(gate + i, g);
            ldcg8(up + i, u);
        } else if (!in.remote(i) || !in.remote(i + 7)) {
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = (*this)(i + e);
            return;
        } else {
            in.get8((size_t)i, g);
            in.get8((size_t)in.w->pmb_ffn + i, u);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = XSilu::f(g[e], u[e]);
    }
};

// x of a launch; TPX (a tensor-parallel launch) adds the reads of pushed inputs
template <int XM, int TPX>
struct GProvider;
template <>
struct GProvider<kXPlain, 0> {
    static IAM_DEV XPlain make(const BGProblem& p, float*, const PullIn&) { return XPlain{p.x}; }
};
template <>
struct GProvider<kXPlain, 1> {
    static IAM_DEV GXPlain make(const BGProblem& p, float*, const PullIn& in) { return GXPlain{p.x, in}; }
};
template <int TPX>
struct GProvider<kXRms, TPX> {
    static IAM_DEV XRms make(const BGProblem& p, float* red, const PullIn&) {
        return XRms{p.x, p.gain, block_rms_scale<kGT>(p.x, p.norm_n, p.norm_eps, red)};
    }
};
template <>
struct GProvider<kXSilu, 0> {
    static IAM_DEV XSilu make(const BGProblem& p, float*, const PullIn&) { return XSilu{p.x, p.x2}; }
};
template <>
struct GProvider<kXSilu, 1> {
    static IAM_DEV GXSilu make(const BGProblem& p, float*, const PullIn& in) { return GXSilu{p.x, p.x2, in}; }
};

// Bin of v: monotone non-decreasing in v (a fixed subtraction and a multiplication by a
// positive constant, each correctly rounded, then truncation and clamping).
IAM_DEV int vbin(float v, float mn, float inv_w) {
    const float e = __fmul_rn(__fsub_rn(v, mn), inv_w);
    return e <= 0.0f ? 0 : (e >= (float)(kNB - 1) ? kNB - 1 : (int)e);
}

IAM_DEV void mbar_init_cta(unsigned long long* b) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"((uint32_t)__cvta_generic_to_shared(b)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

IAM_DEV bool mbar_try(unsigned long long* b, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"((uint32_t)__cvta_generic_to_shared(b)), "r"(parity)
        : "memory");
    return done != 0u;
}

// Bounded wait for phase 0 of the stats-copy barrier.
IAM_DEV bool mbar_wait_bounded(unsigned long long* b) {
    for (long long n = 0; n < kBulkWaitPolls; ++n)
        if (mbar_try(b, 0u)) return true;
    return false;
}

// One bulk copy global -> shared memory completing on the barrier (both addresses 16-byte
// aligned, bytes a multiple of 16; a plain copy of this GPU's memory, no multicast).
IAM_DEV void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, unsigned long long* bar) {
    const uint32_t b = (uint32_t)__cvta_generic_to_shared(bar);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(b), "r"(bytes) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     (uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(__cvta_generic_to_global(src)), "r"(bytes), "r"(b)
                 : "memory");
}

// Grid-wide barrier of one launch over a {arrivals, generation, error} word triple that
// returns to arrivals = 0 after every use.  Called by every thread of every CTA.  A wait that
// runs out sets the error word and goes on (the launch's outputs are then invalid).
IAM_DEV void grid_barrier(unsigned* bar) {
    __syncthreads();
    if (threadIdx.x == 0) {
        // arrival with release semantics (this CTA's partials are visible before the count
        // moves), generation read with acquire semantics (the others' partials are visible
        // after it moves)
        unsigned gen;
        asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(gen) : "l"(bar + 1) : "memory");
        unsigned arrived;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(arrived) : "l"(bar) : "memory");
        if (arrived == gridDim.x - 1) {
            asm volatile("st.relaxed.gpu.global.u32 [%0], 0;" ::"l"(bar) : "memory");
            asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(bar + 1), "r"(gen + 1u) : "memory");
        } else {
            long long n = 0;
            for (;;) {
                unsigned g, err;
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(g) : "l"(bar + 1) : "memory");
                if (g != gen) break;
                asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(err) : "l"(bar + 2) : "memory");
                if (++n > kBarrierPolls || err != 0u) {
                    atomicOr(bar + 2, 1u);
                    break;
                }
                if (n > 256) __nanosleep(32);
            }
        }
    }
    __syncthreads();
}

// Adds x * w (V columns of one row, packed fp16 with the slot in the low 4 bits) into the
// lane's accumulators: slot s / column k at acc_lane + s * (1 << kSS) + k * 128.
template <int V>
IAM_DEV void acc_row(uint32_t acc_lane, uint32_t w0, uint32_t w1, float x) {
    constexpr uint32_t M = 15u << kSS;
    const uint32_t ws[2] = {w0, w1};
    uint32_t a[V];
    float old[V];
#pragma unroll
    for (int k = 0; k < V; ++k) {
        const uint32_t word = ws[k >> 1];
        a[k] = ((k & 1) ? ((word >> (16 - kSS)) & M) : ((word << kSS) & M)) | acc_lane;
    }
    if constexpr (V >= 1) old[0] = lds_f32<0>(a[0]);
    if constexpr (V >= 2) old[1] = lds_f32<128>(a[1]);
    if constexpr (V >= 3) old[2] = lds_f32<256>(a[2]);
    if constexpr (V >= 4) old[3] = lds_f32<384>(a[3]);
#pragma unroll
    for (int k = 0; k < V; ++k) {
        const uint32_t word = ws[k >> 1];
        old[k] = fmaf(x, h2f((k & 1) ? (word >> 16) : (word & 0xffffu)), old[k]);
    }
    if constexpr (V >= 1) sts_f32<0>(a[0], old[0]);
    if constexpr (V >= 2) sts_f32<128>(a[1], old[1]);
    if constexpr (V >= 3) sts_f32<256>(a[2], old[2]);
    if constexpr (V >= 4) sts_f32<384>(a[3], old[3]);
}

template <int V>
struct RowLoad;
template <>
struct RowLoad<1> {
    using T = uint32_t;
    static constexpr int kD = 32;
    static IAM_DEV T load(const uint16_t* p) { return (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(p)); }
    static IAM_DEV uint32_t w0(T v) { return v; }
    static IAM_DEV uint32_t w1(T) { return 0u; }
};
template <>
struct RowLoad<2> {
    using T = uint32_t;
    static constexpr int kD = 32;
    static IAM_DEV T load(const uint16_t* p) { return __ldg(reinterpret_cast<const unsigned int*>(p)); }
    static IAM_DEV uint32_t w0(T v) { return v; }
    static IAM_DEV uint32_t w1(T) { return 0u; }
};
template <>
struct RowLoad<4> {
    using T = uint2;
    static constexpr int kD = 16;
    static IAM_DEV T load(const uint16_t* p) { return __ldg(reinterpret_cast<const uint2*>(p)); }
    static IAM_DEV uint32_t w0(T v) { return v.x; }
    static IAM_DEV uint32_t w1(T v) { return v.y; }
};

// One chunk of n list rows for one lane: rows j0, j0 + NSETS, ... in order, a ring of kD loads
// in flight; past the end a lane re-reads the last row and adds exact zeros.
template <int V, int NSETS>
IAM_DEV void acc_chunk(const uint2* __restrict__ list, int n, int j0, int mw, const uint16_t* __restrict__ wbase,
                       uint32_t acc_lane) {
    using RL = RowLoad<V>;
    constexpr int kD = RL::kD;
    const int jlast = n - 1;
    typename RL::T w[kD];
#pragma unroll
    for (int d = 0; d < kD; ++d) w[d] = RL::load(wbase + list[min(j0 + d * NSETS, jlast)].x);
    int j = j0;
    for (int base = 0; base < mw; base += kD) {
#pragma unroll
        for (int d = 0; d < kD; ++d) {
            const float x = j < n ? __uint_as_float(list[j].y) : 0.0f;
            acc_row<V>(acc_lane, RL::w0(w[d]), RL::w1(w[d]), x);
            w[d] = RL::load(wbase + list[min(j + kD * NSETS, jlast)].x);
            j += NSETS;
        }
    }
}

// Tensor-parallel exchange inside the kernel (tp_fused): element e of this rank's range partials
// ([local range][M]) is stored into every peer's mailbox as one 8-byte {value bits, epoch} store
// (seen whole: no fence, no flag); the reduction polls its own mailbox, bounded, until the
// element of the awaited epoch is there.  Mailbox halves alternate by epoch parity: a rank can
// only reach epoch e + 2 after every peer has finished the launch of epoch e.
IAM_DEV uint2* fused_slot(const TpWindow& w, int owner, unsigned epoch, int src) {
    return reinterpret_cast<uint2*>(w.base[owner] + w.fused_off) +
           ((size_t)(epoch & 1u) * w.world + src) * (size_t)w.fused_floats;
}

IAM_DEV void fused_send(const TpWindow& w, unsigned epoch, int e, float v) {
    for (int p = 0; p < w.world; ++p)
        if (p != w.rank)
            asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(fused_slot(w, p, epoch, w.rank) + e),
                         "r"(__float_as_uint(v)), "r"(epoch)
                         : "memory");
}

// Element e of rank src's partials for this launch (bounded wait; on a timeout the window's
// error word is set and 0 returned, and later waits do not wait).
IAM_DEV float fused_recv(const TpWindow& w, unsigned epoch, int src, int e) {
    volatile unsigned* err = reinterpret_cast<volatile unsigned*>(w.base[w.rank] + w.err_off);
    const uint2* q = fused_slot(w, w.rank, epoch, src) + e;
    for (long long n = 0;; ++n) {
        uint2 v;
        asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(q) : "memory");
        if (v.y == epoch) return __uint_as_float(v.x);
        if (n > w.spin_limit || *err != 0u) {
            *err = 1u;
            return 0.0f;
        }
        if (n > 64) __nanosleep(32);
    }
}

// The dense stream of one CTA (tile = dense_rows output rows, range of rin <= 1024 inputs, rin a
// multiple of 8): a lane holds x and the selection masks of inputs 8*lane + 256c .. + 8 in
// registers; each warp takes output rows tile_begin + warp + 16j, reads the row's range with
// 16-byte loads, and adds x[i]*w for the weights whose rank bit is set in mask[i] -- the same
// weights a bucket-row selection picks (row r of input i holds, in each column group of 16
// outputs, the weight of rank r).  The weight value is the bucket word: the high 12 bits of the
// stored word with the output's slot (o mod 16) as the low 4 (bucketMul.cl:419-425).  Per row a
// lane adds its products in input order, then the warp sums the lanes (xor tree): the sum
// depends on the range only.  Writes the range's partial of each output.
template <int TPX>
IAM_DEV void dense_rows_stream(const BGProblem& pr, const float* xr, const uint16_t* mask, int rin, int i0, int tile,
                               int M, float* part, int warp, int lane, const BGBatch& b, unsigned fepoch,
                               int range) {
    constexpr int NCH = 4;
    float xv[NCH][8];
    uint32_t mk[NCH][4];
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
        const int k0 = 256 * c + 8 * lane;
        if (k0 < rin) {
            const float4 a = *reinterpret_cast<const float4*>(xr + k0);
            const float4 d = *reinterpret_cast<const float4*>(xr + k0 + 4);
            const uint4 m = *reinterpret_cast<const uint4*>(mask + k0);
            xv[c][0] = a.x; xv[c][1] = a.y; xv[c][2] = a.z; xv[c][3] = a.w;
            xv[c][4] = d.x; xv[c][5] = d.y; xv[c][6] = d.z; xv[c][7] = d.w;
            mk[c][0] = m.x; mk[c][1] = m.y; mk[c][2] = m.z; mk[c][3] = m.w;
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) xv[c][e] = 0.0f;
#pragma unroll
            for (int q = 0; q < 4; ++q) mk[c][q] = 0u;
        }
    }
    const int TO = pr.dense_rows;
    const int o_end = min(M, tile * TO + TO);
    const size_t ld = (size_t)pr.n_in;
    const uint16_t* base = pr.dense + (size_t)(i0 - pr.in_begin);
    // two rows per step (warp rows o and o + 16): both rows' loads are in flight together
    for (int o = tile * TO + warp; o < o_end; o += 2 * kGW) {
        const bool two = o + kGW < o_end;
        const uint4* row0 = reinterpret_cast<const uint4*>(base + (size_t)o * ld);
        const uint4* row1 = reinterpret_cast<const uint4*>(base + (size_t)(two ? o + kGW : o) * ld);
        uint4 w0[NCH], w1[NCH];
#pragma unroll
        for (int c = 0; c < NCH; ++c)
            if (256 * c + 8 * lane < rin) {
                w0[c] = __ldg(row0 + 32 * c + lane);
                w1[c] = __ldg(row1 + 32 * c + lane);
            }
        float acc0 = 0.0f, acc1 = 0.0f;
        const uint32_t slot0 = (uint32_t)(o & 15) * 0x10001u, slot1 = (uint32_t)((o + kGW) & 15) * 0x10001u;
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
            if (256 * c + 8 * lane >= rin) continue;
            const uint32_t a[4] = {w0[c].x, w0[c].y, w0[c].z, w0[c].w};
            const uint32_t d[4] = {w1[c].x, w1[c].y, w1[c].z, w1[c].w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t m2 = mk[c][q];  // masks of inputs 2q (low half) and 2q + 1 (high half)
                const float x0 = xv[c][2 * q], x1 = xv[c][2 * q + 1];
                {
                    const uint32_t v = (a[q] & 0xFFF0FFF0u) | slot0;
                    acc0 = fmaf(((m2 >> (a[q] & 15u)) & 1u) ? x0 : 0.0f, h2f(v & 0xffffu), acc0);
                    acc0 = fmaf(((m2 >> (16u + ((a[q] >> 16) & 15u))) & 1u) ? x1 : 0.0f, h2f(v >> 16), acc0);
                }
                {
                    const uint32_t v = (d[q] & 0xFFF0FFF0u) | slot1;
                    acc1 = fmaf(((m2 >> (d[q] & 15u)) & 1u) ? x0 : 0.0f, h2f(v & 0xffffu), acc1);
                    acc1 = fmaf(((m2 >> (16u + ((d[q] >> 16) & 15u))) & 1u) ? x1 : 0.0f, h2f(v >> 16), acc1);
                }
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, off);
            acc1 += __shfl_xor_sync(0xffffffffu, acc1, off);
        }
        if (lane == 0) {
            part[o] = acc0;
            if constexpr (TPX) {
                if (b.tp_fused) fused_send(b.tp, fepoch, range * M + o, acc0);
            }
            if (two) {
                part[o + kGW] = acc1;
                if constexpr (TPX) {
                    if (b.tp_fused) fused_send(b.tp, fepoch, range * M + o + kGW, acc1);
                }
            }
        }
    }
}

template <int ROWL, int XM, int DN, int TPX>
__global__ void __launch_bounds__(kGT, 1) bg_kernel(const __grid_constant__ BGBatch b) {
    constexpr int COLL = 32 / ROWL, NSETS = kGW * ROWL;
    static_assert(kChunk % NSETS == 0, "chunks keep the set of every row");
    int pi = 0;
    while (pi + 1 < b.nprob && (int)blockIdx.x >= b.p[pi + 1].cta_begin) ++pi;
    const BGProblem& pr = b.p[pi];
    const int local = (int)blockIdx.x - pr.cta_begin;
    const int tile = local % pr.n_tiles, range = local / pr.n_tiles;
    const int vec = pr.vec;
    const int TW = COLL * vec;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    long long* tr =
        (b.trace && tid == 0 && (int)blockIdx.x < b.trace_cap) ? b.trace + kTraceSlots * blockIdx.x : nullptr;
    debug_stamp(tr, 0);
    const long long clk0 = clock64();

    const int R = pr.n_ranges;
    const int i0 = pr.in_begin + (int)((long long)range * pr.n_in / R);
    const int i1 = pr.in_begin + (int)((long long)(range + 1) * pr.n_in / R);
    const int rin = i1 - i0;
    const int P = pr.P;
    const int M = 16 * pr.cols;

    extern __shared__ __align__(16) unsigned char smem_raw[];
    const GOffsets off = g_offsets(pr.range_max, b.stage_stats != 0);
    GHeader& h = *reinterpret_cast<GHeader*>(smem_raw);
    float* xall = reinterpret_cast<float*>(smem_raw + off.xall);
    float* xr = reinterpret_cast<float*>(smem_raw + off.xr);
    uint16_t* mask = reinterpret_cast<uint16_t*>(smem_raw + off.mask);
    int* pre = reinterpret_cast<int*>(smem_raw + off.pre);
    uint16_t* sts = reinterpret_cast<uint16_t*>(smem_raw + off.sts);
    uint2* list = reinterpret_cast<uint2*>(smem_raw + off.list);
    // per-warp accumulator regions aligned to their size in the shared window, so a slot's
    // bits can be OR-ed into the lane's address (acc_row)
    const uint32_t acc_sh0 = (uint32_t)__cvta_generic_to_shared(smem_raw + off.acc);
    const uint32_t acc_sh = (acc_sh0 + kRegion - 1) & ~(kRegion - 1);
    float* acc = reinterpret_cast<float*>(smem_raw + off.acc + (acc_sh - acc_sh0));
    // cutoff scratch inside the accumulators (they are cleared after the cutoff)
    int* hist = reinterpret_cast<int*>(acc);               // [kNB]
    int* start = hist + kNB;                              // [kNB + 1]
    int* cursor = start + kNB + 4;                        // [kNB]
    float* sorted = reinterpret_cast<float*>(cursor + kNB);  // [P]
    float* wbuf = sorted + kProbes;                          // [kWinMax]
    float* wsorted = wbuf + kWinMax;                         // [kWinMax]

    // ---- 0. prologue on weights only (nothing an earlier kernel of the stream writes)
    const uint16_t* st_src = pr.stats + (pr.row0 + 16LL * i0) * pr.stats_stride;
    const bool stage = b.stage_stats && rin > 0;
    if (tid == 0) {
        h.staged = 0;
        h.maxbin = 0;
        h.wn = 0;
        h.blo = 0;
        h.bhi = kNB - 1;
        if (stage) {
            mbar_init_cta(&h.bar);
            bulk_copy_g2s(sts, st_src, 32u * (uint32_t)rin, &h.bar);
        }
        if (((reinterpret_cast<uintptr_t>(pr.probes) & 15u) == 0) && (P % 8) == 0)
            prefetch_l2(pr.probes, (uint32_t)P * 2u);
    }
    if (!stage) {
        const long long sbytes = 32LL * rin * pr.stats_stride;
        if (((reinterpret_cast<uintptr_t>(st_src) & 15u) == 0))
            for (long long o = (long long)tid * 16384; o < sbytes; o += (long long)kGT * 16384)
                prefetch_l2(reinterpret_cast<const unsigned char*>(st_src) + o, (uint32_t)min(16384LL, sbytes - o) & ~15u);
    }
    for (int k = tid; k < kNB; k += kGT) hist[k] = 0;
    pdl_wait();  // from here on: x, residuals written by earlier kernels
    unsigned push_epoch = 0u;
    PullIn pin{nullptr, 0, 0, 0, 0u};
    if constexpr (TPX) {
        if (b.tp_fused && tid == 0)  // the previous fused launch's epoch, written after its barrier
            h.fepoch = *reinterpret_cast<const volatile unsigned*>(b.tp.base[b.tp.rank] + b.tp.fused_epoch_off) + 1u;
        // pushed inputs: this launch's epoch (the kind's consumed count + 1, read before the barrier)
        push_epoch =
            b.tp_push ? tp_push_epoch(b.tp, b.tp_push - 1) : (b.tp_wait ? tp_push_epoch(b.tp, b.tp_wait - 1) : 0u);
        if (b.tp_wait) pin = PullIn{&b.tp, b.tp_wait - 1, pr.in_begin, pr.in_begin + pr.n_in, push_epoch};
    }

    const auto xp = GProvider<XM, TPX>::make(pr, h.red, pin);

    // ---- 1. cutoff values: thread t owns x[8t, 8t + 8)
    float v[kVPT];
    unsigned mnb = 0x7f800000u, mxb = 0u;  // importances are >= +0: float order == bit order
    {
        const int j0 = tid * kVPT;
        if (P == kProbes && xp.aligned16() && ((reinterpret_cast<uintptr_t>(pr.probes) & 15u) == 0)) {
            const uint4 pb = __ldg(reinterpret_cast<const uint4*>(pr.probes + j0));
            float xv[8];
            xp.load8(j0, xv);
            const uint32_t pw[4] = {pb.x, pb.y, pb.z, pb.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const uint32_t hb = (e & 1) ? (pw[e >> 1] >> 16) : (pw[e >> 1] & 0xffffu);
                v[e] = importance(xv[e], h2f(hb));
                mnb = min(mnb, __float_as_uint(v[e]));
                mxb = max(mxb, __float_as_uint(v[e]));
            }
            *reinterpret_cast<float4*>(xall + j0) = make_float4(xv[0], xv[1], xv[2], xv[3]);
            *reinterpret_cast<float4*>(xall + j0 + 4) = make_float4(xv[4], xv[5], xv[6], xv[7]);
        } else {
#pragma unroll
            for (int k = 0; k < kVPT; ++k) {
                const int j = j0 + k;
                if (j < P) {
                    const float xv = xp(j);
                    xall[j] = xv;
                    v[k] = importance(xv, h2f(__ldg(pr.probes + j)));
                    mnb = min(mnb, __float_as_uint(v[k]));
                    mxb = max(mxb, __float_as_uint(v[k]));
                } else {
                    v[k] = -1.0f;  // no value: never binned, never counted
                }
            }
        }
    }
    mnb = __reduce_min_sync(0xffffffffu, mnb);
    mxb = __reduce_max_sync(0xffffffffu, mxb);
    if (lane == 0) {
        h.wmin[warp] = __uint_as_float(mnb);
        h.wmax[warp] = __uint_as_float(mxb);
    }
    __syncthreads();
    float mn = h.wmin[0], mx = h.wmax[0];
#pragma unroll
    for (int w = 1; w < kGW; ++w) {
        mn = fminf(mn, h.wmin[w]);
        mx = fmaxf(mx, h.wmax[w]);
    }
    debug_stamp(tr, 1);

    // ---- 2. cutoff: counting sort by bin, then the bisection on one bin per step
    float inv_w = mx > mn ? __fdiv_rn((float)kNB, __fsub_rn(mx, mn)) : 0.0f;
    if (!(inv_w < 3.0e38f)) inv_w = 0.0f;  // a vanishing range: one bin (monotone still)
    int bin[kVPT];
#pragma unroll
    for (int k = 0; k < kVPT; ++k) {
        bin[k] = v[k] >= 0.0f ? vbin(v[k], mn, inv_w) : -1;
        if (bin[k] >= 0) atomicAdd(&hist[bin[k]], 1);
    }
    __syncthreads();
    debug_stamp(tr, 8);
    {
        // start[b] = values in bins below b (2 bins per thread, block scan)
        constexpr int BPT = kNB / kGT;
        const int k0 = tid * BPT;
        int hv[BPT];
        int s = 0;
#pragma unroll
        for (int u = 0; u < BPT; ++u) {
            hv[u] = hist[k0 + u];
            s += hv[u];
        }
        int incl = s;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        if (lane == 31) h.wsum[warp] = incl;
        int mb = max(hv[0], hv[BPT - 1]);
        mb = __reduce_max_sync(0xffffffffu, mb);
        if (lane == 0) atomicMax(&h.maxbin, mb);
        __syncthreads();
        int run = incl - s;
        for (int w = 0; w < warp; ++w) run += h.wsum[w];
#pragma unroll
        for (int u = 0; u < BPT; ++u) {
            start[k0 + u] = run;
            cursor[k0 + u] = run;
            run += hv[u];
        }
        if (tid == kGT - 1) start[kNB] = run;
    }
    __syncthreads();
    debug_stamp(tr, 9);
    // The bisection's decisions depend on the values only through the 8 order statistics
    // d_{T-3} >= ... >= d_{T+4} around the target rank T (rank 1 = largest): for any tested
    // mid, count(mid) = (T - 4) + #{u : d_{T-3+u} > mid} is exact whenever it lies in
    // [T-3, T+3], and otherwise lands on the same side of every test of bucketMul.cl:150-198
    // (below target, equal to it, and bracket counts 3 or more apart).  Those statistics sit
    // in the bins covering ascending positions P-T-4 .. P-T+3; their values are gathered and
    // ranked, and one warp replays the bisection in registers.
    const int T = pr.target, nval = start[kNB];
    const int wlo = max(0, nval - T - 4), whi = min(nval - 1, nval - T + 3);
#pragma unroll
    for (int u = 0; u < kNB / kGT; ++u) {
        const int bb = tid * (kNB / kGT) + u;
        if (start[bb] <= wlo && wlo < start[bb + 1]) h.blo = bb;
        if (start[bb] <= whi && whi < start[bb + 1]) h.bhi = bb;
    }
    __syncthreads();
    const int blo = h.blo, bhi = h.bhi;
    const int w0 = start[blo], nw = start[bhi + 1] - w0;
    if (nw <= kWinMax) {
#pragma unroll
        for (int k = 0; k < kVPT; ++k)
            if (bin[k] >= blo && bin[k] <= bhi) wbuf[atomicAdd(&h.wn, 1)] = v[k];
        __syncthreads();
        for (int j = tid; j < nw; j += kGT) {  // rank among the gathered values (ties by slot)
            const float wj = wbuf[j];
            int r = 0;
            for (int i = 0; i < nw; ++i) {
                const float wi = wbuf[i];
                r += (wi < wj || (wi == wj && i < j)) ? 1 : 0;
            }
            wsorted[r] = wj;
        }
        __syncthreads();
        debug_stamp(tr, 10);
        if (warp == 0) {
            float d[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int pos = nval - (T - 3 + u);  // ascending position of d_{T-3+u}
                d[u] = pos > nval - 1 ? INFINITY : (pos < 0 ? -INFINITY : wsorted[pos - w0]);
            }
            float lo = mn, hi = mx, mid = bisect_mid(lo, hi);
            int minc = P, maxc = 0, it = 0;
            float result = mid;
            for (; it < kMaxIters;) {
                int c = T - 4;
#pragma unroll
                for (int u = 0; u < 8; ++u) c += d[u] > mid ? 1 : 0;  // ">" (bucketMul.cl:155)
                const bool below = c < T;
                hi = below ? mid : hi;
                maxc = below ? c : maxc;
                lo = below ? lo : mid;
                minc = below ? minc : c;
                const float next = bisect_mid(lo, hi);
                ++it;
                if ((c == T) | (__fsub_rn(hi, lo) < 1e-5f) | (abs(maxc - minc) < 3)) {
                    result = mid;
                    break;
                }
                mid = next;
                result = next;
            }
            if (lane == 0) {
                h.result = result;
                h.it = it;
            }
        }
    } else {
        // crowded bins: sort every value by bin and count each tested mid's own bin
#pragma unroll
        for (int k = 0; k < kVPT; ++k)
            if (bin[k] >= 0) sorted[atomicAdd(&cursor[bin[k]], 1)] = v[k];
        __syncthreads();
        debug_stamp(tr, 10);
        if (warp == 0) {
            // bucketMul.cl:139-213: count(mid) = values in bins above mid's bin + the values
            // of mid's bin above mid (">", :155); the update and stop rules of :150-213
            float lo = mn, hi = mx, mid = bisect_mid(lo, hi);
            int minc = P, maxc = 0, it = 0;
            float result = mid;
            for (; it < kMaxIters;) {
                const int bb = vbin(mid, mn, inv_w);
                const int s0 = start[bb], s1 = start[bb + 1];
                int c = 0;
                for (int j = s0 + lane; j < s1; j += 32) c += sorted[j] > mid ? 1 : 0;
                c = (nval - s1) + __reduce_add_sync(0xffffffffu, c);
                const bool below = c < T;
                hi = below ? mid : hi;
                maxc = below ? c : maxc;
                lo = below ? lo : mid;
                minc = below ? minc : c;
                const float next = bisect_mid(lo, hi);
                ++it;
                if ((c == T) | (__fsub_rn(hi, lo) < 1e-5f) | (abs(maxc - minc) < 3)) {
                    result = mid;
                    break;
                }
                mid = next;
                result = next;
            }
            if (lane == 0) {
                h.result = result;
                h.it = it;
            }
        }
    }
    __syncthreads();
    const float cutoff = h.result;
    const int iters = h.it;
    debug_stamp(tr, 2);

    // ---- 3. selection of the range's rows: masks, then a prefix over the inputs
    bool have_sts = false;
    if (stage) {
        have_sts = mbar_wait_bounded(&h.bar);
        if (!have_sts && tid == 0) h.staged = -1;  // read the stats from global memory instead
    }
    for (int k = tid; k < rin; k += kGT) {
        const int i = i0 + k;
        const float xi = i < P ? xall[i] : xp(i);
        xr[k] = xi;
        const int rmax = min(16, pr.n_rows_valid - 16 * i);
        unsigned m = 0u;
        if (pr.stats_stride == 1 && rmax == 16 && (have_sts || ((reinterpret_cast<uintptr_t>(st_src) & 15u) == 0))) {
            uint4 a, c;
            if (have_sts) {
                a = *reinterpret_cast<const uint4*>(sts + 16 * k);
                c = *reinterpret_cast<const uint4*>(sts + 16 * k + 8);
            } else {
                a = __ldg(reinterpret_cast<const uint4*>(st_src + 16 * k));
                c = __ldg(reinterpret_cast<const uint4*>(st_src + 16 * k + 8));
            }
            const uint32_t wds[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                const uint32_t hb = (r & 1) ? (wds[r >> 1] >> 16) : (wds[r >> 1] & 0xffffu);
                m |= (importance(xi, h2f(hb)) >= cutoff) ? (1u << r) : 0u;  // ">=" (bucketMul.cl:380)
            }
        } else {
            const uint16_t* sp = pr.stats + (pr.row0 + 16LL * i) * pr.stats_stride + (pr.stats_stride - 1);
            for (int r = 0; r < rmax; ++r)
                m |= (importance(xi, h2f(__ldg(sp + (size_t)r * pr.stats_stride))) >= cutoff) ? (1u << r) : 0u;
        }
        mask[k] = (uint16_t)m;
        if (pr.x_capture && tile == 0) pr.x_capture[i - pr.in_begin] = xi;
        pre[k] = __popc(m);
    }
    __syncthreads();
    {
        const int per = (rin + kGT - 1) / kGT;
        const int k0 = min(rin, tid * per), k1 = min(rin, k0 + per);
        int s = 0;
        for (int k = k0; k < k1; ++k) s += pre[k];
        int incl = s;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        if (lane == 31) h.wsum[warp] = incl;
        __syncthreads();
        int run = incl - s;
        for (int w = 0; w < warp; ++w) run += h.wsum[w];
        for (int k = k0; k < k1; ++k) {
            const int c = pre[k];
            pre[k] = run;
            run += c;
        }
        if (tid == kGT - 1) {
            pre[rin] = run;
            h.total = run;
        }
    }
    __syncthreads();
    const int S = h.total;
    debug_stamp(tr, 3);

    float* part = pr.partials + (size_t)range * M;
    if constexpr (DN) {
        dense_rows_stream<TPX>(pr, xr, mask, rin, i0, tile, M, part, warp, lane, b, h.fepoch, range);
        debug_stamp(tr, 4);
    } else {
    // ---- 4. accumulation: list position j goes to set j % NSETS = (warp, row lane)
    const int rl = lane / COLL, q = lane % COLL;
    const int col = tile * TW + q * vec;
    const bool col_ok = col < pr.cols;
    const uint16_t* __restrict__ wbase = pr.buckets + (col_ok ? col : 0);
    const uint32_t acc_lane = acc_sh + (uint32_t)warp * kRegion + (uint32_t)lane * 4u;
    float* my_acc = acc + (size_t)warp * (kRegion / 4) + lane;
#pragma unroll 4
    for (int j = 0; j < 16 * kVMax; ++j) my_acc[j * 32] = 0.0f;
    const long long rowbase = pr.row0 - pr.bucket_row0;  // list offsets are relative to buckets[0]
    const uint32_t cols_u = (uint32_t)pr.cols;
    for (int c0 = 0; c0 < S; c0 += kChunk) {
        const int n = min(kChunk, S - c0);
        // this chunk's rows: every thread writes the selected rows of its inputs that fall in it
        for (int k = tid; k < rin; k += kGT) {
            const int lo = pre[k], hi = pre[k + 1];
            if (hi <= c0 || lo >= c0 + n) continue;
            unsigned m = mask[k];
            const uint32_t xb = __float_as_uint(xr[k]);
            const long long r0 = rowbase + 16LL * (i0 + k);
            for (int j = lo; m; ++j) {
                const int r = __ffs(m) - 1;
                m &= m - 1u;
                if (j >= c0 && j < c0 + n) list[j - c0] = make_uint2((uint32_t)((r0 + r) * cols_u), xb);
            }
        }
        __syncthreads();
        const int first = warp * ROWL;
        const int mw = n > first ? (n - first + NSETS - 1) / NSETS : 0;  // rows of the warp's first set
        if (mw > 0) {
            const int j0 = first + rl;
            if (vec == 4) acc_chunk<4, NSETS>(list, n, j0, mw, wbase, acc_lane);
            else if (vec == 2) acc_chunk<2, NSETS>(list, n, j0, mw, wbase, acc_lane);
            else acc_chunk<1, NSETS>(list, n, j0, mw, wbase, acc_lane);
        }
        __syncthreads();
    }
    debug_stamp(tr, 4);

    // ---- 5. integrate: sets in order -> this CTA's partial of its tile.  A warp reads the 32
    // lanes' accumulators of one (slot, column) of every warp in turn (conflict free); the row
    // lanes of an output are then added in row-lane order.
    const int kOut = 16 * TW;
    for (int idx = tid; idx < 32 * 16 * vec; idx += kGT) {  // a multiple of 32: whole warps
        const int ln = idx & 31, pair = idx >> 5;
        const int e = pair % vec, slot = pair / vec;
        const int qq = ln % COLL;
        float s = 0.0f;
#pragma unroll
        for (int w2 = 0; w2 < kGW; ++w2) s += acc[(size_t)w2 * (kRegion / 4) + (slot * kVMax + e) * 32 + ln];
        const int o = (qq * vec + e) * 16 + slot;  // tile output index: column * 16 + slot
        if (ROWL == 2) {
            const float other = __shfl_down_sync(0xffffffffu, s, 16);  // row lane 1 of the same column
            s = s + other;
        }
        if (ln < COLL && tile * TW + o / 16 < pr.cols) {
            part[(size_t)tile * kOut + o] = s;
            if constexpr (TPX) {
                if (b.tp_fused) fused_send(b.tp, h.fepoch, range * M + tile * kOut + o, s);
            }
        }
    }
    }
    int* rows_of = reinterpret_cast<int*>(pr.partials + (size_t)R * M);
    if (tile == 0 && tid == 0) rows_of[range] = S;
    debug_stamp(tr, 5);
    if (b.partials_only) {  // the ranges are summed by the tensor-parallel exchange
        if (local == 0 && tid == 0) {
            if (pr.cutoff_out) *pr.cutoff_out = cutoff;
            if (pr.iters_out) *pr.iters_out = iters;
        }
        if (stage && !have_sts && tid == 0) mbar_wait_bounded(&h.bar);
        if (tr) {
            debug_stamp(tr, 6);
            tr[7] = S;
        }
        pdl_trigger();
        return;
    }
    grid_barrier(b.barrier);  // every partial of the launch is written
    debug_stamp(tr, 11);
    pdl_trigger();  // every CTA of this launch is past the barrier: the successor may start

    // ---- 6. this CTA's slice of the outputs: the partials added in range order
    const int nc = pr.n_tiles * R;
    const int o0 = (int)((long long)local * M / nc), o1 = (int)((long long)(local + 1) * M / nc);
    const int no = o1 - o0;
    float* red = acc;  // [kRedFloats]: partials staged so that all loads are in flight together
    if constexpr (!TPX) {
        const int per_pass = max(1, kRedFloats / R);
        for (int p0 = 0; p0 < no; p0 += per_pass) {
            const int pn = min(per_pass, no - p0);
            for (int k = tid; k < pn * R; k += kGT) {
                const int r = k / pn, oo = k - r * pn;
                red[oo * R + r] = __ldcg(pr.partials + (size_t)r * M + o0 + p0 + oo);
            }
            __syncthreads();
            for (int oo = tid; oo < pn; oo += kGT) {
                float s = 0.0f;
                for (int r = 0; r < R; ++r) s += red[oo * R + r];
                const int o = o0 + p0 + oo;
                if (pr.residual) s = pr.residual[o] + s;  // add32 (bucketMul.cl:517-520)
                pr.out[o] = s;
            }
            __syncthreads();
        }
    } else {
        // tp_fused: the ranges of every rank, rank r holding global ranges r * R .. r * R + R - 1
        // (this rank's from its partials, the others' from its mailbox, all loads first)
        const int RG = b.tp_fused ? R * b.tp.world : R;
        const int own = b.tp_fused ? b.tp.rank : 0;
        const int per_pass = max(1, kRedFloats / RG);
        for (int p0 = 0; p0 < no; p0 += per_pass) {
            const int pn = min(per_pass, no - p0);
            for (int k = tid; k < pn * R; k += kGT) {
                const int r = k / pn, oo = k - r * pn;
                red[oo * RG + own * R + r] = __ldcg(pr.partials + (size_t)r * M + o0 + p0 + oo);
            }
            if (b.tp_fused)
                for (int k = tid; k < pn * RG; k += kGT) {
                    const int g = k / pn, oo = k - g * pn;
                    const int owner = g / R;
                    if (owner != own) red[oo * RG + g] = fused_recv(b.tp, h.fepoch, owner, (g - owner * R) * M + o0 + p0 + oo);
                }
            __syncthreads();
            for (int oo = tid; oo < pn; oo += kGT) {
                float s = 0.0f;
                for (int r = 0; r < RG; ++r) s += red[oo * RG + r];
                const int o = o0 + p0 + oo;
                if (pr.residual) s = pr.residual[o] + s;  // add32 (bucketMul.cl:517-520)
                pr.out[o] = s;
                if (b.tp_push && pr.out_begin + o < b.push_limit)
                    tp_push_send(b.tp, b.tp_push - 1, (size_t)pi * b.tp.pmb_ffn + pr.out_begin + o, s, push_epoch);
            }
            __syncthreads();
        }
    }
    if (local == 0 && tid == 0) {
        if constexpr (TPX) {
            if (b.tp_fused && pi == 0)  // every CTA read the previous epoch before the barrier
                *reinterpret_cast<volatile unsigned*>(b.tp.base[b.tp.rank] + b.tp.fused_epoch_off) = h.fepoch;
            if (b.tp_wait && pi == 0) tp_push_consumed(b.tp, b.tp_wait - 1, push_epoch);  // (likewise)
        }
        int t = 0;
        for (int r = 0; r < R; ++r) t += __ldcg(rows_of + r);
        if (pr.count_out) *pr.count_out = t;
        if (pr.cutoff_out) *pr.cutoff_out = cutoff;
        if (pr.iters_out) *pr.iters_out = iters;
    }
    // a stats copy that did not land in time must not be left writing shared memory
    if (stage && !have_sts && tid == 0) mbar_wait_bounded(&h.bar);
    if (tr) {
        debug_stamp(tr, 6);
        tr[7] = S;
        tr[12] = h.maxbin;
        tr[13] = iters;
        tr[14] = h.staged;
        tr[15] = clock64() - clk0;  // SM cycles from [0] to [6]: the clock the stamps ran at
    }
}

template <int ROWL, int XM, int DN, int TPX>
cudaError_t bg_set_attrs() {
    static std::atomic<unsigned long long> done{0};
    return once_per_device(done, [] {
        return cudaFuncSetAttribute(bg_kernel<ROWL, XM, DN, TPX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    227 * 1024);
    });
}

template <int ROWL, int XM, int DN, int TPX>
int bg_launch_t(const BGBatch& b, int ctas, size_t smem, cudaStream_t s) {
    cudaError_t e = bg_set_attrs<ROWL, XM, DN, TPX>();
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(bg_kernel)");
    IAM_CUDA_TRY(launch_ex(bg_kernel<ROWL, XM, DN, TPX>, dim3((unsigned)ctas), dim3(kGT), smem, s, b.pdl != 0, b));
    return IAM_OK;
}

// The tensor-parallel exchanges (tp_fused, tp_push, tp_wait) live in their own instantiation:
// a one-GPU launch compiles none of their code.
template <int ROWL, int DN, int TPX>
int bg_launch_xt(const BGBatch& b, int ctas, size_t smem, cudaStream_t s) {
    switch (b.xmode) {
        case kXRms: return bg_launch_t<ROWL, kXRms, DN, TPX>(b, ctas, smem, s);
        case kXSilu: return bg_launch_t<ROWL, kXSilu, DN, TPX>(b, ctas, smem, s);
        default: return bg_launch_t<ROWL, kXPlain, DN, TPX>(b, ctas, smem, s);
    }
}

template <int ROWL, int DN>
int bg_launch_x(const BGBatch& b, int ctas, size_t smem, cudaStream_t s) {
    if (b.tp_fused || b.tp_push || b.tp_wait) return bg_launch_xt<ROWL, DN, 1>(b, ctas, smem, s);
    return bg_launch_xt<ROWL, DN, 0>(b, ctas, smem, s);
}

int bg_range_max(const BGBatch& b) {
    int m = 1;
    for (int i = 0; i < b.nprob; ++i) {
        const BGProblem& p = b.p[i];
        for (int r = 0; r < p.n_ranges; ++r)
            m = std::max(m, (int)((long long)(r + 1) * p.n_in / p.n_ranges) - (int)((long long)r * p.n_in / p.n_ranges));
    }
    return m;
}

int sm_count_current() {
    static std::mutex mu;
    static int cache[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lk(mu);
    if (!cache[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

// The widest columns per lane a problem's column count and buckets alignment allow.
int vec_cap(const BGProblem& p) {
    int v = kVMax;
    const uintptr_t a = reinterpret_cast<uintptr_t>(p.buckets);
    while (v > 1 && (p.cols % v != 0 || (a & (uintptr_t)(2 * v - 1)) != 0)) v >>= 1;
    return v;
}

}  // namespace

int bg_plan(BGBatch& b) {
    int begin = 0;
    for (int i = 0; i < b.nprob; ++i) {
        BGProblem& p = b.p[i];
        if (b.dense) {
            p.n_tiles = (16 * p.cols + p.dense_rows - 1) / p.dense_rows;
        } else {
            const int tw = (32 / b.rowl) * p.vec;
            p.n_tiles = (p.cols + tw - 1) / tw;
        }
        p.cta_begin = begin;
        begin += p.n_tiles * p.n_ranges;
    }
    const int rm = bg_range_max(b);
    for (int i = 0; i < b.nprob; ++i) b.p[i].range_max = rm;
    return begin;
}

size_t bg_smem_bytes(const BGBatch& b) { return g_offsets(bg_range_max(b), b.stage_stats != 0).total; }

// Input ranges of a dense launch over the whole matrix: the fewest that keep a range within
// 1024 inputs (the stream holds them in registers) in a multiple of 8; a multiple of 8 ranges
// for row-parallel matrices, so that every tensor-parallel rank holds whole ranges.  0: none.
int bg_dense_ranges(int full_in, bool row_parallel) {
    for (int r = 1; r <= kMaxRanges; ++r) {
        if (full_in % r) continue;
        const int rin = full_in / r;
        if (rin > 1024 || rin % 8) continue;
        if (row_parallel && r % 8) continue;
        return r;
    }
    return 0;
}

// Dense launches: ranges from the whole matrix (the sum order follows from them only), then
// tiles of output rows -- CTAs in proportion to each problem's work, one wave in total.
void bg_choose_shape_dense(BGBatch& b) {
    const int sms = sm_count_current();
    b.rowl = 1;
    double work = 0.0;
    for (int i = 0; i < b.nprob; ++i) work += 16.0 * b.p[i].cols * b.p[i].n_in;
    int total = 0;
    for (int i = 0; i < b.nprob; ++i) {
        BGProblem& p = b.p[i];
        const int fi = p.full_in > 0 ? p.full_in : p.n_in;
        const int rf = bg_dense_ranges(fi, p.fixed_ranges > 0);
        p.n_ranges = std::max(1, (int)((long long)rf * p.n_in / fi));
        p.vec = 1;
        const int M = 16 * p.cols;
        const double share = work > 0 ? 16.0 * p.cols * p.n_in / work : 1.0;
        int tiles = std::max(1, (int)(sms * share / p.n_ranges));
        p.dense_rows = ((M + tiles - 1) / tiles + 15) / 16 * 16;
        total += ((M + p.dense_rows - 1) / p.dense_rows) * p.n_ranges;
    }
    while (total > sms) {  // widen the tiles of the problem with the most CTAs
        int k = 0, kc = 0;
        for (int i = 0; i < b.nprob; ++i) {
            const int c = ((16 * b.p[i].cols + b.p[i].dense_rows - 1) / b.p[i].dense_rows) * b.p[i].n_ranges;
            if (c > kc) { kc = c; k = i; }
        }
        BGProblem& p = b.p[k];
        const int M = 16 * p.cols;
        const int t = (M + p.dense_rows - 1) / p.dense_rows;
        if (t == 1) break;
        p.dense_rows = ((M + t - 2) / (t - 1) + 15) / 16 * 16;
        total += (((M + p.dense_rows - 1) / p.dense_rows) - t) * p.n_ranges;
    }
    b.stage_stats = 1;
    for (int i = 0; i < b.nprob; ++i)
        if (b.p[i].stats_stride != 1 || (reinterpret_cast<uintptr_t>(b.p[i].stats) & 15u) || (b.p[i].row0 % 8))
            b.stage_stats = 0;
    if (bg_smem_bytes(b) > 227 * 1024) b.stage_stats = 0;
}

void bg_choose_shape(BGBatch& b) {
    if (b.dense) {
        bg_choose_shape_dense(b);
        return;
    }
    int widest = 0;
    for (int i = 0; i < b.nprob; ++i) widest = std::max(widest, b.p[i].full_cols > 0 ? b.p[i].full_cols : b.p[i].cols);
    b.rowl = widest >= 512 ? 1 : 2;
    const int sms = sm_count_current();
    // input ranges of the whole matrices: one GPU's wave
    double work = 0.0;
    int full_tiles[kGMaxProblems], full_r[kGMaxProblems];
    for (int i = 0; i < b.nprob; ++i) {
        const BGProblem& p = b.p[i];
        const int fc = p.full_cols > 0 ? p.full_cols : p.cols, fi = p.full_in > 0 ? p.full_in : p.n_in;
        full_tiles[i] = (fc + 32 / b.rowl * kVMax - 1) / (32 / b.rowl * kVMax);
        work += (double)fc * fi;
    }
    int total = 0;
    for (int i = 0; i < b.nprob; ++i) {
        const BGProblem& p = b.p[i];
        const int fc = p.full_cols > 0 ? p.full_cols : p.cols, fi = p.full_in > 0 ? p.full_in : p.n_in;
        const double share = work > 0 ? (double)fc * fi / work : 1.0;
        int r = (int)(sms * share / full_tiles[i]);
        full_r[i] = std::max(1, std::min(std::min(r, kMaxRanges), fi));
        total += full_r[i] * full_tiles[i];
    }
    while (total > sms) {  // a problem with more tiles than its share of the SMs
        int k = 0;
        for (int i = 1; i < b.nprob; ++i)
            if (full_r[i] * full_tiles[i] > full_r[k] * full_tiles[k]) k = i;
        if (full_r[k] == 1) break;
        full_r[k] -= 1;
        total -= full_tiles[k];
    }
    // this shard: its ranges, then tiles as wide as the vector loads allow, narrowed while the
    // launch still fits in one wave
    total = 0;
    int tiles[kGMaxProblems];
    for (int i = 0; i < b.nprob; ++i) {
        BGProblem& p = b.p[i];
        const int fi = p.full_in > 0 ? p.full_in : p.n_in;
        const int rf = p.fixed_ranges > 0 ? p.fixed_ranges : full_r[i];
        p.n_ranges = std::max(1, (int)((long long)rf * p.n_in / fi));
        p.vec = vec_cap(p);
        tiles[i] = (p.cols + (32 / b.rowl) * p.vec - 1) / ((32 / b.rowl) * p.vec);
        total += tiles[i] * p.n_ranges;
    }
    for (bool more = true; more;) {
        more = false;
        for (int i = 0; i < b.nprob; ++i) {
            BGProblem& p = b.p[i];
            if (p.vec == 1) continue;
            const int t2 = (p.cols + (32 / b.rowl) * (p.vec / 2) - 1) / ((32 / b.rowl) * (p.vec / 2));
            if (total + (t2 - tiles[i]) * p.n_ranges > sms) continue;
            if (t2 == tiles[i]) continue;
            total += (t2 - tiles[i]) * p.n_ranges;
            tiles[i] = t2;
            p.vec /= 2;
            more = true;
        }
    }
    // stage each range's stats in shared memory when the packed layout allows it
    b.stage_stats = 1;
    for (int i = 0; i < b.nprob; ++i)
        if (b.p[i].stats_stride != 1 || (reinterpret_cast<uintptr_t>(b.p[i].stats) & 15u) || (b.p[i].row0 % 8))
            b.stage_stats = 0;
    if (bg_smem_bytes(b) > 227 * 1024) b.stage_stats = 0;
}

int bg_launch(const BGBatch& b0, cudaStream_t s) {
    BGBatch b = b0;
    if (b.nprob < 1 || b.nprob > kGMaxProblems) return fail(IAM_ERR_ARG, "bucketmul: 1 to 3 problems per launch");
    if (b.rowl != 1 && b.rowl != 2) return fail(IAM_ERR_ARG, "bucketmul: row lanes must be 1 or 2");
    if (!b.barrier) return fail(IAM_ERR_ARG, "bucketmul: no barrier scratch");
    for (int i = 0; i < b.nprob; ++i) {
        const BGProblem& p = b.p[i];
        if (p.P < 1 || p.P > kProbes || p.cols < 1 || p.n_in < 1 || !p.partials)
            return fail(IAM_ERR_ARG, "bucketmul: empty problem or no partial scratch");
        if (p.vec < 1 || p.vec > kVMax || (p.vec & (p.vec - 1)) || p.cols % p.vec)
            return fail(IAM_ERR_ARG, "bucketmul: bad columns per lane");
        if (p.n_ranges < 1 || p.n_ranges > kMaxRanges || p.n_ranges > p.n_in)
            return fail(IAM_ERR_ARG, "bucketmul: bad input ranges");
        if ((long long)16 * (p.in_begin + p.n_in) * p.cols >= (1LL << 31))
            return fail(IAM_ERR_UNSUPPORTED, "bucketmul: rows * bucket_cols must stay below 2^31 elements");
        if (b.dense && (!p.dense || (reinterpret_cast<uintptr_t>(p.dense) & 15u) || p.n_in % p.n_ranges ||
                        (p.n_in / p.n_ranges) % 8 || p.n_in / p.n_ranges > 1024 || p.dense_rows < 16 ||
                        p.dense_rows % 16))
            return fail(IAM_ERR_ARG, "bucketmul: dense stream needs aligned rows and ranges of <= 1024 inputs "
                                     "(a multiple of 8)");
    }
    if ((b.tp_push || b.tp_wait) && (b.partials_only || b.tp.world < 2 || (b.tp_push && b.tp_wait)))
        return fail(IAM_ERR_ARG, "bucketmul: pushed inputs or outputs need the range reduction and a peer window");
    const int ctas = bg_plan(b);
    if (ctas > sm_count_current())
        return fail(IAM_ERR_UNSUPPORTED, "bucketmul: the launch needs more CTAs than SMs (one wave)");
    const size_t smem = bg_smem_bytes(b);
    if (smem > 227 * 1024) return fail(IAM_ERR_UNSUPPORTED, "bucketmul: an input range too large for shared memory");
    if (b.dense) return bg_launch_x<1, 1>(b, ctas, smem, s);
    if (b.rowl == 1) return bg_launch_x<1, 0>(b, ctas, smem, s);
    return bg_launch_x<2, 0>(b, ctas, smem, s);
}

}  // namespace iam
