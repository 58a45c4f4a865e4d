// iam_tp.h -- one-shot collectives of the tensor-parallel decode step over NVLink peer memory.
//
// Every rank holds one "window" allocation (the exchanged activations, a double-buffered
// mailbox of 8-byte {value, epoch} elements, per-CTA epochs, an error word); the peers map it
// through CUDA IPC.  A collective is one launch of kTpCtas CTAs: each element of this rank's
// data is stored, with the call's epoch beside it, into every peer's mailbox; each rank polls
// its own mailbox (bounded) until the epochs match.  No multicast, no NVLS: plain peer stores.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace iam {

constexpr int kTpMaxWorld = 8;
constexpr int kTpCtas = 32;      // CTAs of every collective launch (one epoch copy each)
constexpr int kTpThreads = 256;

struct TpWindow {
    char* base[kTpMaxWorld];  // every rank's window (base[rank] is this rank's own)
    int rank, world;
    size_t epoch_off;         // u32 [kTpCtas]: this rank's epoch per slice
    size_t err_off;           // u32: set when a wait gave up
    size_t mbox_off;          // uint2 [2][world][mbox_floats]: {value bits, epoch} from rank r
    int mbox_floats;          // elements per mailbox slot
    long long spin_limit;     // polls of one element before a wait gives up (kTpSpinLimit by default)
    // the mailbox of the exchanges done inside the bucketMul kernel (the o / down range
    // partials): uint2 [2][world][fused_floats], and the epoch of the last such launch (u32)
    size_t fused_off, fused_epoch_off;
    int fused_floats;
    // inputs pushed by their producing kernels (iam_tp_push.cuh): u32 [kTpPushKinds] epochs
    // consumed so far, and per kind a mailbox of uint2 {value bits, epoch}: the heads
    // [n_heads * head_dim], the gate/up values [2][pmb_ffn] (gate, then up)
    size_t xin_off;
    size_t pmb_off[2];
    int pmb_ffn;
};

// Kinds of pushed activations: the attention heads (o's input), the gate/up slices (down's).
constexpr int kTpPushHeads = 0, kTpPushFfn = 1, kTpPushKinds = 2;

// Default poll bound of a wait (~1 s on a B200 with the back-off of the poll loop).
constexpr long long kTpSpinLimit = 1LL << 21;

// Rank r's chunk [r*chunk, (r+1)*chunk) of the float buffer(s) at window offset off_a (and
// off_b unless it is SIZE_MAX) is copied to the same place in every peer.
int tp_allgather(const TpWindow& w, size_t off_a, size_t off_b, int chunk, cudaStream_t s, bool pdl);
// buf[0, n) at window offset off := sum over ranks, added in rank order (identical on all ranks).
int tp_allreduce_sum(const TpWindow& w, size_t off, int n, cudaStream_t s, bool pdl);
// out[0, M) := residual (may be null) + the sum of R = world * r_local range partials in range
// order, rank r holding ranges r * r_local .. (partials [r_local][M] floats, then r_local int row
// counts, in this rank's memory); identical on every rank and to one GPU's bucketMul sum.
// *count_out (may be null) := this rank's rows.
int tp_gather_reduce(const TpWindow& w, const float* partials, int M, int r_local, const float* residual, float* out,
                     int* count_out, cudaStream_t s, bool pdl);
// *key := max over ranks (the packed greedy argmax key).
int tp_keymax(const TpWindow& w, unsigned long long* key, cudaStream_t s, bool pdl);

}  // namespace iam
