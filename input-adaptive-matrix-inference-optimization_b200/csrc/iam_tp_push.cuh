// iam_tp_push.cuh -- activations pushed into the peers' windows by the kernel that makes them.
//
// Under tensor parallelism the o and down launches of every rank read, for their cutoff, the
// first P inputs of the whole matrix: all attention heads (o) and the leading gate/up values
// (down), most of them made on other ranks.  Instead of an all-gather launch between producer
// and consumer, the producing kernel (attention, the gate/up bucketMul) stores each such
// output element, as one 8-byte {value bits, epoch} store, into every peer's push mailbox; the
// consuming bucketMul reads the elements it needs that other ranks made from its own mailbox,
// polling each (bounded) until it carries the awaited epoch.  No flag and no fence: an aligned
// 8-byte store is seen whole.
//
// Epochs: the consumer of a kind records, after its range reduction, how many inputs of that
// kind it has consumed (u32 at xin_off + 4 * kind); the next producer of the kind on this
// rank runs after that consumer (stream order) and tags its elements with that count + 1, and
// the next consumer awaits the same count + 1.  Every rank runs the same sequence, so the
// counts agree.  One mailbox per kind suffices: a rank pushes layer l + 1's elements only
// after its o or down of layer l has finished, which needed every peer's range partials of
// that launch; a peer sends those after it has read its inputs, so no peer still reads the
// elements being overwritten, and stale elements carry an older epoch.
#pragma once

#include "iam_common.cuh"
#include "iam_tp.h"

namespace iam {

IAM_DEV unsigned* tp_consumed(const TpWindow& w) { return reinterpret_cast<unsigned*>(w.base[w.rank] + w.xin_off); }

// The epoch of this rank's next pushed inputs of `kind` (produced and consumed alike).
IAM_DEV unsigned tp_push_epoch(const TpWindow& w, int kind) {
    return reinterpret_cast<const volatile unsigned*>(tp_consumed(w))[kind] + 1u;
}

IAM_DEV uint2* tp_push_mbox(const TpWindow& w, int owner, int kind) {
    return reinterpret_cast<uint2*>(w.base[owner] + w.pmb_off[kind]);
}

// Element idx of `kind` to every peer's mailbox.
IAM_DEV void tp_push_send(const TpWindow& w, int kind, size_t idx, float v, unsigned epoch) {
    for (int p = 0; p < w.world; ++p)
        if (p != w.rank)
            asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(tp_push_mbox(w, p, kind) + idx),
                         "r"(__float_as_uint(v)), "r"(epoch)
                         : "memory");
}

// Element idx of `kind` made by another rank (bounded wait; on a timeout the window's error
// word is set and 0 returned, and later waits of this rank do not wait).
IAM_DEV float tp_push_recv(const TpWindow& w, int kind, size_t idx, unsigned epoch) {
    const uint2* q = tp_push_mbox(w, w.rank, kind) + idx;
    volatile unsigned* err = reinterpret_cast<volatile unsigned*>(w.base[w.rank] + w.err_off);
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

// The consumer's record, by one thread once every CTA of the launch has read the old count.
IAM_DEV void tp_push_consumed(const TpWindow& w, int kind, unsigned epoch) {
    reinterpret_cast<volatile unsigned*>(tp_consumed(w))[kind] = epoch;
}

}  // namespace iam
