// peer_sync.cuh -- device side of the peer-memory all-gather (cfi_peer.h): a rank's signals to its
// peers and its bounded wait for theirs.
//
// Every launch of a rank adds exactly CFI_PEER_UNIT to its slot on each peer: each CTA, once its
// stores are visible at system scope (one fence by thread 0 after the CTA barrier; the fence is
// cumulative), adds 1 (CTA 0 adds CFI_PEER_UNIT - ctas + 1), so a slot reaches the next multiple
// of CFI_PEER_UNIT only after every CTA of the peer's launch has signalled.  A wait polls this
// rank's slots with relaxed system-scope loads, bounded by %globaltimer, and ends with a
// system-scope fence: the fence-fence synchronisation of the PTX memory model (release pattern on
// each signalling CTA, acquire pattern on the waiting thread).  Counters wrap modulo 2^32.
#pragma once
#include "cfi_common.cuh"
#include "cfi_kernels.h"
#include "sm100_ptx.cuh"

constexpr unsigned int CFI_PEER_ERR = 0x9e0000u;  // | rank of the peer that was given up on
constexpr unsigned int CFI_PEER_UNIT = 65536u;    // a launch's total signal (CTAs per launch below it)

CFI_DEV void peer_fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

CFI_DEV unsigned int peer_ld_relaxed(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Thread 0 of a CTA, after the CTA barrier that follows its stores: adds this CTA's share of the
// launch's signal to this rank's slot on every peer (ranks in turn from this one).
CFI_DEV void peer_signal_cta(const CfiPeerDev& p, unsigned int ctas, bool first_cta) {
    peer_fence_sys();
    const unsigned int add = first_cta ? CFI_PEER_UNIT - ctas + 1u : 1u;
    for (int i = 1; i < p.world; i++) {
        const int r = p.rank + i < p.world ? p.rank + i : p.rank + i - p.world;
        asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p.sig_remote[r]), "r"(add) : "memory");
    }
}

// One thread: wait until every other rank r's slot has reached expect[r] + CFI_PEER_UNIT (its
// next launch has signalled in full), then count the wait.  A peer that has not signalled
// within p.limit_ns records CFI_PEER_ERR | r; once such a code is in the error word, later
// waits do not wait out the limit again.
CFI_DEV void peer_wait_all(const CfiPeerDev& p, unsigned int* err) {
    const bool gave_up = ((*(volatile unsigned int*)err) >> 16) == (CFI_PEER_ERR >> 16);
    for (int i = 1; i < p.world; i++) {
        const int r = p.rank + i < p.world ? p.rank + i : p.rank + i - p.world;
        const unsigned int want = p.expect[r] + CFI_PEER_UNIT;
        const uint64_t t0 = sm100::globaltimer();
        for (uint32_t it = 0; !gave_up && (int)(peer_ld_relaxed(p.sig_local + r) - want) < 0; it++) {
            if ((it & 15u) == 15u && sm100::globaltimer() - t0 > p.limit_ns) {
                cfi_set_error(err, CFI_PEER_ERR | (unsigned int)r);
                break;
            }
        }
        p.expect[r] = want;
    }
    // acquire: the peers' stores before their signals are visible to what follows (in this
    // launch's completion, to the kernels after it)
    peer_fence_sys();
}
