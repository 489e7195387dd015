// ep_signal.cuh -- arrival signalling of the expert-parallel exchange.
//
// Every kernel that writes into other ranks' memory (dispatch, return, the
// combine that returns partial sums) runs a grid of CTAs that stride over
// the rows, each CTA writing rows for any destination.  A CTA, after all of
// its stores, fences them system-wide once and counts itself on a local
// per-phase counter; the CTA that completes the count (the launch's grid
// size) resets the counter for the next forward and raises every peer's
// flag for (phase, this rank) by one, after a second system fence.  The
// fences and the counter form a release/acquire chain from every CTA's
// stores to each flag increment, so a waiting rank that observes its flag
// (acquire) sees all of them.  One fence per CTA and one remote atomic per
// peer and phase per forward; a flag holds the number of forwards whose
// phase has arrived from that rank.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace qmoe {

QMOE_DEV int *ep_flag(const EpPeerDev &d, int owner, int phase, int from) {
    return reinterpret_cast<int *>(d.base[owner] + d.off_flags) + phase * d.world + from;
}

// Called by one thread of each of the launch's `units` CTAs, after a CTA
// barrier that follows all of the CTA's stores into peer memory.
QMOE_DEV void ep_signal_all(const EpPeerDev &d, int phase, int units) {
    __threadfence_system();
    int *cnt = d.cnt + phase * kEpMaxWorld;
    if (atomicAdd(cnt, 1) == units - 1) {
        *cnt = 0;                                  // no CTA of this launch touches it again
        __threadfence_system();
        for (int dst = 0; dst < d.world; ++dst)
            if (dst != d.rank) atomicAdd_system(ep_flag(d, dst, phase, d.rank), 1);
    }
}

}  // namespace qmoe
