// ep_signal.cuh -- arrival signalling of the expert-parallel exchange.
//
// Every kernel that writes into another rank's memory (dispatch, return,
// the combine that returns partial sums) is made of units -- CTAs or work
// tasks -- each of which writes part of what goes to one destination rank.
// A unit, after its stores, fences them system-wide and counts itself on a
// local per-(phase, destination) counter; the unit that completes the count
// (the number of units writing to that destination in this launch) resets
// the counter for the next forward and raises the destination's flag for
// (phase, this rank) by one with a system-scope release.  The fences and the
// counter form a release/acquire chain from every unit's stores to that one
// flag increment, so a waiting rank that observes the flag (acquire) sees
// all of them.  One remote atomic per destination and phase per forward,
// instead of one per row; a flag holds the number of forwards whose phase
// has arrived from that rank.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace qmoe {

QMOE_DEV int *ep_flag(const EpPeerDev &d, int owner, int phase, int from) {
    return reinterpret_cast<int *>(d.base[owner] + d.off_flags) + phase * d.world + from;
}

// Called by one thread of a unit after the unit's stores to rank dst (dst !=
// this rank) are issued; `units` = the launch's units writing to dst.
QMOE_DEV void ep_signal(const EpPeerDev &d, int dst, int phase, int units) {
    __threadfence_system();
    int *cnt = d.cnt + phase * kEpMaxWorld + dst;
    if (atomicAdd(cnt, 1) == units - 1) {
        *cnt = 0;                                  // no unit of this launch touches it again
        __threadfence_system();
        atomicAdd_system(ep_flag(d, dst, phase, d.rank), 1);
    }
}

}  // namespace qmoe
