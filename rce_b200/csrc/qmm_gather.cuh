// qmm_gather.cuh -- device side of the fused all-gather over peer memory.
// A row-sharded matmul writes its output rows into its own y and, as 8-byte
// words {value, epoch}, straight into every other rank's receive buffer
// (NVLink stores to peer-mapped memory).  An aligned 8-byte store arrives
// whole, so a receiver that reads a word carrying the epoch it expects has
// that value: no fence, counter or flag is needed on the sending side, and
// the receiver's bounded wait is per word.  Epochs only grow.
#pragma once
#include <cuda_runtime.h>

#include "qmm_internal.h"

namespace rce {

__device__ __forceinline__ unsigned gather_epoch(const GatherArgs &ga) {
    return ga.epoch_base ? ga.epoch + *reinterpret_cast<const volatile unsigned *>(ga.epoch_base) : ga.epoch;
}

__device__ __forceinline__ unsigned long long ll_word(float v, unsigned epoch) {
    return ((unsigned long long)epoch << 32) | (unsigned long long)__float_as_uint(v);
}

// The value at offset `off` (row-major, leading dimension ldy) to every
// other rank's receive buffer.
__device__ __forceinline__ void gather_send(const GatherArgs &ga, size_t off, float v, unsigned epoch) {
    const unsigned long long w = ll_word(v, epoch);
    for (int r = 0; r < ga.world; r++)
        if (r != ga.rank) *reinterpret_cast<volatile unsigned long long *>(ga.ll[r] + off) = w;
}

}  // namespace rce
