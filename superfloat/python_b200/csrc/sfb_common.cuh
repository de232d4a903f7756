// Shared device helpers of libsfb200 (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "sfb200.h"

namespace sfb {

// Width constants: M = 2^(N-1) - 1 the largest code, sh = N - 1 so that one
// unit is 2^sh (src/sf/_format.py:40-48).
struct Width {
    int bits, sh, M;
};

__host__ __device__ inline Width width(int bits) { return Width{bits, bits - 1, (1 << (bits - 1)) - 1}; }

__device__ __forceinline__ int clampi(int v, int lo, int hi) { return min(max(v, lo), hi); }

// trunc(p / 2^sh), rounding toward zero.
__device__ __forceinline__ int tdiv_pow2(int p, int sh) {
    const int bias = (p >> 31) & ((1 << sh) - 1);
    return (p + bias) >> sh;
}

// Event counters of one thread, reduced per warp, then per block in shared
// memory, then added to the caller's sfb_counts with one atomic per counter.
struct Counts {
    unsigned over = 0, under = 0, div0 = 0, inval = 0, clip = 0;
};

__device__ __forceinline__ void flush_counts(const Counts &c, sfb_counts *g, unsigned *smem5) {
    const unsigned lane = threadIdx.x & 31;
    const unsigned o = __reduce_add_sync(0xffffffffu, c.over);
    const unsigned u = __reduce_add_sync(0xffffffffu, c.under);
    const unsigned d = __reduce_add_sync(0xffffffffu, c.div0);
    const unsigned v = __reduce_add_sync(0xffffffffu, c.inval);
    const unsigned k = __reduce_add_sync(0xffffffffu, c.clip);
    if (lane == 0) {
        if (o) atomicAdd(&smem5[0], o);
        if (u) atomicAdd(&smem5[1], u);
        if (d) atomicAdd(&smem5[2], d);
        if (v) atomicAdd(&smem5[3], v);
        if (k) atomicAdd(&smem5[4], k);
    }
    __syncthreads();
    if (threadIdx.x == 0 && g != nullptr) {
        if (smem5[0]) atomicAdd(&g->overflow, (unsigned long long)smem5[0]);
        if (smem5[1]) atomicAdd(&g->underflow, (unsigned long long)smem5[1]);
        if (smem5[2]) atomicAdd(&g->divide, (unsigned long long)smem5[2]);
        if (smem5[3]) atomicAdd(&g->invalid, (unsigned long long)smem5[3]);
        if (smem5[4]) atomicAdd(&g->acc_clipped, (unsigned long long)smem5[4]);
    }
}

__device__ __forceinline__ void zero_counts_smem(unsigned *smem5) {
    if (threadIdx.x < 5) smem5[threadIdx.x] = 0;
    __syncthreads();
}

// Host side: error reporting into a per-thread message buffer.
int set_error(int code, const char *fmt, ...);
int check_launch(const char *what);
int sm_count();

// A number naming the calling thread's current CUDA context for the life of
// the process (the driver's cuCtxGetId): the context that replaces one torn
// down by a device reset gets a new number, so per-device set-up cached
// under it (kernel attributes, a static array's device address) is redone
// rather than reused.  0 when no context is current yet.
unsigned long long context_id();

}  // namespace sfb
