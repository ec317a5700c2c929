// Block-wide exclusive scan and the scan of per-block totals, shared by the kernels that
// write variable-length output in a sequential loop's order (subdivide, mesh extraction):
// count per block, scan the block totals, then each block rescans and writes.
#pragma once

#include <cstdint>

namespace tb_scan {

// Exclusive scan of one value per thread across a block of kThreads threads; *total = the
// block's sum. Every thread of the block must call it.
template <int kThreads>
__device__ __forceinline__ int64_t block_exclusive_scan(int64_t v, int64_t* total) {
    static_assert(kThreads % 32 == 0 && kThreads <= 1024, "block size");
    __shared__ int64_t warp_sums[kThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int64_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int64_t s = lane < kThreads / 32 ? warp_sums[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int64_t y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        if (lane < kThreads / 32) warp_sums[lane] = s;   // inclusive
    }
    __syncthreads();
    const int64_t warp_off = warp > 0 ? warp_sums[warp - 1] : 0;
    *total = warp_sums[kThreads / 32 - 1];
    __syncthreads();
    return warp_off + x - v;
}

// One block of kThreads: exclusive scan of the nb block totals in place; *grand = their sum.
template <int kThreads, int kPer>
__global__ void k_scan_block_totals(int64_t* __restrict__ sums, int64_t nb, int64_t* __restrict__ grand) {
    int64_t carry = 0;
    for (int64_t base = 0; base < nb; base += (int64_t)kThreads * kPer) {
        int64_t v[kPer];
        int64_t s = 0;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int64_t k = base + (int64_t)threadIdx.x * kPer + j;
            v[j] = k < nb ? sums[k] : 0;
            s += v[j];
        }
        int64_t total;
        int64_t off = block_exclusive_scan<kThreads>(s, &total) + carry;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int64_t k = base + (int64_t)threadIdx.x * kPer + j;
            if (k < nb) sums[k] = off;
            off += v[j];
        }
        carry += total;
    }
    if (threadIdx.x == 0) *grand = carry;
}

}  // namespace tb_scan
