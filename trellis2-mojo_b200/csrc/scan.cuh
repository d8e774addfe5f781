// Warp- and block-level exclusive scans (shuffle-based), shared by the
// neighbour-map exports and the subdivision compaction.
#pragma once
#include <stdint.h>

namespace t2sc {

// Inclusive warp scan of a 64-bit value across the 32 lanes.
__device__ __forceinline__ int64_t warp_inclusive_scan(int64_t v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    int64_t u = __shfl_up_sync(0xffffffffu, v, d);
    if (lane >= d) v += u;
  }
  return v;
}

// Exclusive block scan (blockDim.x a multiple of 32, <= 1024). `smem` holds
// 33 int64 (32 warp offsets + the block total). Returns the exclusive prefix of this thread; *total = block sum.
__device__ __forceinline__ int64_t block_exclusive_scan(int64_t v, int64_t *smem, int64_t *total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  int64_t inc = warp_inclusive_scan(v);
  if (lane == 31) smem[wid] = inc;
  __syncthreads();
  if (wid == 0) {
    int64_t s = lane < nw ? smem[lane] : 0;
    int64_t si = warp_inclusive_scan(s);
    if (lane < nw) smem[lane] = si - s;  // exclusive warp offsets
    if (lane == nw - 1) smem[32] = si;   // block total
  }
  __syncthreads();
  int64_t res = smem[wid] + inc - v;
  int64_t tot = smem[32];
  __syncthreads();
  *total = tot;
  return res;
}

}  // namespace t2sc
