// Three-phase exclusive scan of int32 counts into int64 offsets:
// (1) per-block sums, (2) one block scans the block sums, (3) per-block
// scan plus block offset. No inter-block waiting, so nothing can spin.
#include "internal.h"
#include "scan.cuh"

namespace t2sc {
namespace {
constexpr int kScanThreads = 256;
constexpr int kScanItems = 8;  // per thread
constexpr int kScanTile = kScanThreads * kScanItems;

__global__ void __launch_bounds__(kScanThreads) scan_reduce_kernel(const int32_t *__restrict__ in, int64_t n,
                                                                  int64_t *__restrict__ block_sums) {
  __shared__ int64_t sm[33];
  int64_t base = (int64_t)blockIdx.x * kScanTile + (int64_t)threadIdx.x * kScanItems;
  int64_t s = 0;
#pragma unroll
  for (int i = 0; i < kScanItems; i++)
    if (base + i < n) s += in[base + i];
  int64_t tot;
  block_exclusive_scan(s, sm, &tot);
  if (threadIdx.x == 0) block_sums[blockIdx.x] = tot;
}

__global__ void __launch_bounds__(1024) scan_blocks_kernel(int64_t *__restrict__ block_sums, int64_t nb,
                                                          int64_t *__restrict__ d_total) {
  __shared__ int64_t sm[33];
  int64_t carry = 0;
  for (int64_t b0 = 0; b0 < nb; b0 += blockDim.x) {
    int64_t i = b0 + threadIdx.x;
    int64_t v = i < nb ? block_sums[i] : 0;
    int64_t tot;
    int64_t ex = block_exclusive_scan(v, sm, &tot);
    if (i < nb) block_sums[i] = carry + ex;
    carry += tot;
  }
  if (threadIdx.x == 0 && d_total) *d_total = carry;
}

__global__ void __launch_bounds__(kScanThreads) scan_apply_kernel(const int32_t *__restrict__ in, int64_t n,
                                                                 const int64_t *__restrict__ block_offs,
                                                                 int64_t *__restrict__ out) {
  __shared__ int64_t sm[33];
  int64_t base = (int64_t)blockIdx.x * kScanTile + (int64_t)threadIdx.x * kScanItems;
  int32_t v[kScanItems];
  int64_t s = 0;
#pragma unroll
  for (int i = 0; i < kScanItems; i++) {
    v[i] = base + i < n ? in[base + i] : 0;
    s += v[i];
  }
  int64_t tot;
  int64_t ex = block_exclusive_scan(s, sm, &tot) + block_offs[blockIdx.x];
#pragma unroll
  for (int i = 0; i < kScanItems; i++) {
    if (base + i < n) out[base + i] = ex;
    ex += v[i];
  }
}
}  // namespace

int scan_counts(t2sc_ctx *ctx, const int32_t *in, int64_t n, int64_t *out, int64_t *d_total) {
  std::string &err = ctx->last_error;
  if (n <= 0) {
    if (d_total) T2SC_CUDA(cudaMemsetAsync(d_total, 0, sizeof(int64_t), ctx->stream), "scan memset");
    return T2SC_OK;
  }
  int64_t nb = (n + kScanTile - 1) / kScanTile;
  int64_t *bs = nullptr;
  T2SC_CUDA(cudaMallocAsync((void **)&bs, nb * sizeof(int64_t), ctx->stream), "scan scratch");
  scan_reduce_kernel<<<(unsigned)nb, kScanThreads, 0, ctx->stream>>>(in, n, bs);
  T2SC_LAUNCHED(ctx, "scan_reduce");
  scan_blocks_kernel<<<1, 1024, 0, ctx->stream>>>(bs, nb, d_total);
  T2SC_LAUNCHED(ctx, "scan_blocks");
  scan_apply_kernel<<<(unsigned)nb, kScanThreads, 0, ctx->stream>>>(in, n, bs, out);
  T2SC_LAUNCHED(ctx, "scan_apply");
  T2SC_CUDA(cudaFreeAsync(bs, ctx->stream), "scan scratch free");
  return T2SC_OK;
}

int scan_counts_into(t2sc_ctx *ctx, const int32_t *in, int64_t n, int64_t *out, int64_t *d_total,
                     int64_t *block_sums) {
  static_assert(kScanTile == kScanTileItems, "scan tile size");
  std::string &err = ctx->last_error;
  if (n <= 0) {
    if (d_total) T2SC_CUDA(cudaMemsetAsync(d_total, 0, sizeof(int64_t), ctx->stream), "scan memset");
    return T2SC_OK;
  }
  const int64_t nb = scan_block_count(n);
  scan_reduce_kernel<<<(unsigned)nb, kScanThreads, 0, ctx->stream>>>(in, n, block_sums);
  T2SC_LAUNCHED(ctx, "scan_reduce");
  scan_blocks_kernel<<<1, 1024, 0, ctx->stream>>>(block_sums, nb, d_total);
  T2SC_LAUNCHED(ctx, "scan_blocks");
  scan_apply_kernel<<<(unsigned)nb, kScanThreads, 0, ctx->stream>>>(in, n, block_sums, out);
  T2SC_LAUNCHED(ctx, "scan_apply");
  return T2SC_OK;
}

}  // namespace t2sc
