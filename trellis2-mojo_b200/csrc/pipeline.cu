// Pipeline glue on the device around the decoder: the FlexiDualGrid head
// and the 1024 cascade's coordinate quantisation.
//
//  * fdg_head (trellis2_mojo/models/sc_vaes/fdg_vae.mojo:17-50): decoded
//    [T, 7] f32 features -> vertices [T, 3] = (1 + 2m) * sigmoid(f[0:3]) - m,
//    intersected [T, 3] = (f[3:6] > 0) as 1.0 / 0.0, quad_lerp [T, 1] =
//    softplus(f[6]) (f itself above 20). One thread per row.
//  * cascade_coords (trellis2_mojo/pipelines/image_to_3d.mojo:219-270):
//    q = int((xyz + 0.5) / lr_resolution * (hr_resolution / 16)) in f32,
//    rows (b, q) deduplicated and sorted lexicographically; hr_resolution
//    drops by 128 until the token count is below the budget or it is 1024.
//    Keys ((b*m + qx)*m + qy)*m + qz with m = max q + 1 order rows exactly
//    lexicographically; they are radix-sorted, unique keys flagged and
//    compacted with the library's scan. One host read-back per iteration
//    (max q and batch, then the token count): the loop's exit depends on it.
#include <cub/device/device_radix_sort.cuh>

#include "internal.h"

namespace t2sc {
namespace {

inline unsigned nblocks(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }

__global__ void fdg_head_kernel(const float *__restrict__ f, int64_t t, float m, float *__restrict__ vert,
                                float *__restrict__ inter, float *__restrict__ quad) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= t) return;
  const float *row = f + 7 * r;
  const float scale = __fadd_rn(1.f, __fmul_rn(2.f, m));
#pragma unroll
  for (int c = 0; c < 3; c++)
    vert[3 * r + c] = __fsub_rn(__fdiv_rn(scale, __fadd_rn(1.f, expf(-row[c]))), m);
#pragma unroll
  for (int c = 0; c < 3; c++) inter[3 * r + c] = row[3 + c] > 0.f ? 1.f : 0.f;
  const float q = row[6];
  quad[r] = q > 20.f ? q : logf(__fadd_rn(1.f, expf(q)));
}

// q per row and axis, plus the largest q and batch index (for the key radix)
// and a flag for negative inputs, which the key packing does not take.
__global__ void __launch_bounds__(256) cascade_quant_kernel(const int4 *__restrict__ c, int64_t n, float lr, float k,
                                     int4 *__restrict__ q, int *__restrict__ maxima, int *err) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int mq = 0, mb = 0;  // every lane reaches the warp reduction below
  if (r < n) {
    const int4 v = c[r];
    if (v.x < 0 || v.y < 0 || v.z < 0 || v.w < 0) {
      atomicOr(err, kDevErrRange);
    } else {
      int4 o;
      o.x = v.x;
      o.y = (int)__fmul_rn(__fdiv_rn(__fadd_rn((float)v.y, 0.5f), lr), k);
      o.z = (int)__fmul_rn(__fdiv_rn(__fadd_rn((float)v.z, 0.5f), lr), k);
      o.w = (int)__fmul_rn(__fdiv_rn(__fadd_rn((float)v.w, 0.5f), lr), k);
      q[r] = o;
      mq = max(o.y, max(o.z, o.w));
      mb = o.x;
    }
  }
  // one atomic pair per block: same-address atomics serialise in L2
  __shared__ int wq[8], wb[8];
  mq = __reduce_max_sync(0xffffffffu, mq);
  mb = __reduce_max_sync(0xffffffffu, mb);
  if ((threadIdx.x & 31) == 0) wq[threadIdx.x >> 5] = mq, wb[threadIdx.x >> 5] = mb;
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = blockDim.x >> 5;
    mq = __reduce_max_sync(0xffffffffu, threadIdx.x < nw ? wq[threadIdx.x] : 0);
    mb = __reduce_max_sync(0xffffffffu, threadIdx.x < nw ? wb[threadIdx.x] : 0);
    if (threadIdx.x == 0) {
      atomicMax(&maxima[0], mq);
      atomicMax(&maxima[1], mb);
    }
  }
}

__global__ void cascade_key_kernel(const int4 *__restrict__ q, int64_t n, uint64_t m, uint64_t *__restrict__ keys) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  const int4 v = q[r];
  keys[r] = (((uint64_t)v.x * m + (uint64_t)v.y) * m + (uint64_t)v.z) * m + (uint64_t)v.w;
}

__global__ void unique_flag_kernel(const uint64_t *__restrict__ keys, int64_t n, int32_t *__restrict__ flag) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  flag[r] = (r == 0 || keys[r] != keys[r - 1]) ? 1 : 0;
}

__global__ void cascade_emit_kernel(const uint64_t *__restrict__ keys, const int32_t *__restrict__ flag,
                                    const int64_t *__restrict__ pos, int64_t n, uint64_t m, int4 *__restrict__ out) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n || !flag[r]) return;
  uint64_t key = keys[r];
  int4 o;
  o.w = (int)(key % m);
  key /= m;
  o.z = (int)(key % m);
  key /= m;
  o.y = (int)(key % m);
  o.x = (int)(key / m);
  out[pos[r]] = o;
}

struct Scratch {
  void *p = nullptr;
  cudaStream_t st = nullptr;
  ~Scratch() {
    if (p) cudaFreeAsync(p, st);
  }
};

}  // namespace

int fdg_head_device(t2sc_ctx *ctx, const float *feats, int64_t t, float margin, float *vertices, float *intersected,
                    float *quad, std::string &err) {
  if (t == 0) return T2SC_OK;
  fdg_head_kernel<<<nblocks(t, 256), 256, 0, ctx->stream>>>(feats, t, margin, vertices, intersected, quad);
  T2SC_LAUNCHED(ctx, "fdg_head");
  return T2SC_OK;
}

int cascade_coords_device(t2sc_ctx *ctx, const int32_t *hr_coords, int64_t n, int lr_resolution, int resolution,
                          int64_t max_num_tokens, int32_t *out_coords, int64_t *num_tokens, int *hr_resolution,
                          std::string &err) {
  cudaStream_t st = ctx->stream;
  *num_tokens = 0;
  *hr_resolution = resolution;
  if (n == 0) return T2SC_OK;
  // scratch: q [n] int4 | keys in/out [n] u64 x 2 | flags [n] i32 | pos [n] i64 | maxima, total
  const size_t q_b = (size_t)n * 16, k_b = (size_t)n * 8, f_b = ((size_t)n * 4 + 15) & ~size_t(15);
  size_t sort_b = 0;
  cub::DeviceRadixSort::SortKeys(nullptr, sort_b, (const uint64_t *)nullptr, (uint64_t *)nullptr, (int)n, 0, 64, st);
  sort_b = (sort_b + 255) & ~size_t(255);
  Scratch s;
  s.st = st;
  const size_t total = q_b + 2 * k_b + f_b + k_b + 64 + sort_b;
  T2SC_CUDA(cudaMallocAsync(&s.p, total, st), "cascade scratch");
  uint8_t *b = (uint8_t *)s.p;
  int4 *q = (int4 *)b;
  uint64_t *keys_in = (uint64_t *)(b + q_b), *keys = (uint64_t *)(b + q_b + k_b);
  int32_t *flag = (int32_t *)(b + q_b + 2 * k_b);
  int64_t *pos = (int64_t *)(b + q_b + 2 * k_b + f_b);
  int *maxima = (int *)(b + q_b + 3 * k_b + f_b);
  int64_t *d_total = (int64_t *)(maxima + 4);
  void *sort_tmp = b + q_b + 3 * k_b + f_b + 64;
  for (int hr = resolution;; hr -= 128) {
    const int k = hr / 16;
    if (k <= 0) {
      err = "cascade_coords: the token budget was not met before hr_resolution reached 16";
      return T2SC_ERR_INVALID;
    }
    T2SC_CUDA(cudaMemsetAsync(maxima, 0, 16, st), "cascade memset");
    cascade_quant_kernel<<<nblocks(n, 256), 256, 0, st>>>((const int4 *)hr_coords, n, (float)lr_resolution,
                                                          (float)k, q, maxima, ctx->d_err);
    T2SC_LAUNCHED(ctx, "cascade_quant");
    int h[2] = {0, 0};
    T2SC_CUDA(cudaMemcpyAsync(h, maxima, 8, cudaMemcpyDeviceToHost, st), "cascade read-back");
    int flags = 0;
    int rc = read_dev_err(ctx, &flags);  // synchronises the stream (h is then valid)
    if (rc != T2SC_OK) return rc;
    if (flags & kDevErrRange) {
      err = "cascade_coords: coordinates must be non-negative";
      return T2SC_ERR_RANGE;
    }
    const uint64_t m = (uint64_t)h[0] + 1, bmax = (uint64_t)h[1];
    // every key below (bmax + 1) * m^3 must fit 64 bits
    const long double span = (long double)(bmax + 1) * (long double)m * (long double)m * (long double)m;
    if (span >= 18446744073709551615.0L) {
      err = "cascade_coords: quantised key range exceeds 64 bits";
      return T2SC_ERR_RANGE;
    }
    int end_bit = 1;
    while (end_bit < 64 && ((long double)((uint64_t)1 << end_bit)) < span) end_bit++;
    cascade_key_kernel<<<nblocks(n, 256), 256, 0, st>>>(q, n, m, keys_in);
    T2SC_LAUNCHED(ctx, "cascade_key");
    size_t tb = sort_b;
    T2SC_CUDA(cub::DeviceRadixSort::SortKeys(sort_tmp, tb, keys_in, keys, (int)n, 0, end_bit, st), "cascade sort");
    unique_flag_kernel<<<nblocks(n, 256), 256, 0, st>>>(keys, n, flag);
    T2SC_LAUNCHED(ctx, "cascade_unique");
    rc = scan_counts(ctx, flag, n, pos, d_total);
    if (rc != T2SC_OK) return rc;
    int64_t tokens = 0;
    T2SC_CUDA(cudaMemcpyAsync(&tokens, d_total, 8, cudaMemcpyDeviceToHost, st), "cascade read-back");
    T2SC_CUDA(cudaStreamSynchronize(st), "cascade read-back");
    if (tokens < max_num_tokens || hr == 1024) {
      cascade_emit_kernel<<<nblocks(n, 256), 256, 0, st>>>(keys, flag, pos, n, m, (int4 *)out_coords);
      T2SC_LAUNCHED(ctx, "cascade_emit");
      *num_tokens = tokens;
      *hr_resolution = hr;
      return T2SC_OK;
    }
  }
}

}  // namespace t2sc
