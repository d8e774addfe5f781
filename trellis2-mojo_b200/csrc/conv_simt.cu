// CUDA-core SubM conv used where the tensor-core kernel's shape rules do not
// hold (Ci % 8 != 0 or Co % 16 != 0) and, in this build, for the f32 mode.
// Output-stationary like the tensor-core kernel: a block owns 32 rows (in
// the map's sorted order, written back to their own positions) x 64
// output channels, stages each offset's 32 neighbour rows and the matching
// weight slice in shared memory, and accumulates with FMAs in f32 (k
// ascending, then input channel ascending).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "internal.h"

namespace t2sc {
namespace {

constexpr int kRows = 32, kCols = 64, kCiChunk = 32;

template <int DT>
__device__ __forceinline__ float load_el(const void *p, int64_t i) {
  if (DT == T2SC_DT_F32) return static_cast<const float *>(p)[i];
  if (DT == T2SC_DT_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
  return __half2float(static_cast<const __half *>(p)[i]);
}
template <int DT>
__device__ __forceinline__ void store_el(void *p, int64_t i, float v) {
  if (DT == T2SC_DT_F32)
    static_cast<float *>(p)[i] = v;
  else if (DT == T2SC_DT_BF16)
    static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
  else
    static_cast<__half *>(p)[i] = __float2half_rn(v);
}

template <int DT>
__global__ void __launch_bounds__(256) conv_simt_kernel(const void *__restrict__ x, void *__restrict__ y,
                                                        const void *__restrict__ res, const float *__restrict__ w,
                                                        const float *__restrict__ bias,
                                                        const int32_t *__restrict__ nbr_sorted,
                                                        const int32_t *__restrict__ perm, int64_t n_pad, int ci,
                                                        int co, int kvol, int flags) {
  __shared__ float xs[kRows][kCiChunk + 1];
  __shared__ float ws[kCiChunk][kCols];
  __shared__ int32_t srcs[kRows];
  const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;  // 64 x 4
  const int64_t r0 = (int64_t)blockIdx.x * kRows;
  const int o = blockIdx.y * kCols + tx;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; i++) acc[i] = 0.f;
  for (int k = 0; k < kvol; k++) {
    __syncthreads();
    if (threadIdx.x < kRows) {
      srcs[threadIdx.x] = nbr_sorted[(int64_t)k * n_pad + r0 + threadIdx.x];
    }
    __syncthreads();
    for (int c0 = 0; c0 < ci; c0 += kCiChunk) {
      for (int e = threadIdx.x; e < kRows * kCiChunk; e += 256) {
        const int rr = e / kCiChunk, cc = e % kCiChunk;
        const int32_t s = srcs[rr];
        xs[rr][cc] = (s >= 0 && c0 + cc < ci) ? load_el<DT>(x, (int64_t)s * ci + c0 + cc) : 0.f;
      }
      for (int e = threadIdx.x; e < kCiChunk * kCols; e += 256) {
        const int cc = e / kCols, oo = e % kCols;
        const int oc = blockIdx.y * kCols + oo;
        ws[cc][oo] = (c0 + cc < ci && oc < co) ? w[((int64_t)k * ci + c0 + cc) * co + oc] : 0.f;
      }
      __syncthreads();
#pragma unroll 4
      for (int cc = 0; cc < kCiChunk; cc++) {
        const float wv = ws[cc][tx];
#pragma unroll
        for (int i = 0; i < 8; i++) acc[i] = fmaf(xs[ty + 4 * i][cc], wv, acc[i]);
      }
      __syncthreads();
    }
  }
  if (o >= co) return;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const int64_t r = perm[r0 + ty + 4 * i];  // sorted position -> output row
    if (r < 0) continue;
    float v = acc[i] + bias[o];
    if (flags & T2SC_SILU) v = v / (1.0f + expf(-v));
    if (flags & T2SC_RESIDUAL) v += load_el<DT>(res, r * co + o);
    store_el<DT>(y, r * co + o, v);
  }
}

}  // namespace

int conv_simt_prepare(t2sc_conv *cv, const float *w, std::string &err) {
  const int co = cv->co, ci = cv->ci, K = cv->kvol;
  std::vector<float> t((size_t)K * ci * co);
  for (int o = 0; o < co; o++)
    for (int k = 0; k < K; k++)
      for (int i = 0; i < ci; i++) t[((size_t)k * ci + i) * co + o] = w[((size_t)o * K + k) * ci + i];
  if (cv->dtype != T2SC_DT_F32) {
    // the 16-bit modes compute with the 16-bit-rounded weights
    for (auto &v : t) {
      if (cv->dtype == T2SC_DT_BF16)
        v = __bfloat162float(__float2bfloat16_rn(v));
      else
        v = __half2float(__float2half_rn(v));
    }
  }
  T2SC_CUDA(cudaMalloc((void **)&cv->d_w_simt, t.size() * sizeof(float)), "simt weights");
  T2SC_CUDA(cudaMemcpy(cv->d_w_simt, t.data(), t.size() * sizeof(float), cudaMemcpyHostToDevice), "simt weights");
  return T2SC_OK;
}

int conv_simt_launch(t2sc_conv *cv, t2sc_map *m, const void *x, void *y, int flags, const void *residual,
                     std::string &err) {
  if (m->n == 0) return T2SC_OK;
  // rows in the map's sorted order (n_pad is a multiple of the 32-row block)
  dim3 grid((unsigned)(m->n_pad / kRows), (unsigned)((cv->co + kCols - 1) / kCols));
  cudaStream_t st = cv->ctx->stream;
  switch (cv->dtype) {
    case T2SC_DT_F32:
      conv_simt_kernel<T2SC_DT_F32><<<grid, 256, 0, st>>>(x, y, residual, cv->d_w_simt, cv->d_bias, m->nbr_sorted, m->perm,
                                                          m->n_pad,
                                                          cv->ci, cv->co, cv->kvol, flags);
      break;
    case T2SC_DT_BF16:
      conv_simt_kernel<T2SC_DT_BF16><<<grid, 256, 0, st>>>(x, y, residual, cv->d_w_simt, cv->d_bias, m->nbr_sorted, m->perm,
                                                          m->n_pad,
                                                           cv->ci, cv->co, cv->kvol, flags);
      break;
    default:
      conv_simt_kernel<T2SC_DT_F16><<<grid, 256, 0, st>>>(x, y, residual, cv->d_w_simt, cv->d_bias, m->nbr_sorted, m->perm,
                                                          m->n_pad,
                                                          cv->ci, cv->co, cv->kvol, flags);
  }
  T2SC_LAUNCHED(cv->ctx, "conv_simt");
  return T2SC_OK;
}

}  // namespace t2sc
